"""jules_custom_call: the extern_kernel name -> kernel dispatch a runtime's
custom-call handler uses (buffers + one jules_call_desc as opaque bytes).
Argument checks run on CPU; on the GPU every routed name must give exactly the
result of the direct entry point."""
import ctypes

import numpy as np
import pytest

from conftest import F32_REL_L2, rel_l2
from helpers import arg_buffer

JULES_ERR_ARG, JULES_ERR_UNSUPPORTED = 6, 7


def _raw_call(jb, name, n_buffers=2, opaque_len=None):
    d = jb.CallDesc()
    fake = arg_buffer().value  # the calls fail validation before any launch
    bufs = (ctypes.c_void_p * n_buffers)(*([fake] * n_buffers))
    return jb.lib().jules_custom_call(name.encode(), None, bufs, n_buffers,
                                      ctypes.cast(ctypes.pointer(d), ctypes.c_void_p),
                                      ctypes.sizeof(d) if opaque_len is None else opaque_len)


def test_custom_call_argument_errors(jb):
    assert _raw_call(jb, "noSuchKernel") == JULES_ERR_ARG
    assert _raw_call(jb, "matmulInt8", n_buffers=2) == JULES_ERR_ARG
    assert _raw_call(jb, "fusedSoftmax", opaque_len=8) == JULES_ERR_ARG
    assert _raw_call(jb, "fusedSoftmax", n_buffers=3) == JULES_ERR_ARG
    assert _raw_call(jb, "fusedMatmulBiasGelu", n_buffers=3) == JULES_ERR_ARG
    assert _raw_call(jb, "flashAttention", n_buffers=3) == JULES_ERR_ARG
    assert ctypes.sizeof(jb.CallDesc) == 6 * 8 + 2 * 4 + 2 * 4


@pytest.mark.gpu
def test_custom_call_matches_direct_entry_points(jb):
    import torch
    g = torch.Generator(device="cuda").manual_seed(11)
    dev = "cuda"
    bf, f32 = torch.bfloat16, torch.float32
    # fusedMatmulGelu (bf16) and fusedMatmulBiasRelu (f32 in/out)
    M, N, K = 300, 512, 256
    A = (torch.randn((M, K), generator=g, device=dev) / 16).to(bf)
    W = (torch.randn((K, N), generator=g, device=dev) / 16).to(bf)
    bias = torch.randn(N, generator=g, device=dev) * 0.1
    C = torch.empty((M, N), dtype=bf, device=dev)
    jb.custom_call("fusedMatmulGelu", [A, W, C], dims=(M, N, K), dtype=jb.DT_BF16)
    assert torch.equal(C, jb.gemm_bias_act(A, W, act="gelu"))
    C32 = torch.empty((M, N), dtype=f32, device=dev)
    jb.custom_call("fusedMatmulBiasGelu", [A, W, bias, C32], dims=(M, N, K), dtype=jb.DT_BF16,
                   flags=1)
    assert torch.equal(C32, jb.gemm_bias_act(A, W, bias, act="gelu", out_dtype=f32))
    Af, Wf = A.float(), W.float()
    Cf = torch.empty((M, N), dtype=f32, device=dev)
    jb.custom_call("fusedMatmulBiasRelu", [Af, Wf, bias, Cf], dims=(M, N, K), dtype=jb.DT_F32)
    assert torch.equal(Cf, jb.gemm_bias_act(Af, Wf, bias, act="relu"))
    # blasMatmul with transposed B: C = 0.5 * A . B^T
    Bt = torch.randn((N, K), generator=g, device=dev)
    Cb = torch.empty((M, N), dtype=f32, device=dev)
    jb.custom_call("blasMatmul", [Af, Bt, Cb], dims=(M, N, K), fparams=(0.5, 0.0),
                   dtype=jb.DT_F32, flags=2)
    assert rel_l2(Cb.cpu().numpy(), (0.5 * Af @ Bt.T).cpu().numpy()) <= F32_REL_L2
    # fusedLayerNorm: the routed form (no affine) and the affine form
    X = torch.randn((64, 1000), generator=g, device=dev)
    gam, bet = 1 + 0.1 * torch.randn(1000, generator=g, device=dev), 0.1 * torch.randn(1000, generator=g, device=dev)
    Y2 = torch.empty_like(X)
    jb.custom_call("fusedLayerNorm", [X, Y2], dims=(64, 1000), dtype=jb.DT_F32)
    want = torch.nn.functional.layer_norm(X, (1000,), eps=1e-5)
    assert rel_l2(Y2.cpu().numpy(), want.cpu().numpy()) <= F32_REL_L2
    Y4 = torch.empty_like(X)
    jb.custom_call("fusedLayerNorm", [X, gam, bet, Y4], dims=(64, 1000), fparams=(1e-5,),
                   dtype=jb.DT_F32)
    assert torch.equal(Y4, jb.layernorm(X, gam, bet))
    # fusedGelu, fusedSoftmax
    Yg = torch.empty_like(X)
    jb.custom_call("fusedGelu", [X, Yg], dims=(X.numel(),), dtype=jb.DT_F32)
    assert torch.equal(Yg, jb.gelu(X))
    Ys = torch.empty_like(X)
    jb.custom_call("fusedSoftmax", [X, Ys], dims=(64, 1000), dtype=jb.DT_F32)
    assert torch.equal(Ys, jb.softmax(X))
    # fusedCrossEntropyLoss, with and without the gradient
    T = torch.randint(0, 1000, (64,), generator=g, device=dev, dtype=torch.int32)
    loss, grad = torch.empty((), dtype=f32, device=dev), torch.empty_like(X)
    jb.custom_call("fusedCrossEntropyLoss", [X, T, grad, loss], dims=(64, 1000), dtype=jb.DT_F32)
    l_ref, g_ref = jb.cross_entropy_loss(X, T)
    assert torch.equal(grad, g_ref)
    assert abs(float(loss) - float(l_ref)) <= 1e-6 * abs(float(l_ref))
    loss2 = torch.empty((), dtype=f32, device=dev)
    jb.custom_call("fusedCrossEntropyLoss", [X, T, loss2], dims=(64, 1000), dtype=jb.DT_F32)
    assert abs(float(loss2) - float(l_ref)) <= 1e-6 * abs(float(l_ref))
    # flashAttention: causal, grouped-query, with lse
    B, Hq, Hkv, S, D = 1, 4, 2, 300, 128
    Q = torch.randn((B, Hq, S, D), generator=g, device=dev).to(bf)
    Kt = torch.randn((B, Hkv, S, D), generator=g, device=dev).to(bf)
    V = torch.randn((B, Hkv, S, D), generator=g, device=dev).to(bf)
    O, L = torch.empty_like(Q), torch.empty((B, Hq, S), dtype=f32, device=dev)
    jb.custom_call("flashAttention", [Q, Kt, V, O, L], dims=(B, Hq, Hkv, S, D), dtype=jb.DT_BF16,
                   flags=1)
    O_ref, L_ref = jb.flash_attention_fwd(Q, Kt, V, causal=True)
    assert torch.equal(O, O_ref) and torch.equal(L, L_ref)
    # fusedMLPForward (runs without allocation)
    Tn, d, dff = 128, 256, 1024
    Xm = torch.randn((Tn, d), generator=g, device=dev).to(bf)
    gm, bm = 1 + 0.02 * torch.randn(d, generator=g, device=dev), 0.02 * torch.randn(d, generator=g, device=dev)
    W1 = (0.02 * torch.randn((d, dff), generator=g, device=dev)).to(bf)
    b1 = 0.02 * torch.randn(dff, generator=g, device=dev)
    W2 = (0.02 * torch.randn((dff, d), generator=g, device=dev)).to(bf)
    b2 = 0.02 * torch.randn(d, generator=g, device=dev)
    Om = torch.empty((Tn, d), dtype=f32, device=dev)
    jb.custom_call("fusedMLPForward", [Xm, gm, bm, W1, b1, W2, b2, Om], dims=(Tn, d, dff),
                   fparams=(1e-5,), dtype=jb.DT_BF16, flags=1)
    assert torch.equal(Om, jb.mlp_block(Xm, gm, bm, W1, b1, W2, b2, out_dtype=f32))
    # matmulInt8 with bias
    Ai = torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
    Bi = torch.randint(-128, 128, (K, N), generator=g, device=dev, dtype=torch.int8)
    Ci = torch.empty((M, N), dtype=f32, device=dev)
    jb.custom_call("matmulInt8", [Ai, Bi, bias, Ci], dims=(M, N, K), fparams=(0.01, 0.02))
    assert torch.equal(Ci, jb.matmul_int8(Ai, Bi, 0.01, 0.02, bias))
    torch.cuda.synchronize()
    assert jb.device_error() == 0
