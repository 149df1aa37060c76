"""Attention backward (jules_flash_attention_bwd): dQ, dK, dV from the
forward's O and lse.

The reference has no attention gradient, so the oracle restates the exact
gradient of the forward in double (oracle/restate.c orc_attention_bwd); it
is pinned here against torch autograd through scaled_dot_product_attention
in float64.  The GPU paths (tcgen05 for bf16 head_dim 128, CUDA cores for
fp32 and other head dims) are compared with the oracle on the same inputs:
bf16 within max-abs 2e-2 (relative to the gradient's scale) and rel-L2 5e-3,
fp32 within rel-L2 1e-5."""
import ctypes

import numpy as np
import pytest

from conftest import BF16_MAX_ABS, BF16_REL_L2, max_abs, rel_l2

JULES_ERR_SHAPE, JULES_ERR_DTYPE, JULES_ERR_ARG, JULES_ERR_WORKSPACE = 1, 3, 6, 8
F32_BWD_REL_L2 = 1e-5


def _oracle():
    import oracle
    return oracle.Restated()


def _inputs(B, Hq, Hkv, S, D, seed):
    g = np.random.default_rng(seed)
    Q = g.standard_normal((B, Hq, S, D)).astype(np.float32)
    K = g.standard_normal((B, Hkv, S, D)).astype(np.float32)
    V = g.standard_normal((B, Hkv, S, D)).astype(np.float32)
    dO = g.standard_normal((B, Hq, S, D)).astype(np.float32)
    return Q, K, V, dO


@pytest.mark.parametrize("B,Hq,Hkv,S,D,causal", [(1, 2, 2, 77, 64, False), (2, 4, 2, 130, 32, True),
                                                 (1, 2, 1, 200, 128, True), (1, 1, 1, 1, 16, False)])
def test_oracle_attention_bwd_matches_torch_autograd(B, Hq, Hkv, S, D, causal):
    import torch
    Q, K, V, dO = _inputs(B, Hq, Hkv, S, D, S + D)
    dq, dk, dv = _oracle().attention_bwd(Q, K, V, dO, causal)
    q, k, v = (torch.from_numpy(x).double().requires_grad_() for x in (Q, K, V))
    rep = Hq // Hkv
    o = torch.nn.functional.scaled_dot_product_attention(
        q, k.repeat_interleave(rep, dim=1), v.repeat_interleave(rep, dim=1), is_causal=causal)
    o.backward(torch.from_numpy(dO).double())
    for ours, ref in ((dq, q.grad), (dk, k.grad), (dv, v.grad)):
        assert rel_l2(ours, ref.numpy()) <= 1e-6


def test_attention_bwd_argument_errors(jb):
    L = jb.lib()
    p = ctypes.c_void_p(256)  # never dereferenced: the checks come first
    f = ctypes.cast(p, ctypes.c_void_p)
    need = L.jules_flash_attention_bwd_workspace_bytes(1, 2, 300, 128, jb.DT_BF16)
    assert need == 2 * 2 * 384 * 4  # lse2 and delta, padded to whole 128-row tiles
    args = [p] * 5 + [f] + [p] * 3
    assert L.jules_flash_attention_bwd(*args, 1, 2, 2, 300, 128, 0.0, 1, jb.DT_BF16, p, need - 16, None) == JULES_ERR_WORKSPACE
    assert L.jules_flash_attention_bwd(*args, 1, 3, 2, 300, 128, 0.0, 1, jb.DT_BF16, p, need, None) == JULES_ERR_SHAPE
    assert L.jules_flash_attention_bwd(*args, 1, 2, 2, 300, 512, 0.0, 1, jb.DT_BF16, p, need, None) == JULES_ERR_SHAPE
    assert L.jules_flash_attention_bwd(*args, 1, 2, 2, 300, 128, 0.0, 1, 2, p, need, None) == JULES_ERR_DTYPE
    assert L.jules_flash_attention_bwd(None, *args[1:], 1, 2, 2, 300, 128, 0.0, 1, jb.DT_BF16, p, need, None) == JULES_ERR_ARG


def _run_gpu(jb, Q, K, V, dO, causal, dtype):
    import torch
    t = lambda a: torch.from_numpy(a).cuda().to(dtype)
    q, k, v, do = t(Q), t(K), t(V), t(dO)
    O, lse = jb.flash_attention_fwd(q, k, v, causal=causal)
    dq, dk, dv = jb.flash_attention_bwd(q, k, v, O, do, lse, causal=causal)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    # the oracle sees exactly the values the GPU saw
    rounded = [x.float().cpu().numpy() for x in (q, k, v, do)]
    return [x.float().cpu().numpy() for x in (dq, dk, dv)], rounded


def _check_bf16(got, want):
    for g, w in zip(got, want):
        if not np.abs(w).max() > 0:
            # an exactly-zero gradient (e.g. dQ with one key: dS = dP - D = 0)
            # has no relative error; the GPU's rounding residue must be tiny
            assert max_abs(g, w) <= 1e-4
            continue
        assert rel_l2(g, w) <= BF16_REL_L2
        assert max_abs(g, w) <= BF16_MAX_ABS * max(1.0, float(np.abs(w).max()))


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hkv,S,causal", [(1, 2, 2, 256, False), (1, 2, 2, 256, True),
                                               (2, 4, 2, 300, True), (1, 8, 1, 130, False),
                                               (1, 1, 1, 1, True), (1, 2, 2, 1000, True),
                                               (1, 2, 1, 517, False)])
def test_attention_bwd_tensor_cores_bf16(jb, B, Hq, Hkv, S, causal):
    """bf16, head_dim 128: the tcgen05 kernels (ragged S, grouped-query heads,
    causal diagonal tiles)."""
    import torch
    Q, K, V, dO = _inputs(B, Hq, Hkv, S, 128, 3 * S + Hq)
    got, (q, k, v, do) = _run_gpu(jb, Q, K, V, dO, causal, torch.bfloat16)
    _check_bf16(got, _oracle().attention_bwd(q, k, v, do, causal))


@pytest.mark.gpu
@pytest.mark.parametrize("B,Hq,Hkv,S,D,causal", [(1, 2, 2, 100, 64, True), (2, 4, 1, 65, 128, False),
                                                 (1, 2, 2, 33, 200, True)])
def test_attention_bwd_cuda_cores_fp32(jb, B, Hq, Hkv, S, D, causal):
    import torch
    Q, K, V, dO = _inputs(B, Hq, Hkv, S, D, S * D)
    got, (q, k, v, do) = _run_gpu(jb, Q, K, V, dO, causal, torch.float32)
    want = _oracle().attention_bwd(q, k, v, do, causal)
    for g, w in zip(got, want):
        assert rel_l2(g, w) <= F32_BWD_REL_L2 if np.abs(w).max() > 0 else max_abs(g, w) <= 1e-6


@pytest.mark.gpu
def test_attention_bwd_cuda_cores_bf16_other_head_dim(jb):
    import torch
    Q, K, V, dO = _inputs(1, 4, 2, 150, 64, 5)
    got, (q, k, v, do) = _run_gpu(jb, Q, K, V, dO, True, torch.bfloat16)
    _check_bf16(got, _oracle().attention_bwd(q, k, v, do, True))


@pytest.mark.gpu
def test_attention_bwd_deterministic_and_autograd(jb):
    """Two runs give identical bits (no atomics); jb.attention's autograd
    backward is the same computation."""
    import torch
    Q, K, V, dO = _inputs(2, 4, 2, 384, 128, 9)
    q, k, v, do = (torch.from_numpy(a).cuda().to(torch.bfloat16) for a in (Q, K, V, dO))
    O, lse = jb.flash_attention_fwd(q, k, v, causal=True)
    r1 = jb.flash_attention_bwd(q, k, v, O, do, lse, causal=True)
    r2 = jb.flash_attention_bwd(q, k, v, O, do, lse, causal=True)
    assert all(torch.equal(a, b) for a, b in zip(r1, r2))
    qa, ka, va = (x.clone().requires_grad_() for x in (q, k, v))
    out = jb.attention(qa, ka, va, causal=True)
    assert torch.equal(out, O)
    out.backward(do)
    assert torch.equal(qa.grad, r1[0]) and torch.equal(ka.grad, r1[1]) and torch.equal(va.grad, r1[2])


@pytest.mark.gpu
def test_attention_bwd_long_sequence_sampled(jb):
    """A longer causal case (S = 4096, the C3 sequence length) on one head
    pair against the oracle."""
    import torch
    Q, K, V, dO = _inputs(1, 2, 1, 4096, 128, 41)
    got, (q, k, v, do) = _run_gpu(jb, Q, K, V, dO, True, torch.bfloat16)
    _check_bf16(got, _oracle().attention_bwd(q, k, v, do, True))


@pytest.mark.gpu
def test_attention_bwd_unaligned_bf16_falls_back(jb):
    """bf16 head_dim 128 with buffers off 16-byte alignment: the CUDA-core
    path (as the forward), same results bar."""
    import torch
    B, Hq, Hkv, S, D = 1, 2, 1, 96, 128

    def off(a):  # a copy of `a` whose storage starts 2 bytes past an aligned address
        buf = torch.empty(a.size + 8, dtype=torch.bfloat16, device="cuda")
        t = buf[1:1 + a.size].view(a.shape)
        t.copy_(torch.from_numpy(a).to(torch.bfloat16))
        assert t.data_ptr() % 16 != 0
        return t
    Q, K, V, dO = _inputs(B, Hq, Hkv, S, D, 17)
    q, k, v, do = off(Q), off(K), off(V), off(dO)
    O, lse = jb.flash_attention_fwd(q, k, v, causal=True)
    dq, dk, dv = jb.flash_attention_bwd(q, k, v, O, do, lse, causal=True)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = _oracle().attention_bwd(*(x.float().cpu().numpy() for x in (q, k, v, do)), causal=True)
    _check_bf16([x.float().cpu().numpy() for x in (dq, dk, dv)], want)
