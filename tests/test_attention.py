"""Flash-attention forward: CUDA kernels vs the oracle.

fp32 (config C1) against the reference's own flashAttention compiled from
source (oracle/_ref); bf16 tcgen05 kernel (causal, grouped-query, lse)
against the C restatement on the same bf16 values."""
import numpy as np
import pytest

from conftest import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, max_abs, rel_l2
from helpers import attn_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


def _gpu_attn(jb, Q, K, V, causal, dtype="bf16"):
    import torch
    O, lse = jb.flash_attention_fwd(to_dev(Q, dtype), to_dev(K, dtype), to_dev(V, dtype),
                                    causal=causal)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    return to_np(O), lse.cpu().numpy()


def test_attention_fp32_config_c1_vs_reference(jb, ref, orc):
    """Config C1: [1,8,512,64] fp32, non-causal, scale 1/sqrt(64)."""
    Q, K, V = attn_inputs(1, 8, 8, 512, 64, seed=1, bf16=False)
    want = ref.flash_attention(Q, K, V)
    got, lse = _gpu_attn(jb, Q, K, V, False, "f32")
    assert rel_l2(got, want) <= F32_REL_L2
    _, lse_want = orc.flash_attention(Q, K, V, causal=False)
    assert max_abs(lse, lse_want) <= 1e-4


@pytest.mark.parametrize("S,D", [(1, 64), (100, 32), (77, 128), (256, 96)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_fp32_shapes(jb, orc, S, D, causal):
    Q, K, V = attn_inputs(2, 3, 3, S, D, seed=S + D, bf16=False)
    want, lse_want = orc.flash_attention(Q, K, V, causal=causal)
    got, lse = _gpu_attn(jb, Q, K, V, causal, "f32")
    assert rel_l2(got, want) <= F32_REL_L2
    assert max_abs(lse, lse_want) <= 1e-4


@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 2, 2, 128), (1, 2, 2, 256), (2, 4, 4, 384),
                                        (1, 2, 2, 200), (1, 3, 3, 333), (1, 8, 2, 384),
                                        (1, 1, 1, 1), (1, 4, 1, 129)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_bf16_tc(jb, orc, B, Hq, Hkv, S, causal):
    Q, K, V = attn_inputs(B, Hq, Hkv, S, 128, seed=B * 100 + S)
    want, lse_want = orc.flash_attention(Q, K, V, causal=causal)
    got, lse = _gpu_attn(jb, Q, K, V, causal)
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2
    assert max_abs(lse, lse_want) <= 2e-3


@pytest.mark.parametrize("D", [64, 96])
def test_attention_bf16_other_head_dims(jb, orc, D):
    Q, K, V = attn_inputs(1, 4, 2, 300, D, seed=D)
    want, lse_want = orc.flash_attention(Q, K, V, causal=True)
    got, lse = _gpu_attn(jb, Q, K, V, True)
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2


def _sampled_check(jb, orc, B, Hq, Hkv, S, units, q_windows, seed, every_row=False):
    """Full-size run on the GPU; oracle on sampled (b, h) units and query
    windows (inputs generated on the GPU, sampled slices copied back).
    every_row: also every row of every head against a plain fp32 torch
    computation of softmax(scale Q K^T, causal) V (no tf32)."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    D = 128
    Q = torch.randn((B, Hq, S, D), generator=g, device="cuda").to(torch.bfloat16)
    K = torch.randn((B, Hkv, S, D), generator=g, device="cuda").to(torch.bfloat16)
    V = torch.randn((B, Hkv, S, D), generator=g, device="cuda").to(torch.bfloat16)
    O, lse = jb.flash_attention_fwd(Q, K, V, causal=True)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    group = Hq // Hkv
    for u in units:
        b, h = divmod(u, Hq)
        hk = h // group
        q = to_np(Q[b, h])[None, None]
        k = to_np(K[b, hk])[None, None]
        v = to_np(V[b, hk])[None, None]
        for (q0, q1) in q_windows:
            want, lw = orc.flash_attention(q, k, v, causal=True, q_begin=q0, q_end=q1)
            got = to_np(O[b, h, q0:q1])
            assert max_abs(got, want[0, 0, q0:q1]) <= BF16_MAX_ABS
            assert rel_l2(got, want[0, 0, q0:q1]) <= BF16_REL_L2
            assert max_abs(lse[b, h, q0:q1].cpu().numpy(), lw[0, 0, q0:q1]) <= 2e-3
    # Size-independent property over every row: softmax weights sum to one,
    # so each output row lies inside the convex hull of V; in particular
    # |O| <= max |V| per column.
    vmax = V.float().abs().amax(dim=2, keepdim=True)  # [B,Hkv,1,D]
    vmax = vmax.repeat_interleave(group, dim=1)
    assert bool((O.float().abs() <= vmax * (1 + 1e-2) + 1e-2).all())
    assert bool(torch.isfinite(lse).all())
    if every_row:
        prev = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            mask = torch.triu(torch.full((S, S), float("-inf"), device="cuda"), 1)
            err2 = ref2 = 0.0
            worst = 0.0
            for b in range(B):
                for h0 in range(0, Hq, 4):
                    hs = slice(h0, h0 + 4)
                    q = Q[b, hs].float()
                    kk = K[b, [h // group for h in range(h0, h0 + 4)]].float()
                    vv = V[b, [h // group for h in range(h0, h0 + 4)]].float()
                    sc = q @ kk.transpose(-1, -2) / D ** 0.5 + mask
                    want = torch.softmax(sc, -1) @ vv
                    got = O[b, hs].float()
                    worst = max(worst, float((got - want).abs().max()))
                    err2 += float(((got - want) ** 2).sum())
                    ref2 += float((want ** 2).sum())
                    lw = torch.logsumexp(sc, -1)
                    assert float((lse[b, hs] - lw).abs().max()) <= 2e-3
            assert worst <= BF16_MAX_ABS
            assert (err2 / ref2) ** 0.5 <= BF16_REL_L2
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.slow
def test_attention_config_c3_sampled(jb, orc):
    """Config C3: [8,32,4096,128] causal bf16 + lse."""
    _sampled_check(jb, orc, 8, 32, 32, 4096, units=[0, 37, 100, 163, 200, 255],
                   q_windows=[(0, 130), (1024, 1152), (2000, 2100), (3968, 4096)], seed=3,
                   every_row=True)


@pytest.mark.slow
def test_attention_config_c5_sampled(jb, orc):
    """Config C5: [4, Hq=64, Hkv=8, 16384, 128] causal bf16 (grouped-query)."""
    _sampled_check(jb, orc, 4, 64, 8, 16384, units=[0, 71, 100, 190, 255],
                   q_windows=[(16256, 16384), (5000, 5064), (0, 64), (9000, 9128)], seed=5)


# --- fp16 operands and head dim 64 on tcgen05 ------------------------------
@pytest.mark.parametrize("D", [128, 64])
@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 2, 2, 256), (1, 8, 2, 384), (1, 3, 3, 333), (1, 4, 1, 129)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_f16_tc(jb, orc, D, B, Hq, Hkv, S, causal):
    from helpers import f16_np
    Q, K, V = (f16_np(x) for x in attn_inputs(B, Hq, Hkv, S, D, seed=B * 7 + S + D, bf16=False))
    want, lse_want = orc.flash_attention(Q, K, V, causal=causal)
    got, lse = _gpu_attn(jb, Q, K, V, causal, "f16")
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2
    assert max_abs(lse, lse_want) <= 2e-3


@pytest.mark.parametrize("B,Hq,Hkv,S", [(1, 2, 2, 128), (2, 4, 4, 384), (1, 8, 2, 300),
                                        (4, 4, 4, 512), (1, 1, 1, 1)])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_bf16_d64_tc(jb, orc, B, Hq, Hkv, S, causal):
    """Head dim 64 (the reference benchmark's shapes, benchmarks/bench_kernel.cpp:509-512)
    on the tensor-core kernel."""
    Q, K, V = attn_inputs(B, Hq, Hkv, S, 64, seed=B * 100 + S + 64)
    want, lse_want = orc.flash_attention(Q, K, V, causal=causal)
    got, lse = _gpu_attn(jb, Q, K, V, causal)
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2
    assert max_abs(lse, lse_want) <= 2e-3


def test_attention_f16_other_head_dims(jb, orc):
    """fp16 with head dim 96: the CUDA-core kernel."""
    from helpers import f16_np
    Q, K, V = (f16_np(x) for x in attn_inputs(1, 4, 2, 200, 96, seed=96, bf16=False))
    want, _ = orc.flash_attention(Q, K, V, causal=True)
    got, _ = _gpu_attn(jb, Q, K, V, True, "f16")
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2
