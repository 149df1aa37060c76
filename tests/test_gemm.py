"""Fused GEMM + bias + activation (+ residual): CUDA kernels vs the oracle.

bf16 tensor-core path (tcgen05) against the C restatement of
tiledMatmulWithActivation / fusedMatmulBiasRelu on the same bf16 values;
fp32 CUDA-core path against the reference's own kernels (oracle/_ref)."""
import numpy as np
import pytest

from conftest import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, max_abs, rel_l2
from helpers import bf16_np, gemm_inputs, to_dev, to_np

pytestmark = pytest.mark.gpu


def _run_bf16(jb, A, W, b, act, residual=None):
    import torch
    r = to_dev(residual) if residual is not None else None
    bias = torch.from_numpy(b).cuda() if b is not None else None
    C = jb.gemm_bias_act(to_dev(A), to_dev(W), bias, r, act=act)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    return to_np(C)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (129, 264, 72), (1, 8, 8),
                                   (300, 520, 136), (640, 1024, 1024)])
@pytest.mark.parametrize("act", ["none", "gelu"])
def test_gemm_tc_shapes(jb, orc, M, N, K, act):
    A, W, b = gemm_inputs(M, N, K, seed=M + N + K)
    got = _run_bf16(jb, A, W, b, act)
    want = orc.gemm_bias_act(A, W, b, None, act)
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2


@pytest.mark.parametrize("act", ["relu", "sigmoid", "tanh"])
def test_gemm_tc_activations(jb, orc, act):
    A, W, b = gemm_inputs(256, 512, 320, seed=7)
    got = _run_bf16(jb, A, W, b, act)
    want = orc.gemm_bias_act(A, W, b, None, act)
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2


@pytest.mark.parametrize("act", ["none", "gelu"])
def test_gemm_tc_fp32_output(jb, orc, act):
    """bf16 operands, fp32 result (the cast back to an fp32 caller's type)."""
    import torch
    A, W, b = gemm_inputs(320, 640, 448, seed=13)
    R = bf16_np(np.random.default_rng(14).standard_normal((320, 640)).astype(np.float32))
    got = jb.gemm_bias_act(to_dev(A), to_dev(W), torch.from_numpy(b).cuda(), to_dev(R), act=act,
                           out_dtype=torch.float32)
    got16 = jb.gemm_bias_act(to_dev(A), to_dev(W), torch.from_numpy(b).cuda(), to_dev(R), act=act)
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    want = orc.gemm_bias_act(A, W, b, R, act)
    assert max_abs(to_np(got), want) <= 2e-3
    assert rel_l2(to_np(got), want) <= 1e-3
    assert torch.equal(got16, got.to(torch.bfloat16))


@pytest.mark.parametrize("M,N,K", [(2560, 2048, 520), (2560, 2048, 136), (4096, 4096, 1024)])
@pytest.mark.parametrize("out", ["bf16", "f32"])
def test_gemm_tc_split_tail(jb, orc, M, N, K, out):
    """Shapes whose last round of 256x256 tiles is split in two along K
    (80 tiles on 74 CTA pairs; 256 tiles); odd and even k-block counts."""
    import torch
    A, W, b = gemm_inputs(M, N, K, seed=M + K)
    R = bf16_np(np.random.default_rng(K).standard_normal((M, N)).astype(np.float32))
    od = torch.float32 if out == "f32" else torch.bfloat16
    for _ in range(2):  # second call reuses the scratch counters
        got = jb.gemm_bias_act(to_dev(A), to_dev(W), torch.from_numpy(b).cuda(), to_dev(R),
                               act="gelu", out_dtype=od)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    rows = np.concatenate([np.arange(0, M, 97), [M - 1]])
    want = orc.gemm_bias_act(np.ascontiguousarray(A[rows]), W, b, np.ascontiguousarray(R[rows]),
                             "gelu")
    g = to_np(got[torch.from_numpy(rows).cuda()])
    assert max_abs(g, want) <= BF16_MAX_ABS
    assert rel_l2(g, want) <= BF16_REL_L2


def test_gemm_tc_no_bias_residual(jb, orc):
    A, W, _ = gemm_inputs(384, 768, 512, seed=3, bias=False)
    R = bf16_np(np.random.default_rng(4).standard_normal((384, 768)).astype(np.float32))
    got = _run_bf16(jb, A, W, None, "none", residual=R)
    want = orc.gemm_bias_act(A, W, None, R, "none")
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2


def test_gemm_tc_config_c2_sampled(jb, orc):
    """Config C2 at full size (4096^3, bias + GELU); 256 rows checked
    against the oracle, all rows through a size-independent property."""
    import torch
    M = N = K = 4096
    A, W, b = gemm_inputs(M, N, K, seed=20260)
    dA, dW = to_dev(A), to_dev(W)
    bias = torch.from_numpy(b).cuda()
    C = jb.gemm_bias_act(dA, dW, bias, act="gelu")
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    rows = np.linspace(0, M - 1, 256).astype(np.int64)
    got = to_np(C[torch.from_numpy(rows).cuda()])
    want = orc.gemm_bias_act(np.ascontiguousarray(A[rows]), W, b, None, "gelu")
    assert max_abs(got, want) <= BF16_MAX_ABS
    assert rel_l2(got, want) <= BF16_REL_L2
    # Scaling A by 2 is exact in bf16 and fp32: the no-activation product must
    # double bit-exactly in every row.
    C1 = jb.gemm_bias_act(dA, dW, act="none")
    C2 = jb.gemm_bias_act(dA * 2, dW, act="none")
    torch.cuda.synchronize()
    assert torch.equal(C2, C1 * 2)


@pytest.mark.parametrize("M,N,K", [(64, 96, 80), (33, 17, 129), (256, 256, 256)])
@pytest.mark.parametrize("act", ["none", "relu", "gelu"])
def test_gemm_fp32_vs_reference(jb, ref, M, N, K, act):
    """fp32 CUDA-core path vs the reference's own tiled kernel."""
    import torch
    g = np.random.default_rng(M * 7 + K)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    W = g.uniform(-1, 1, (K, N)).astype(np.float32)
    want = ref.tiled_matmul_act(A, W, act)
    got = jb.gemm_bias_act(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), act=act)
    assert rel_l2(to_np(got), want) <= F32_REL_L2


@pytest.mark.parametrize("M,N,K", [(256, 256, 256), (512, 768, 1000), (300, 264, 4096)])
@pytest.mark.parametrize("act", ["none", "gelu"])
def test_gemm_f32_tc_vs_reference(jb, ref, M, N, K, act):
    """3xTF32 tensor-core fp32 GEMM vs the reference's own tiled kernel, at
    the fp32 bar (rel-L2 1e-5); ragged K (3K not a multiple of the 32-wide
    k-block) and partial tiles included."""
    import torch
    g = np.random.default_rng(M + 3 * N + K)
    A = g.uniform(-1, 1, (M, K)).astype(np.float32)
    W = g.uniform(-1, 1, (K, N)).astype(np.float32)
    want = ref.tiled_matmul_act(A, W, act)
    got = jb.gemm_f32_tc(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(), act=act)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    assert rel_l2(to_np(got), want) <= F32_REL_L2
    # against float64 too (K = 4096 runs as four 1024-column chunks, each
    # adding the running sum in fp32); tf32 alone (~5e-4) would fail this by far
    exact = A.astype(np.float64) @ W.astype(np.float64)
    if act == "none":
        assert rel_l2(to_np(got), exact) <= F32_REL_L2


def test_gemm_f32_tc_bias_and_tail_split(jb):
    """Bias + GELU at a shape whose last round runs as half-width units (80
    tiles on 74 pairs), vs float64."""
    import torch
    g = np.random.default_rng(17)
    M, N, K = 2560, 2048, 96
    A = g.standard_normal((M, K)).astype(np.float32)
    W = (g.standard_normal((K, N)) / 8).astype(np.float32)
    b = g.standard_normal(N).astype(np.float32)
    got = to_np(jb.gemm_f32_tc(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(),
                               torch.from_numpy(b).cuda(), act="gelu"))
    z = A.astype(np.float64) @ W + b
    want = 0.5 * z * (1 + np.tanh(0.7978845608 * (z + 0.044715 * z ** 3)))
    assert rel_l2(got, want) <= 2e-6
    assert np.abs(got - want).max() <= 1e-4


def test_gemm_f32_tc_fallback_and_workspace(jb):
    """Shapes the tensor cores do not take (N % 8 != 0, M < 256) run the fp32
    CUDA-core GEMM; a workspace below the size query is refused."""
    import torch
    g = np.random.default_rng(3)
    for (M, N, K) in ((300, 260, 64), (100, 512, 64)):
        A = g.uniform(-1, 1, (M, K)).astype(np.float32)
        W = g.uniform(-1, 1, (K, N)).astype(np.float32)
        got = jb.gemm_f32_tc(torch.from_numpy(A).cuda(), torch.from_numpy(W).cuda(),
                             workspace=torch.empty(16, dtype=torch.uint8, device="cuda"))
        assert rel_l2(to_np(got), A.astype(np.float64) @ W) <= F32_REL_L2
    M, N, K = 512, 512, 128
    need = jb.gemm_f32_tc_workspace_bytes(M, N, K)
    a256 = lambda n: (n + 255) // 256 * 256
    assert need == a256(M * 3 * K * 4) + 3 * K * N * 4  # A3 and W3T
    assert jb.gemm_f32_tc_workspace_bytes(M, N, 3000) == a256(M * 9000 * 4) + 9000 * N * 4
    A = torch.zeros((M, K), device="cuda")
    W = torch.zeros((K, N), device="cuda")
    C = torch.empty((M, N), device="cuda")
    ws = torch.empty(need - 256, dtype=torch.uint8, device="cuda")
    rc = jb.lib().jules_gemm_f32_tc(jb._ptr(A), jb._ptr(W), None, jb._ptr(C), M, N, K, 0,
                                    jb._ptr(ws), ws.numel(), None)
    assert rc == 8  # JULES_ERR_WORKSPACE


def test_gemm_fp32_bias_relu_vs_reference(jb, ref):
    import torch
    g = np.random.default_rng(11)
    X = g.uniform(-1, 1, (96, 200)).astype(np.float32)
    W = g.uniform(-1, 1, (200, 144)).astype(np.float32)
    b = g.uniform(-1, 1, 144).astype(np.float32)
    want = ref.fused_matmul_bias_relu(X, W, b)
    got = jb.gemm_bias_act(torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda(),
                           torch.from_numpy(b).cuda(), act="relu")
    assert rel_l2(to_np(got), want) <= F32_REL_L2


@pytest.mark.parametrize("ta,tb", [(False, False), (True, False), (False, True), (True, True)])
def test_sgemm_vs_reference_blas(jb, ref, ta, tb):
    import torch
    g = np.random.default_rng(5)
    M, N, K = 70, 50, 90
    A = g.uniform(-1, 1, (K, M) if ta else (M, K)).astype(np.float32)
    B = g.uniform(-1, 1, (N, K) if tb else (K, N)).astype(np.float32)
    C0 = g.uniform(-1, 1, (M, N)).astype(np.float32)
    want = (A.T if ta else A).astype(np.float64) @ (B.T if tb else B) * 0.5 + 2.0 * C0
    dC = torch.from_numpy(C0.copy()).cuda()
    got = jb.sgemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), dC, alpha=0.5, beta=2.0,
                   transA=ta, transB=tb)
    assert rel_l2(to_np(got), want) <= F32_REL_L2
    if not ta and not tb:
        r = ref.blas_matmul(A, B)
        got2 = jb.sgemm(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda())
        assert rel_l2(to_np(got2), r) <= F32_REL_L2


# --- fp16 operands (tcgen05 kind::f16 with the f16 format; the reference's
# mixed-precision pass treats f16 like bf16, MixedPrecisionPass.cpp:76) ----
@pytest.mark.parametrize("M,N,K", [(256, 512, 256), (129, 264, 72), (640, 1024, 1024), (7, 40, 24)])
@pytest.mark.parametrize("act", ["none", "gelu"])
def test_gemm_f16(jb, orc, M, N, K, act):
    import torch
    from helpers import f16_np
    g = np.random.default_rng(M + 3 * N + K)
    s = 1.0 / np.sqrt(K)
    A = f16_np(g.uniform(-1, 1, (M, K)).astype(np.float32) * s)
    W = f16_np(g.uniform(-1, 1, (K, N)).astype(np.float32) * s)
    b = (g.standard_normal(N) * 0.02).astype(np.float32)
    R = f16_np(g.standard_normal((M, N)).astype(np.float32))
    bias = torch.from_numpy(b).cuda()
    C = jb.gemm_bias_act(to_dev(A, "f16"), to_dev(W, "f16"), bias, to_dev(R, "f16"), act=act)
    C32 = jb.gemm_bias_act(to_dev(A, "f16"), to_dev(W, "f16"), bias, to_dev(R, "f16"), act=act,
                           out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    assert C.dtype == torch.float16
    want = orc.gemm_bias_act(A, W, b, R, act)
    assert max_abs(to_np(C), want) <= BF16_MAX_ABS
    assert rel_l2(to_np(C), want) <= BF16_REL_L2
    assert max_abs(to_np(C32), want) <= 2e-3
    assert torch.equal(C, C32.to(torch.float16))  # one rounding, at the store


def test_gemm_f16_rejects_mixed_dtypes(jb):
    import torch
    a = torch.zeros((256, 256), dtype=torch.float16, device="cuda")
    w = torch.zeros((256, 256), dtype=torch.bfloat16, device="cuda")
    c = torch.empty((256, 256), dtype=torch.bfloat16, device="cuda")
    rc = jb.lib().jules_gemm_bias_act(jb._ptr(a), jb._ptr(a), None, None, jb._ptr(c), 256, 256, 256,
                                      0, jb.DT_F16, jb.DT_BF16, jb._stream(None))
    assert rc == 3  # JULES_ERR_DTYPE: f16 operands give f16 or fp32 C
    del w


# --- more 256 x 256 tiles than the 74 CTA pairs, with a partial last round
# (run as half-width units when it is at most half full) ---------------------
@pytest.mark.parametrize("M,N,K", [(2560, 2048, 128),   # 80 tiles: last round 6 -> 12 halves
                                   (4096, 4096, 320),   # 256 tiles: 34 -> 68 halves
                                   (2600, 2056, 200),   # ragged rows / columns / K, 99 tiles
                                   (4096, 2048, 1024)]) # 128 tiles: last round 54, whole
def test_gemm_multi_round(jb, orc, M, N, K):
    import torch
    A, W, b = gemm_inputs(M, N, K, seed=M + N + 3 * K)
    g = np.random.default_rng(K)
    R = bf16_np(g.standard_normal((M, N)).astype(np.float32))
    rows = np.linspace(0, M - 1, 64).astype(np.int64)
    Ad, Wd, Rd, bd = to_dev(A), to_dev(W), to_dev(R), torch.from_numpy(b).cuda()
    C = jb.gemm_bias_act(Ad, Wd, bd, Rd, act="gelu")
    C32 = jb.gemm_bias_act(Ad, Wd, bd, Rd, act="gelu", out_dtype=torch.float32)
    C_again = jb.gemm_bias_act(Ad, Wd, bd, Rd, act="gelu")
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = orc.gemm_bias_act(A[rows], W, b, R[rows], "gelu")
    got = to_np(C32[torch.from_numpy(rows).cuda()])
    assert max_abs(got, want) <= 2e-3
    assert rel_l2(got, want) <= 1e-3
    assert torch.equal(C, C32.to(torch.bfloat16))   # one rounding, at the store
    assert torch.equal(C, C_again)                   # deterministic across launches
    # the last tiles (the half-width units): whole columns against the oracle
    cols = np.arange(N - 256, N)
    tail_rows = np.arange(max(0, M - 256), M)
    want_t = orc.gemm_bias_act(np.ascontiguousarray(A[tail_rows]), np.ascontiguousarray(W[:, cols]),
                               np.ascontiguousarray(b[cols]),
                               np.ascontiguousarray(R[np.ix_(tail_rows, cols)]), "gelu")
    got_t = to_np(C32[torch.from_numpy(tail_rows).cuda()][:, torch.from_numpy(cols).cuda()])
    assert max_abs(got_t, want_t) <= 2e-3
