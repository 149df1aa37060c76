"""fp8 (E4M3 / E5M2): the element cast (jules_cast) and the fp8 GEMM
(jules_gemm_fp8, tcgen05 kind::f8f6f4 and the CUDA-core fallback).

The reference names the two fp8 types in its mixed-precision pass
(lib/Passes/MixedPrecisionPass.cpp:55-62) but has no fp8 arithmetic, so the
oracle restates the OCP 8-bit float formats (oracle/restate.c
orc_fp8_to_f32 / orc_f32_to_fp8); it is pinned here against torch's own
float8_e4m3fn / float8_e5m2 conversions, an independent implementation of
the same formats.  The GPU cast is bit-exact against the oracle; the GEMM is
compared with the oracle's exact (double) sum of the decoded products."""
import ctypes

import numpy as np
import pytest

from conftest import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, max_abs, rel_l2

JULES_ERR_DTYPE = 3
FMTS = {"e4m3": 2, "e5m2": 3}
LIMIT = {"e4m3": (448.0, 464.0), "e5m2": (57344.0, 61440.0)}  # max finite, overflow threshold


def _oracle():
    import oracle
    return oracle.Restated()


def _torch_f8(fmt):
    import torch
    return torch.float8_e4m3fn if fmt == "e4m3" else torch.float8_e5m2


def _cast_inputs(fmt, n=200003, seed=0):
    """Random values over the format's range, every exact value, every
    midpoint between neighbours (ties), their float neighbours, and the
    specials (zeros, overflow, infinities, NaN)."""
    R = _oracle()
    vals = R.fp8_decode(np.arange(256, dtype=np.uint8), fmt)
    vals = np.unique(vals[np.isfinite(vals)]).astype(np.float64)
    mids = ((vals[1:] + vals[:-1]) / 2).astype(np.float32)
    g = np.random.default_rng(seed)
    rnd = np.concatenate([g.standard_normal(n // 4) * s for s in (1e-3, 0.3, 20, 3000)])
    x = np.concatenate([rnd.astype(np.float32), vals.astype(np.float32), mids,
                        np.nextafter(mids, np.float32(np.inf)), np.nextafter(mids, np.float32(-np.inf)),
                        np.array([0.0, -0.0, 1e9, -1e9, np.inf, -np.inf, np.nan,
                                  LIMIT[fmt][0] * 1.01, -LIMIT[fmt][1]], np.float32)])
    return x.astype(np.float32)


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_oracle_fp8_codec_matches_torch(fmt):
    """Decode of all 256 codes and encode (nearest-even) of in-range values
    agree bit for bit with torch; out-of-range values saturate."""
    import torch
    R = _oracle()
    codes = np.arange(256, dtype=np.uint8)
    ours = R.fp8_decode(codes, fmt)
    ref = torch.from_numpy(codes).view(_torch_f8(fmt)).float().numpy()
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(ours), nan)
    assert np.array_equal(ours[~nan], ref[~nan])
    x = _cast_inputs(fmt)
    inr = np.isfinite(x) & (np.abs(x) < LIMIT[fmt][1])
    enc = R.fp8_encode(x, fmt)
    want = torch.from_numpy(x[inr]).to(_torch_f8(fmt)).view(torch.uint8).numpy()
    assert np.array_equal(enc[inr], want)
    # saturation (torch has no saturating cast): beyond the largest finite
    # value, infinities included, the result is +-max; NaN stays NaN
    big = ~np.isnan(x) & (np.abs(x) >= LIMIT[fmt][1])
    dec = R.fp8_decode(enc, fmt)
    assert big.any() and np.array_equal(np.abs(dec[big]), np.full(big.sum(), LIMIT[fmt][0], np.float32))
    assert np.array_equal(np.signbit(dec[big]), np.signbit(x[big]))
    assert np.isnan(dec[np.isnan(x)]).all()


def test_fp8_argument_errors(jb):
    L = jb.lib()
    p = ctypes.c_void_p(256)  # never dereferenced: the checks come first
    assert L.jules_gemm_fp8(p, p, None, None, p, 16, 16, 16, 1.0, 0, 1, 2, 0, None) == JULES_ERR_DTYPE
    assert L.jules_gemm_fp8(p, p, None, None, p, 16, 16, 16, 1.0, 0, 2, 3, 2, None) == JULES_ERR_DTYPE
    assert L.jules_cast(p, p, 16, 0, 4, None) == JULES_ERR_DTYPE
    assert L.jules_cast(p, p, 16, -1, 0, None) == JULES_ERR_DTYPE


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
@pytest.mark.parametrize("src", ["f32", "bf16"])
@pytest.mark.parametrize("vector", [True, False])
def test_cast_to_fp8_bit_exact(jb, fmt, src, vector):
    """fp32 / bf16 -> fp8 on the GPU equals the oracle's encode bit for bit
    (vector kernel: n % 8 == 0; scalar kernel otherwise)."""
    import torch
    R = _oracle()
    x = _cast_inputs(fmt, seed=1)
    n = (x.size // 8) * 8 if vector else (x.size // 8) * 8 - 3
    x = x[:n]
    xt = torch.from_numpy(x)
    if src == "bf16":
        xt = xt.to(torch.bfloat16)
        x = xt.float().numpy()
    y = jb.cast(xt.cuda(), _torch_f8(fmt))
    torch.cuda.synchronize()
    got = y.view(torch.uint8).cpu().numpy()
    want = R.fp8_encode(x, fmt)
    nan = np.isnan(x)
    assert np.array_equal(got[~nan], want[~nan])
    assert np.isnan(R.fp8_decode(got[nan], fmt)).all()


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["e4m3", "e5m2"])
def test_cast_from_fp8_exact(jb, fmt):
    import torch
    R = _oracle()
    codes = np.tile(np.arange(256, dtype=np.uint8), 9)
    want = R.fp8_decode(codes, fmt)
    d = torch.from_numpy(codes).cuda().view(_torch_f8(fmt))
    f = jb.cast(d, torch.float32).cpu().numpy()
    b = jb.cast(d, torch.bfloat16).float().cpu().numpy()  # every fp8 value is exact in bf16
    nan = np.isnan(want)
    for got in (f, b):
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(got[~nan], want[~nan])


def _gemm_inputs(M, N, K, seed, a_fmt, w_fmt):
    R = _oracle()
    g = np.random.default_rng(seed)
    A = R.fp8_encode(g.standard_normal((M, K)).astype(np.float32), a_fmt)
    W = R.fp8_encode((g.standard_normal((K, N)) / 8).astype(np.float32), w_fmt)
    bias = (0.1 * g.standard_normal(N)).astype(np.float32)
    res = (0.5 * g.standard_normal((M, N))).astype(np.float32)
    return A, W, bias, res


def _dev(jb, codes, fmt):
    import torch
    return torch.from_numpy(codes).cuda().view(_torch_f8(fmt))


# M, N >= 1 with K and N multiples of 16: CTA-pair tensor-core kernel;
# the rest: CUDA cores.
TC_SHAPES = [(256, 256, 128), (300, 512, 384), (1, 16, 16), (129, 272, 4096), (1000, 784, 528)]
SIMT_SHAPES = [(37, 45, 77), (64, 96, 200), (5, 1000, 33)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", TC_SHAPES + SIMT_SHAPES)
@pytest.mark.parametrize("a_fmt,w_fmt", [("e4m3", "e4m3"), ("e5m2", "e4m3"), ("e4m3", "e5m2")])
def test_gemm_fp8_f32_out(jb, M, N, K, a_fmt, w_fmt):
    """No activation, fp32 out: the fp32 accumulation against the exact sum."""
    import torch
    A, W, bias, _ = _gemm_inputs(M, N, K, M + N + K, a_fmt, w_fmt)
    C = jb.gemm_fp8(_dev(jb, A, a_fmt), _dev(jb, W, w_fmt), torch.from_numpy(bias).cuda(),
                    scale=0.5, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = _oracle().gemm_fp8(A, W, a_fmt, w_fmt, bias, None, "none", 0.5)
    assert rel_l2(C.cpu().numpy(), want) <= F32_REL_L2


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(300, 512, 384), (1000, 784, 528), (64, 96, 200)])
@pytest.mark.parametrize("act", ["gelu", "relu"])
def test_gemm_fp8_bias_act_residual_bf16(jb, M, N, K, act):
    """bias + activation + bf16 residual, bf16 out: within the bf16 bar."""
    import torch
    A, W, bias, res = _gemm_inputs(M, N, K, 7 * M + K, "e4m3", "e4m3")
    rt = torch.from_numpy(res).to(torch.bfloat16)
    C = jb.gemm_fp8(_dev(jb, A, "e4m3"), _dev(jb, W, "e4m3"), torch.from_numpy(bias).cuda(),
                    residual=rt.cuda(), act=act, scale=0.25)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = _oracle().gemm_fp8(A, W, "e4m3", "e4m3", bias, rt.float().numpy(), act, 0.25)
    got = C.float().cpu().numpy()
    assert rel_l2(got, want) <= BF16_REL_L2
    assert max_abs(got, want) <= BF16_MAX_ABS * max(1.0, float(np.abs(want).max()))


@pytest.mark.gpu
def test_gemm_bias_act_routes_fp8(jb):
    """jules_gemm_bias_act with fp8 operands is the fp8 GEMM at scale 1."""
    import torch
    A, W, bias, _ = _gemm_inputs(512, 256, 256, 3, "e5m2", "e5m2")
    a, w, b = _dev(jb, A, "e5m2"), _dev(jb, W, "e5m2"), torch.from_numpy(bias).cuda()
    C1 = jb.gemm_bias_act(a, w, b, act="gelu")
    C2 = jb.gemm_fp8(a, w, b, act="gelu")
    assert C1.dtype == torch.bfloat16 and torch.equal(C1, C2)


@pytest.mark.gpu
def test_cast_other_pairs_bit_exact(jb):
    """fp32 <-> bf16 (round to nearest even, as torch) and fp8 -> other fp8
    (decode, then the saturating encode) through the scalar cast kernel."""
    import torch
    R = _oracle()
    g = np.random.default_rng(3)
    x = np.concatenate([g.standard_normal(100001).astype(np.float32) * 100,
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e38, -1e-40], np.float32)])
    xt = torch.from_numpy(x).cuda()
    b = jb.cast(xt, torch.bfloat16)
    assert torch.equal(b.view(torch.int16).cpu(), xt.cpu().to(torch.bfloat16).view(torch.int16))
    f = jb.cast(b, torch.float32)
    assert torch.equal(f.cpu(), b.cpu().float())
    codes = np.arange(256, dtype=np.uint8)
    for src, dst in (("e4m3", "e5m2"), ("e5m2", "e4m3")):
        d = torch.from_numpy(codes).cuda().view(_torch_f8(src))
        got = jb.cast(d, _torch_f8(dst)).view(torch.uint8).cpu().numpy()
        dec = R.fp8_decode(codes, src)
        want = R.fp8_encode(dec, dst)
        nan = np.isnan(dec)
        assert np.array_equal(got[~nan], want[~nan])
        assert np.isnan(R.fp8_decode(got[nan], dst)).all()
