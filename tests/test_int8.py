"""int8 GEMM (matmulInt8): tcgen05 kind::i8 and the CUDA-core fallback vs
the reference's own matmulInt8 built without AVX-512 (its scalar branch,
oracle/_ref libjules_ref_avx2.so) and vs an exact int64 product.  int32
accumulation is exact, so results match to the fp32 rounding of the scale."""
import numpy as np
import pytest

from conftest import max_abs

pytestmark = pytest.mark.gpu


def _exact(A, B, sa, sb, bias):
    acc = A.astype(np.int64) @ B.astype(np.int64)
    C = acc.astype(np.float32) * np.float32(sa * sb)
    return C + bias if bias is not None else C


# M, N >= 256 take the CTA-pair kernel (256 x 256 tiles), the rest the 1-CTA one
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (300, 512, 384), (1, 16, 16), (129, 272, 4096),
                                   (640, 1024, 1024), (1000, 784, 528), (2048, 2304, 2048)])
@pytest.mark.parametrize("with_bias", [False, True])
def test_matmul_int8_tensor_cores(jb, M, N, K, with_bias):
    import torch
    g = np.random.default_rng(M * 7 + N + K)
    A = g.integers(-128, 128, (M, K)).astype(np.int8)
    B = g.integers(-128, 128, (K, N)).astype(np.int8)
    bias = g.standard_normal(N).astype(np.float32) if with_bias else None
    C = jb.matmul_int8(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), 0.01, 0.02,
                       torch.from_numpy(bias).cuda() if with_bias else None)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = _exact(A, B, 0.01, 0.02, bias)
    # int32 accumulation is exact; the only rounding is float(acc) * scale (+ bias)
    assert max_abs(C.cpu().numpy(), want) <= 1e-6 * max(1.0, float(np.abs(want).max()))


@pytest.mark.parametrize("M,N,K", [(37, 45, 77), (64, 96, 200), (5, 1000, 33)])
def test_matmul_int8_fallback_vs_reference(jb, M, N, K):
    """K or N not a multiple of 16: the CUDA-core kernel; checked against the
    reference build's scalar matmulInt8."""
    import sys
    import torch
    import oracle
    g = np.random.default_rng(K)
    A = g.integers(-128, 128, (M, K)).astype(np.int8)
    B = g.integers(-128, 128, (K, N)).astype(np.int8)
    bias = g.standard_normal(N).astype(np.float32)
    C = jb.matmul_int8(torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda(), 0.5, 0.25,
                       torch.from_numpy(bias).cuda())
    torch.cuda.synchronize()
    ref = oracle.Reference(variant="avx2").matmul_int8(A, B, 0.5, 0.25, bias)
    assert max_abs(C.cpu().numpy(), ref) <= 1e-6 * max(1.0, float(np.abs(ref).max()))
