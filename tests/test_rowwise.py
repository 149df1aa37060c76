"""Row softmax and fused softmax + cross-entropy: CUDA kernels vs the
reference's own fusedSoftmax / fusedCrossEntropyLoss (compiled from source,
oracle/_ref) for fp32, and vs the C restatement on the same bf16 values."""
import numpy as np
import pytest

from conftest import BF16_MAX_ABS, BF16_REL_L2, F32_REL_L2, max_abs, rel_l2
from helpers import to_dev, to_np

pytestmark = pytest.mark.gpu

# warp-per-row path (N <= 1024), the register-resident CTA path at each of its
# sizes (N a multiple of the vector width), the shared-memory-staged path
# (rows of 32 KB and more; M > SM count so CTAs stage several rows), and the
# two-pass CTA path (ragged N, or N beyond 32K fp32)
SHAPES = [(64, 256), (64, 10), (2048, 2048), (7, 1000), (5, 1024), (5, 1025), (3, 5000),
          (4, 8192), (4, 16384), (4, 32768), (300, 16384), (2, 70000), (1, 1), (300, 1)]


def _logits(M, N, seed, scale=3.0):
    g = np.random.default_rng(seed)
    return (scale * g.standard_normal((M, N))).astype(np.float32)


@pytest.mark.parametrize("M,N", SHAPES)
def test_softmax_fp32_vs_reference(jb, ref, M, N):
    import torch
    x = _logits(M, N, seed=M * 31 + N)
    got = jb.softmax(to_dev(x, "f32"))
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = ref.softmax(x)
    assert rel_l2(to_np(got), want) <= F32_REL_L2
    assert np.allclose(to_np(got).sum(axis=1), 1.0, atol=1e-5)


@pytest.mark.parametrize("M,N", [(64, 256), (7, 1000), (3, 5000), (4, 32768), (2, 40000)])
def test_softmax_bf16(jb, orc, M, N):
    import torch
    x = to_dev(_logits(M, N, seed=N), "bf16")
    xs = to_np(x)  # the bf16 values as fp32
    want = orc.softmax(xs)
    got32 = jb.softmax(x, out_dtype=torch.float32)
    got16 = jb.softmax(x)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    assert rel_l2(to_np(got32), want) <= F32_REL_L2  # bf16 in, fp32 arithmetic and out
    assert max_abs(to_np(got16), want) <= BF16_MAX_ABS
    assert rel_l2(to_np(got16), want) <= BF16_REL_L2
    # the bf16 output is the fp32 result rounded once (the two outputs may come
    # from different kernels, so allow the rounding of a 1-ulp fp32 difference)
    assert bool(((got16.float() - got32).abs() <= got32.abs() * 2.0 ** -8).all())


@pytest.mark.parametrize("M,N", [(64, 10), (64, 1000), (13, 37), (5, 3000), (2, 50257),
                                 (300, 1024), (8, 32768), (300, 32768), (3, 40000)])
def test_cross_entropy_fp32_vs_reference(jb, ref, M, N):
    import torch
    x = _logits(M, N, seed=M + 7 * N)
    t = np.random.default_rng(N).integers(0, N, M).astype(np.int32)
    loss, grad = jb.cross_entropy_loss(to_dev(x, "f32"), torch.from_numpy(t).cuda())
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want_loss, want_grad = ref.cross_entropy(x, t)
    assert abs(float(loss) - want_loss) <= 1e-5 * max(1.0, abs(want_loss))
    assert rel_l2(to_np(grad), want_grad) <= F32_REL_L2
    # each gradient row sums to zero: (sum p - 1) / M
    assert np.abs(to_np(grad).astype(np.float64).sum(axis=1)).max() <= 1e-6


def test_cross_entropy_loss_only_and_bf16(jb, orc):
    import torch
    M, N = 96, 3000
    x = to_dev(_logits(M, N, seed=5), "bf16")
    t = torch.from_numpy(np.random.default_rng(6).integers(0, N, M).astype(np.int32)).cuda()
    loss0, none = jb.cross_entropy_loss(x, t, grad=False)
    loss1, grad = jb.cross_entropy_loss(x, t)
    torch.cuda.synchronize()
    assert none is None and jb.device_error() == 0
    want_loss, want_grad = orc.cross_entropy(to_np(x), t.cpu().numpy())
    for lv in (float(loss0), float(loss1)):
        assert abs(lv - want_loss) <= 1e-5 * abs(want_loss)
    assert grad.dtype == torch.bfloat16
    assert rel_l2(to_np(grad), want_grad) <= BF16_REL_L2


def test_cross_entropy_target_out_of_range(jb, orc):
    """A target outside [0, N) is caught by the kernel's own check: the row
    adds no loss, its gradient carries no one-hot term, and the device error
    word is set."""
    import torch
    M, N = 8, 100
    x = _logits(M, N, seed=9)
    t = np.arange(M, dtype=np.int32)
    t[3] = N  # out of range
    loss, grad = jb.cross_entropy_loss(to_dev(x, "f32"), torch.from_numpy(t).cuda())
    torch.cuda.synchronize()
    assert jb.device_error() != 0  # read and cleared
    assert jb.device_error() == 0
    good = np.array([i for i in range(M) if i != 3])
    want_loss, _ = orc.cross_entropy(x[good], t[good])
    assert abs(float(loss) - want_loss * (M - 1) / M) <= 1e-5 * abs(want_loss)
    assert rel_l2(to_np(grad)[3], orc.softmax(x[3:4])[0] / M) <= F32_REL_L2
