"""2-layer MLP training step (jules_mlp_fwd_bwd, the reference's
interleavedMLPForwardBackward) vs the reference built from source, fp32."""
import numpy as np
import pytest

from conftest import F32_REL_L2, rel_l2

pytestmark = pytest.mark.gpu


def _inputs(M, K1, N1, N2, seed):
    g = np.random.default_rng(seed)
    return [g.uniform(-1, 1, (M, K1)).astype(np.float32),
            (g.uniform(-1, 1, (K1, N1)) / np.sqrt(K1)).astype(np.float32),
            (0.1 * g.standard_normal(N1)).astype(np.float32),
            (g.uniform(-1, 1, (N1, N2)) / np.sqrt(N1)).astype(np.float32),
            (0.1 * g.standard_normal(N2)).astype(np.float32),
            g.integers(0, N2, M).astype(np.int32)]


@pytest.mark.parametrize("M,K1,N1,N2", [(64, 784, 256, 10), (128, 100, 48, 10), (37, 33, 65, 17),
                                        (512, 1024, 512, 1000)])
def test_mlp_fwd_bwd_vs_reference(jb, ref, M, K1, N1, N2):
    import torch
    ins = _inputs(M, K1, N1, N2, seed=M + K1)
    got = jb.mlp_fwd_bwd(*[torch.from_numpy(a).cuda() for a in ins])
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    want = ref.mlp_fwd_bwd(*ins)
    assert abs(float(got["loss"]) - want["loss"]) <= 1e-5 * max(1.0, abs(want["loss"]))
    for k in ("out", "dW1", "db1", "dW2", "db2", "dX"):
        assert rel_l2(got[k].cpu().numpy(), want[k]) <= F32_REL_L2, k


def test_mlp_fwd_bwd_without_dx(jb, orc):
    import torch
    ins = _inputs(50, 60, 70, 12, seed=3)
    got = jb.mlp_fwd_bwd(*[torch.from_numpy(a).cuda() for a in ins], want_dx=False)
    torch.cuda.synchronize()
    want = orc.mlp_fwd_bwd(*ins, want_dx=False)
    assert got["dX"] is None
    for k in ("out", "dW1", "db1", "dW2", "db2"):
        assert rel_l2(got[k].cpu().numpy(), want[k]) <= F32_REL_L2, k
