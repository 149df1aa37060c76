"""jules_mlp_block_noalloc: the MLP block for callers that cannot allocate
device memory (a runtime's custom-call handler gets only its operand and
result buffers; the memory belongs to the runtime's allocator).  Its
workspace is an array compiled into the library.

Checked through the C ABI against jules_mlp_block (the entry point that
takes a caller workspace) on two calls in a row.  The file is named so that
pytest collects it last."""
import ctypes

import numpy as np
import pytest

from conftest import BF16_MAX_ABS, BF16_REL_L2, max_abs, rel_l2
from helpers import bf16_np

_vp, _i64 = ctypes.c_void_p, ctypes.c_int64


def _bind(h):
    f = h.jules_mlp_block_noalloc
    f.argtypes = [_vp] * 8 + [ctypes.c_int, _i64, _i64, _i64, ctypes.c_float, _vp]
    f.restype = ctypes.c_int
    g = h.jules_mlp_block_noalloc_max_workspace_bytes
    g.argtypes = []
    g.restype = ctypes.c_size_t
    return f, g


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_rejects_oversized_workspace(jb):
    h = jb.lib()
    f, g = _bind(h)
    assert g() == 32 << 20
    fake = ctypes.c_void_p(256)  # never dereferenced: the size check fails first
    # d=4096, dff=16384: T=820 needs 820*4096*2 + 820*16384*2 > 32 MiB
    rc = f(fake, fake, fake, fake, fake, fake, fake, fake, 1, 820, 4096, 16384, 1e-5, None)
    assert rc == 8  # JULES_ERR_WORKSPACE
    assert b"built-in array" in h.jules_last_error_string()


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point(jb):
    import torch
    h = jb.lib()
    f, _ = _bind(h)
    T, d, dff = 512, 1024, 4096
    g = np.random.default_rng(11)
    dev = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dt)
    gam = dev((1 + 0.02 * g.standard_normal(d)).astype(np.float32))
    bet = dev((0.02 * g.standard_normal(d)).astype(np.float32))
    W1 = dev(bf16_np((0.02 * g.standard_normal((d, dff))).astype(np.float32)), torch.bfloat16)
    b1 = dev((0.02 * g.standard_normal(dff)).astype(np.float32))
    W2 = dev(bf16_np((0.02 * g.standard_normal((dff, d))).astype(np.float32)), torch.bfloat16)
    b2 = dev((0.02 * g.standard_normal(d)).astype(np.float32))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # the second call runs over the first call's leftovers
        X = dev(bf16_np(g.standard_normal((T, d)).astype(np.float32)), torch.bfloat16)
        out = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
        rc = f(_p(X), _p(gam), _p(bet), _p(W1), _p(b1), _p(W2), _p(b2), _p(out), 1, T, d, dff,
               1e-5, stream)
        assert rc == 0, h.jules_last_error_string()
        want = jb.mlp_block(X, gam, bet, W1, b1, W2, b2)  # caller-workspace entry point
        torch.cuda.synchronize()
        assert jb.device_error() == 0
        got_np, want_np = out.float().cpu().numpy(), want.float().cpu().numpy()
        assert max_abs(got_np, want_np) <= BF16_MAX_ABS, call
        assert rel_l2(got_np, want_np) <= BF16_REL_L2, call
