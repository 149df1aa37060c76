"""jules_mlp_block_noalloc: the MLP block for callers that cannot allocate
device memory (a runtime's custom-call handler gets only its operand and
result buffers; the memory belongs to the runtime's allocator).  Its
workspace is an array compiled into the library.

Checked through the C ABI against jules_mlp_block (the entry point that
takes a caller workspace) on two calls in a row: both run the same kernels,
so the outputs must be identical bit for bit; one call is also checked
against the oracle, and the device's free memory must not change across the
calls.  The file is named so that pytest collects it last."""
import ctypes

import numpy as np
import pytest

from helpers import arg_buffer, bf16_np, to_np

_vp, _i64 = ctypes.c_void_p, ctypes.c_int64
DT_F32, DT_BF16 = 0, 1


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
    # d=4096, dff=16384: T=820 needs 820*4096*2 + 820*16384*2 > 32 MiB.  The
    # buffers have the sizes the call names (real device memory on a GPU box);
    # the size check fails before any launch.
    T, d, dff = 820, 4096, 16384
    X, out = arg_buffer(T * d * 2), arg_buffer(T * d * 2)
    W1, W2 = arg_buffer(d * dff * 2), arg_buffer(dff * d * 2)
    gam, bet, b2, b1 = arg_buffer(d * 4), arg_buffer(d * 4), arg_buffer(d * 4), arg_buffer(dff * 4)
    rc = f(X, gam, bet, W1, b1, W2, b2, out, DT_BF16, T, d, dff, 1e-5, None)
    assert rc == 8  # JULES_ERR_WORKSPACE
    assert b"built-in array" in h.jules_last_error_string()


def _inputs(T, d, dff, seed):
    import torch
    g = np.random.default_rng(seed)
    dev = lambda a, dt=torch.float32: torch.from_numpy(np.ascontiguousarray(a)).cuda().to(dt)
    w = dict(
        gam=dev((1 + 0.02 * g.standard_normal(d)).astype(np.float32)),
        bet=dev((0.02 * g.standard_normal(d)).astype(np.float32)),
        W1=dev(bf16_np((0.02 * g.standard_normal((d, dff))).astype(np.float32)), torch.bfloat16),
        b1=dev((0.02 * g.standard_normal(dff)).astype(np.float32)),
        W2=dev(bf16_np((0.02 * g.standard_normal((dff, d))).astype(np.float32)), torch.bfloat16),
        b2=dev((0.02 * g.standard_normal(d)).astype(np.float32)))
    Xs = [dev(bf16_np(g.standard_normal((T, d)).astype(np.float32)), torch.bfloat16)
          for _ in range(2)]
    return w, Xs


# (T, d, dff, out dtype): the second shape puts 80 tiles of 256 x 256 into the
# second GEMM, more than the 74 CTA pairs of a B200, so its last round runs
# split into half-width tiles; it needs 27.3 MB of the 32 MiB array.
@pytest.mark.gpu
@pytest.mark.parametrize("T,d,dff,out_dt", [(512, 1024, 4096, DT_BF16),
                                            (1024, 5120, 8192, DT_F32)])
def test_noalloc_matches_workspace_entry_point(jb, orc, T, d, dff, out_dt):
    import torch
    h = jb.lib()
    f, _ = _bind(h)
    w, Xs = _inputs(T, d, dff, seed=T + d)
    tdt = torch.bfloat16 if out_dt == DT_BF16 else torch.float32
    # The caller-workspace entry point first (its workspace comes from torch).
    wants = [jb.mlp_block(X, w["gam"], w["bet"], w["W1"], w["b1"], w["W2"], w["b2"],
                          out_dtype=tdt) for X in Xs]
    outs = [torch.full((T, d), float("nan"), dtype=tdt, device="cuda") for _ in range(3)]
    torch.cuda.synchronize()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    call = lambda X, out: f(_p(X), _p(w["gam"]), _p(w["bet"]), _p(w["W1"]), _p(w["b1"]),
                            _p(w["W2"]), _p(w["b2"]), _p(out), out_dt, T, d, dff, 1e-5, stream)
    assert call(Xs[1], outs[2]) == 0, h.jules_last_error_string()  # first call: set-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for i in range(2):  # the second call runs over the first call's leftovers
        assert call(Xs[i], outs[i]) == 0, h.jules_last_error_string()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0  # nothing allocated
    assert jb.device_error() == 0
    for i in range(2):
        assert torch.equal(outs[i], wants[i]), i
    # and against the oracle on sampled rows (fp32 restatement of the block)
    rows = np.linspace(0, T - 1, 8).astype(np.int64)
    want = orc.mlp_block(to_np(Xs[0]), *(to_np(w[k]) for k in ("gam", "bet", "W1", "b1", "W2", "b2")),
                         rows=rows)
    got = to_np(outs[0][torch.from_numpy(rows).cuda()])
    excess = np.abs(got.astype(np.float64) - want)
    if out_dt == DT_BF16:  # beyond the output's own bf16 rounding
        excess -= 2.0 ** (np.floor(np.log2(np.maximum(np.abs(want), 2.0 ** -126))) - 8)
    assert float(excess.max()) <= 2e-2
    assert float(np.linalg.norm(got - want) / np.linalg.norm(want)) <= 5e-3
