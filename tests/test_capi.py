"""C ABI checks that need no GPU: the library loads, exports every symbol the
headers declare, validates arguments before touching the device, and the
extern_kernel registry answers."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT
from helpers import arg_buffer

INC = os.path.join(ROOT, "include")


def _c_decls():
    src = open(os.path.join(INC, "jules_kernels.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(jules_[a-z0-9_]+)\s*\(", src)))


def _cxx_decls():
    names = set()
    for f in ("FusedKernels.h", "FlashAttention.h", "InterleavedAutodiff.h"):
        src = open(os.path.join(INC, "jules", "Kernel", f)).read()
        src = re.sub(r"//.*", "", src)
        for m in re.finditer(r"^\s*(?:void|int|bool|float|InterleavedMLPResult)\s+([A-Za-z0-9_]+)\s*\(",
                             src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_library_loads(jb):
    assert jb.lib().jules_version() >= 1


def test_exports_every_c_symbol(jb):
    decls = _c_decls()
    assert len(decls) >= 14
    missing = [n for n in decls if not hasattr(jb.lib(), n)]
    assert not missing, missing


def test_exports_every_cxx_symbol(jb):
    out = subprocess.run(["nm", "-D", "-C", "--defined-only", jb.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    for name in _cxx_decls():
        assert f"jules::kernel::{name}(" in out, name
    for sym in ("jules::kernel::ExecutionArena::ExecutionArena(", "jules::kernel::CacheInfo::detect("):
        assert sym in out, sym


def test_status_strings(jb):
    h = jb.lib()
    for code in range(9):
        assert h.jules_status_string(code)
    assert h.jules_status_string(0) == b"ok"


def test_registry(jb):
    names = jb.kernel_names()
    for n in ("fusedMatmulRelu", "fusedMatmulBiasRelu", "fusedMatmulBiasGelu", "fusedLayerNorm",
              "fusedGelu", "fusedMLPForward", "flashAttention", "fusedSoftmax"):
        assert n in names
        assert jb.kernel_by_name(n) == names.index(n)
    assert jb.kernel_by_name("noSuchKernel") == -1
    h = jb.lib()
    assert h.jules_kernel_implemented(jb.kernel_by_name("flashAttention")) == 1
    assert h.jules_kernel_name(-1) is None


@pytest.fixture(scope="module")
def FAKE():
    return arg_buffer()  # the calls below fail validation before any launch


def test_gemm_argument_errors(jb, FAKE):
    h = jb.lib()
    assert h.jules_gemm_bias_act(None, FAKE, None, None, FAKE, 4, 4, 4, 0, 1, 1, None) == 6
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 4, 0, 4, 0, 1, 1, None) == 1
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 4, 4, 4, 9, 1, 1, None) == 6
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 4, 4, 4, 0, 7, 1, None) == 3
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 1 << 32, 4, 4, 0, 1, 1, None) == 1
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 0, 4, 4, 0, 1, 1, None) == 0
    assert b"NULL" in h.jules_last_error_string() or h.jules_last_error_string() == b""


def test_gemm_f32_tc_argument_errors(jb, FAKE):
    """The 3xTF32 entry point validates before touching the device; its
    workspace query is host arithmetic (A3 [M,3K] padded to 256 bytes, then
    W3T [N,3K])."""
    h = jb.lib()
    f = h.jules_gemm_f32_tc
    assert f(None, FAKE, None, FAKE, 4, 4, 4, 0, None, 0, None) == 6      # NULL A
    assert f(FAKE, FAKE, None, FAKE, 4, 0, 4, 0, None, 0, None) == 1      # N = 0
    assert f(FAKE, FAKE, None, FAKE, 4, 4, 4, 9, None, 0, None) == 6      # act
    assert f(FAKE, FAKE, None, FAKE, 1 << 32, 4, 4, 0, None, 0, None) == 1
    assert f(FAKE, FAKE, None, FAKE, 0, 4, 4, 0, None, 0, None) == 0      # empty
    q = h.jules_gemm_f32_tc_workspace_bytes
    assert q(0, 4, 4) == 0 and q(4, 4, -1) == 0
    a256 = lambda n: (n + 255) // 256 * 256
    for (M, N, K) in ((256, 256, 256), (300, 264, 4096), (2048, 2048, 2048), (3, 5, 7)):
        assert q(M, N, K) == a256(M * 3 * K * 4) + 3 * K * N * 4


def test_attention_argument_errors(jb, FAKE):
    h = jb.lib()
    f = h.jules_flash_attention_fwd
    assert f(None, FAKE, FAKE, FAKE, None, 1, 1, 1, 8, 64, 0.0, 0, 1, None) == 6
    assert f(FAKE, FAKE, FAKE, FAKE, None, 1, 3, 2, 8, 64, 0.0, 0, 1, None) == 1  # Hq % Hkv
    assert f(FAKE, FAKE, FAKE, FAKE, None, 1, 2, 2, 8, 512, 0.0, 0, 1, None) == 1  # D > 256
    assert f(FAKE, FAKE, FAKE, FAKE, None, 0, 2, 2, 8, 64, 0.0, 0, 1, None) == 0   # empty
    assert f(FAKE, FAKE, FAKE, FAKE, None, 1, 2, 2, 0, 64, 0.0, 0, 1, None) == 0   # empty


def test_norm_mlp_argument_errors(jb, FAKE):
    h = jb.lib()
    assert h.jules_layernorm(None, FAKE, FAKE, FAKE, 4, 4, 1e-5, 0, 0, None, None, None) == 6
    assert h.jules_gelu(FAKE, FAKE, -1, 0, None) == 1
    need = h.jules_mlp_block_workspace_bytes(16, 64, 256)
    assert need == 16 * 64 * 2 + 16 * 256 * 2
    assert h.jules_mlp_block_workspace_bytes(0, 64, 256) == 0
    rc = h.jules_mlp_block(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 16, 64, 256, 1e-5,
                           None, 0, None)
    assert rc == 8
    rc = h.jules_mlp_block(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 1, 16, 64, 256, 1e-5,
                           ctypes.c_void_p(FAKE.value + 8), need, None)
    assert rc == 2  # workspace misaligned
    rc = h.jules_mlp_block(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 5, 16, 64, 256, 1e-5,
                           FAKE, need, None)
    assert rc == 3  # bad out dtype


def test_sgemm_argument_errors(jb, FAKE):
    h = jb.lib()
    assert h.jules_sgemm(0, 0, 4, 4, 4, 1.0, None, 4, FAKE, 4, 0.0, FAKE, 4, None) == 6
    assert h.jules_sgemm(0, 0, 4, 4, 4, 1.0, FAKE, 2, FAKE, 4, 0.0, FAKE, 4, None) == 1  # lda < K


def test_selftest_wait_rejects_bad_limits(jb):
    h = jb.lib()
    assert h.jules_selftest_bounded_wait(0, None) == 6
    assert h.jules_selftest_bounded_wait(3_000_000_000, None) == 6


@pytest.mark.gpu
def test_bounded_wait_expires_and_context_survives(jb):
    """A pipeline wait on a barrier that nothing completes gives up after its
    limit, reports JULES_ERR_TIMEOUT with its site through the device error
    word, and the kernel returns: the next launch on the same context works."""
    import time

    import torch
    h = jb.lib()
    assert jb.device_error() == 0
    limit_ns = 50_000_000  # 50 ms
    t0 = time.perf_counter()
    assert h.jules_selftest_bounded_wait(limit_ns, None) == 0
    word = ctypes.c_uint32(0)
    assert h.jules_device_error(ctypes.byref(word), 1) == 5  # JULES_ERR_TIMEOUT
    elapsed = time.perf_counter() - t0
    assert word.value & 0xff == 1 and (word.value >> 8) & 0xff == 250, hex(word.value)
    assert elapsed >= limit_ns * 1e-9
    assert elapsed < 10.0
    assert jb.device_error() == 0  # cleared
    a = torch.ones((256, 256), dtype=torch.bfloat16, device="cuda")
    c = jb.gemm_bias_act(a, a)
    torch.cuda.synchronize()
    assert jb.device_error() == 0
    assert bool((c.float() == 256.0).all())
