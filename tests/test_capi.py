"""C ABI checks that need no GPU: the library loads, exports every symbol the
headers declare, validates arguments before touching the device, and the
extern_kernel registry answers."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import ROOT

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


FAKE = ctypes.c_void_p(256)  # never dereferenced: validation fails first


def test_gemm_argument_errors(jb):
    h = jb.lib()
    assert h.jules_gemm_bias_act(None, FAKE, None, None, FAKE, 4, 4, 4, 0, 1, 1, None) == 6
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 4, 0, 4, 0, 1, 1, None) == 1
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 4, 4, 4, 9, 1, 1, None) == 6
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 4, 4, 4, 0, 7, 1, None) == 3
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 1 << 32, 4, 4, 0, 1, 1, None) == 1
    assert h.jules_gemm_bias_act(FAKE, FAKE, None, None, FAKE, 0, 4, 4, 0, 1, 1, None) == 0
    assert b"NULL" in h.jules_last_error_string() or h.jules_last_error_string() == b""


def test_attention_argument_errors(jb):
    h = jb.lib()
    f = h.jules_flash_attention_fwd
    assert f(None, FAKE, FAKE, FAKE, None, 1, 1, 1, 8, 64, 0.0, 0, 1, None) == 6
    assert f(FAKE, FAKE, FAKE, FAKE, None, 1, 3, 2, 8, 64, 0.0, 0, 1, None) == 1  # Hq % Hkv
    assert f(FAKE, FAKE, FAKE, FAKE, None, 1, 2, 2, 8, 512, 0.0, 0, 1, None) == 1  # D > 256
    assert f(FAKE, FAKE, FAKE, FAKE, None, 0, 2, 2, 8, 64, 0.0, 0, 1, None) == 0   # empty
    assert f(FAKE, FAKE, FAKE, FAKE, None, 1, 2, 2, 0, 64, 0.0, 0, 1, None) == 0   # empty


def test_norm_mlp_argument_errors(jb):
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
                           ctypes.c_void_p(264), need, None)
    assert rc == 2  # workspace misaligned
    rc = h.jules_mlp_block(FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, FAKE, 5, 16, 64, 256, 1e-5,
                           ctypes.c_void_p(256), need, None)
    assert rc == 3  # bad out dtype


def test_sgemm_argument_errors(jb):
    h = jb.lib()
    assert h.jules_sgemm(0, 0, 4, 4, 4, 1.0, None, 4, FAKE, 4, 0.0, FAKE, 4, None) == 6
    assert h.jules_sgemm(0, 0, 4, 4, 4, 1.0, FAKE, 2, FAKE, 4, 0.0, FAKE, 4, None) == 1  # lda < K
