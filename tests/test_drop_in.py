"""The reference's C++ API as a drop-in: a program written against
jules::kernel (tests/cpp/drop_in.cpp) compiles against include/ and links
libjules_b200.so; its results match the reference's own kernels."""
import os
import subprocess

import numpy as np
import pytest

import oracle

from conftest import F32_REL_L2, ROOT, rel_l2

def _compile(tmp, jb):
    exe = os.path.join(tmp, "drop_in")
    libdir = os.path.dirname(jb.LIB_PATH)
    cmd = ["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "drop_in.cpp"), "-o", exe, "-L", libdir,
           "-ljules_b200", f"-Wl,-rpath,{libdir}"]
    subprocess.run(cmd, check=True)
    return exe


def test_compiles_without_gpu(tmp_path, jb):
    _compile(str(tmp_path), jb)


@pytest.mark.gpu
def test_drop_in_matches_reference(tmp_path, jb, ref):
    d = str(tmp_path)
    exe = _compile(d, jb)
    g = np.random.default_rng(42)
    Q, K, V = (g.standard_normal((1, 8, 512, 64), dtype=np.float32) for _ in range(3))
    A = g.uniform(-1, 1, (96, 200)).astype(np.float32)
    W = g.uniform(-1, 1, (200, 136)).astype(np.float32)
    bias = g.uniform(-1, 1, 136).astype(np.float32)
    W2 = g.uniform(-1, 1, (136, 24)).astype(np.float32)
    b2 = g.uniform(-1, 1, 24).astype(np.float32)
    A8 = g.integers(-128, 128, (96, 200)).astype(np.int8)
    B8 = g.integers(-128, 128, (200, 136)).astype(np.int8)
    A9 = g.integers(-128, 128, (256, 256)).astype(np.int8)
    B9 = g.integers(-128, 128, (256, 512)).astype(np.int8)
    b9 = g.standard_normal(512).astype(np.float32)
    A_tc = g.uniform(-1, 1, (320, 200)).astype(np.float32)
    W_tc = g.uniform(-1, 1, (200, 264)).astype(np.float32)
    for name, arr in dict(q=Q, k=K, v=V, a=A, w=W, bias=bias, w2=W2, b2=b2, a8=A8, b8=B8, a9=A9,
                          b9=B9, b9bias=b9, a_tc=A_tc, w_tc=W_tc).items():
        arr.tofile(os.path.join(d, f"in_{name}.bin"))
    subprocess.run([exe, d], check=True)
    out = lambda n, shape: np.fromfile(os.path.join(d, f"out_{n}.bin"), np.float32).reshape(shape)
    assert rel_l2(out("flash", Q.shape), ref.flash_attention(Q, K, V)) <= F32_REL_L2
    assert rel_l2(out("attention", Q.shape), ref.attention(Q, K, V)) <= F32_REL_L2
    assert rel_l2(out("tiled_gelu", (96, 136)), ref.tiled_matmul_act(A, W, "gelu")) <= F32_REL_L2
    # M, N >= 256: the float* API on the 3xTF32 tensor-core GEMM
    assert rel_l2(out("tiled_gelu_tc", (320, 264)), ref.tiled_matmul_act(A_tc, W_tc, "gelu")) <= F32_REL_L2
    assert rel_l2(out("blas_tc", (320, 264)), ref.blas_matmul(A_tc, W_tc)) <= F32_REL_L2
    assert rel_l2(out("bias_relu", (96, 136)), ref.fused_matmul_bias_relu(A, W, bias)) <= F32_REL_L2
    assert rel_l2(out("standard", Q.shape), ref.standard_attention(Q, K, V)) <= F32_REL_L2
    # fusedMatmulRelu takes (M, K, N); a swapped order would not match (M, K, N all differ)
    assert rel_l2(out("relu", (96, 136)), ref.fused_matmul_relu(A, W)) <= F32_REL_L2
    # matmulInt8: int32 accumulation is exact, so the results equal the
    # reference's scalar branch (oracle/_ref avx2 build) bit for bit
    ref8 = oracle.Reference(variant="avx2")
    assert np.array_equal(out("int8_small", (96, 136)), ref8.matmul_int8(A8, B8, 0.5, 0.25, bias))
    assert np.array_equal(out("int8_tc", (256, 512)), ref8.matmul_int8(A9, B9, 0.5, 0.25, b9))
    assert np.array_equal(out("int8_tc_nobias", (256, 512)), ref8.matmul_int8(A9, B9))
    assert rel_l2(out("blas", (96, 136)), ref.blas_matmul(A, W)) <= F32_REL_L2
    ln = ref.layernorm(A, np.ones(200, np.float32), np.zeros(200, np.float32))
    assert rel_l2(out("layernorm", (96, 200)), ln) <= F32_REL_L2
    assert rel_l2(out("gelu", (96, 200)), ref.gelu(A)) <= F32_REL_L2
    assert rel_l2(out("mlp", (96, 24)), ref.mlp_forward(A, W, bias, W2, b2)) <= F32_REL_L2
    # softmax / cross-entropy of C = blasMatmul(A, W) (the last value written to C)
    C = out("blas", (96, 136))
    assert rel_l2(out("softmax", (96, 136)), ref.softmax(C)) <= F32_REL_L2
    tgt = ((np.arange(96) * 7) % 136).astype(np.int32)
    loss, grad = ref.cross_entropy(C, tgt)
    assert rel_l2(out("xent_grad", (96, 136)), grad) <= F32_REL_L2
    assert abs(float(out("xent_loss", (1,))[0]) - loss) <= 1e-5 * max(1.0, abs(loss))
    t24 = (np.arange(96) % 24).astype(np.int32)
    tr = ref.mlp_fwd_bwd(A, W, bias, W2, b2, t24)
    assert rel_l2(out("train_out", (96, 24)), tr["out"]) <= F32_REL_L2
    assert rel_l2(out("train_dW1", (200, 136)), tr["dW1"]) <= F32_REL_L2
    assert rel_l2(out("train_dX", (96, 200)), tr["dX"]) <= F32_REL_L2
    assert abs(float(out("train_loss", (1,))[0]) - tr["loss"]) <= 1e-5 * max(1.0, abs(tr["loss"]))
