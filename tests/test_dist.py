"""Multi-GPU entry points (jules_dist_*): the partition and argument checks on
CPU; on 2 GPUs (skipped with fewer) the sharded GEMM - gather fused into the
epilogue as NVLink stores, and the in-place NCCL gather for other output
buffers - and the sharded attention, each bit-identical to the single-GPU
call on the same inputs, plus a rank that skips a call: the other rank's
bounded wait expires and reports JULES_ERR_TIMEOUT."""
import ctypes
import os
import socket
import subprocess

import pytest

from conftest import ROOT
from jules_b200 import shard


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


def test_dist_shard_matches_row_range(jb):
    for units in (0, 1, 7, 256, 4096, 4097):
        for world in (1, 2, 3, 8):
            for rank in range(world):
                assert jb.dist_shard(units, world, rank) == shard.row_range(units, rank, world)


def test_dist_argument_errors(jb):
    h = jb.lib()
    c = ctypes.c_void_p()
    uid = ctypes.create_string_buffer(128)
    assert h.jules_dist_init(ctypes.byref(c), 9, 0, uid) == 6     # world > 8
    assert h.jules_dist_init(ctypes.byref(c), 2, 2, uid) == 6     # rank >= world
    assert h.jules_dist_gemm_bias_act(None, None, None, None, None, None, 4, 4, 4, 0, 1, 1, None) == 6
    assert h.jules_dist_flash_attention_fwd(None, None, None, None, None, None, 1, 1, 1, 8, 64, 0.0,
                                            0, 1, None) == 6
    b, e = ctypes.c_int64(), ctypes.c_int64()
    assert h.jules_dist_shard(10, 0, 0, ctypes.byref(b), ctypes.byref(e)) == 6
    assert h.jules_status_string(9) == b"collective communication error"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, case):
    import torch
    import torch.distributed as tdist
    import jules_b200 as jb
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    tdist.init_process_group("gloo", rank=rank, world_size=world)
    dist = None
    try:
        dist = jb.Dist.from_torch()
        g = torch.Generator(device="cuda").manual_seed(5)  # the same inputs on every rank
        bf = torch.bfloat16
        out = {}
        if case == "gemm":
            for (M, N, K, act) in ((1024, 768, 512, "gelu"), (1536, 512, 320, "relu")):
                A = (torch.rand((M, K), generator=g, device="cuda") - 0.5).to(bf)
                W = ((torch.rand((K, N), generator=g, device="cuda") - 0.5) / 8).to(bf)
                b = torch.randn(N, generator=g, device="cuda") * 0.02
                R = torch.randn((M, N), generator=g, device="cuda").to(bf)
                want = jb.gemm_bias_act(A, W, b, R, act=act)
                C = dist.alloc_shared((M, N), bf)           # fused gather
                dist.gemm_bias_act(A, W, b, R, act=act, out=C)
                C2 = torch.full((M, N), float("nan"), dtype=bf, device="cuda")  # NCCL gather
                dist.gemm_bias_act(A, W, b, R, act=act, out=C2)
                dist.gemm_bias_act(A, W, b, R, act=act, out=C)  # a second fused call
                torch.cuda.synchronize()
                out[f"fused{M}"] = bool(torch.equal(C, want))
                out[f"nccl{M}"] = bool(torch.equal(C2, want))
                dist.barrier()  # no rank frees C while another still writes it
                torch.cuda.synchronize()
                dist.free_shared(C)
            # ragged rows (1001 over 2 ranks): grouped broadcasts
            A = (torch.rand((1001, 256), generator=g, device="cuda") - 0.5).to(bf)
            W = ((torch.rand((256, 512), generator=g, device="cuda") - 0.5) / 8).to(bf)
            want = jb.gemm_bias_act(A, W)
            C3 = dist.gemm_bias_act(A, W)
            torch.cuda.synchronize()
            out["ragged"] = bool(torch.equal(C3, want))
        elif case == "attn":
            for (B, Hq, Hkv, S) in ((2, 4, 2, 384), (1, 8, 4, 256)):
                Q = torch.randn((B, Hq, S, 128), generator=g, device="cuda").to(bf)
                K = torch.randn((B, Hkv, S, 128), generator=g, device="cuda").to(bf)
                V = torch.randn((B, Hkv, S, 128), generator=g, device="cuda").to(bf)
                Ow, lw = jb.flash_attention_fwd(Q, K, V, causal=True)
                O = torch.full_like(Q, float("nan"))  # NCCL gather
                L = torch.full((B, Hq, S), float("nan"), device="cuda")
                dist.flash_attention_fwd(Q, K, V, causal=True, out=O, lse=L)
                Of = dist.alloc_shared((B, Hq, S, 128), bf)  # gather fused into the kernel
                Lf = dist.alloc_shared((B, Hq, S), torch.float32)
                dist.flash_attention_fwd(Q, K, V, causal=True, out=Of, lse=Lf)
                Of2 = dist.alloc_shared((B, Hq, S, 128), bf)  # fused, without lse
                dist.flash_attention_fwd(Q, K, V, causal=True, out=Of2)
                torch.cuda.synchronize()
                tag = f"{B}x{Hq}x{Hkv}"
                out[f"O{tag}"] = bool(torch.equal(O, Ow))
                out[f"lse{tag}"] = bool(torch.equal(L, lw))
                out[f"Ofused{tag}"] = bool(torch.equal(Of, Ow))
                out[f"lsefused{tag}"] = bool(torch.equal(Lf, lw))
                out[f"Ofused_nolse{tag}"] = bool(torch.equal(Of2, Ow))
                dist.barrier()
                torch.cuda.synchronize()
                for t_ in (Of, Lf, Of2):
                    dist.free_shared(t_)
        elif case == "timeout":
            M, N, K = 1024, 512, 256
            A = (torch.rand((M, K), generator=g, device="cuda") - 0.5).to(bf)
            W = ((torch.rand((K, N), generator=g, device="cuda") - 0.5) / 8).to(bf)
            C = dist.alloc_shared((M, N), bf)
            dist.gemm_bias_act(A, W, out=C)  # both ranks
            torch.cuda.synchronize()
            tdist.barrier()
            if rank == 0:  # rank 1 skips this call: rank 0's wait for it must expire
                dist.gemm_bias_act(A, W, out=C)
                w = ctypes.c_uint32(0)
                out["rc"] = jb.lib().jules_device_error(ctypes.byref(w), 1)
                out["site"] = (w.value >> 8) & 0xff
            tdist.barrier()  # rank 1 stays alive (its C stays mapped) until rank 0 is done
        assert jb.device_error() == 0
        out["multicast"] = dist.multicast
        q.put((rank, out))
    except Exception as ex:  # reported to the parent
        q.put((rank, {"error": repr(ex)}))
    finally:
        if dist is not None:
            dist.close()
        tdist.destroy_process_group()


def _run2(case, multicast=False, gather=None):
    """Two ranks on GPUs 0 and 1.  multicast=False: NVLS off in NCCL and in
    the library (peer stores over CUDA IPC mappings); True: both on.
    gather: JULES_DIST_GATHER for the ranks ("fused", "pull") or None."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    saved = {k: os.environ.get(k) for k in ("NCCL_NVLS_ENABLE", "JULES_DIST_MULTICAST",
                                             "JULES_DIST_GATHER")}
    if gather:
        os.environ["JULES_DIST_GATHER"] = gather
    else:
        os.environ.pop("JULES_DIST_GATHER", None)
    if multicast:
        os.environ.pop("NCCL_NVLS_ENABLE", None)
        os.environ["JULES_DIST_MULTICAST"] = "1"
    else:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        os.environ["JULES_DIST_MULTICAST"] = "0"
    try:
        procs = [ctx.Process(target=_worker, args=(r, 2, port, q, case)) for r in range(2)]
        for p in procs:
            p.start()
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    return res


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")


@pytest.mark.gpu
@needs2
def test_dist_gemm_matches_single_gpu():
    res = _run2("gemm")
    for r in (0, 1):
        assert "error" not in res[r], res[r]
        assert not res[r].pop("multicast")  # peer stores over IPC mappings
        assert all(res[r].values()), res[r]


@pytest.mark.gpu
@needs2
def test_dist_attention_matches_single_gpu():
    res = _run2("attn")
    for r in (0, 1):
        assert "error" not in res[r], res[r]
        assert not res[r].pop("multicast")
        assert all(res[r].values()), res[r]


@pytest.mark.gpu
@needs2
@pytest.mark.parametrize("gather", ["fused", "pull"])
def test_dist_gather_routes_match_single_gpu(gather):
    """Both gather routes, forced: the epilogue's stores to every rank, and
    local stores plus copy-engine pulls of the peers' shares."""
    for case in ("gemm", "attn"):
        res = _run2(case, gather=gather)
        for r in (0, 1):
            assert "error" not in res[r], (case, res[r])
            assert not res[r].pop("multicast")
            assert all(res[r].values()), (case, res[r])


@pytest.mark.gpu
@needs2
def test_dist_gemm_multicast_matches_single_gpu():
    """The fused gather through NVLink multicast stores (NVLS on)."""
    res = _run2("gemm", multicast=True)
    for r in (0, 1):
        assert "error" not in res[r], res[r]
        assert res[r]["multicast"], "no multicast address on this node"
        assert all(res[r].values()), res[r]


@pytest.mark.gpu
@needs2
def test_dist_attention_multicast_matches_single_gpu():
    res = _run2("attn", multicast=True)
    for r in (0, 1):
        assert "error" not in res[r], res[r]
        assert res[r]["multicast"], "no multicast address on this node"
        assert all(res[r].values()), res[r]


@pytest.mark.gpu
@needs2
def test_dist_gemm_wait_expires_when_a_rank_skips_the_call():
    res = _run2("timeout")
    assert "error" not in res[0] and "error" not in res[1], res
    assert res[0]["rc"] == 5 and res[0]["site"] == 251, res[0]


@pytest.mark.gpu
@needs2
def test_dist_gemm_from_a_cpp_host(tmp_path, jb):
    """The sharded GEMM driven by a C++ program (no Python, no PyTorch): two
    processes, one GPU each, the NCCL id passed through a file."""
    exe = os.path.join(tmp_path, "dist_gemm")
    libdir = os.path.dirname(jb.LIB_PATH)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                    "-I", "/usr/local/cuda/include", os.path.join(ROOT, "tests", "cpp", "dist_gemm.cpp"),
                    "-o", exe, "-L", libdir, "-ljules_b200", f"-Wl,-rpath,{libdir}",
                    "-L", "/usr/local/cuda/lib64", "-lcudart"], check=True)
    idf = os.path.join(tmp_path, "nccl.id")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    procs = [subprocess.Popen([exe, str(r), "2", idf], env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.STDOUT, text=True) for r in range(2)]
    outs = [p.communicate(timeout=300)[0] for p in procs]
    for p, o in zip(procs, outs):
        assert p.returncode == 0, o
        assert "dist_gemm ok" in o, o
