"""Benchmark of the Jules fused-kernel hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl jules|reference]
                    [--workload gemm|attn|attn_gqa|mlp|attn_fp32]

Default workload: config C2 of the baseline (fused GEMM + bias + GELU-tanh,
A[4096,4096] . W[4096,4096] bf16, fp32 accumulate, bf16 out), the
fused-GEMM half of the headline metric "flash-attn fwd & fused-GEMM TFLOP/s".
The other workloads are the remaining configs (C3 causal attention, C5
grouped-query causal attention, C4 MLP block, C1 fp32 attention).

One step = one pass of the hot path over one batch of synthetic input.  With
N GPUs (torchrun, one process per GPU, NCCL) every rank runs its own shard of
the token rows / (batch, head) units of a problem N times the single-GPU
size: weak scaling, no collective on the data path.  The output gather the
sharding implies is timed separately and reported under "gather".

Rank 0 prints one JSON line.  ``value`` is total TFLOP/s over all ranks
(algorithmic FLOPs / max-over-ranks device time of the K steps, inputs
resident in HBM, rotating input sets larger than L2 so no step starts warm).
``e2e`` is the same metric through the C ABI with host buffers: every step
copies its inputs from pinned host memory and reads the result back.

``--impl reference`` times the reference's own CPU kernels (compiled from
its sources into oracle/_ref) on the host cores, on a bounded sample of the
same workload, and prints the same line with "impl": "reference".
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["jules", "reference"], default="jules")
    p.add_argument("--workload", choices=["headline", "gemm", "attn", "attn_gqa", "mlp",
                                          "attn_fp32", "softmax", "xent", "int8", "fp8",
                                          "attn_bwd", "gemm_f32", "gelu_f32"],
                   default="headline")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    a = p.parse_args()
    a.warmup = max(a.warmup, 3)
    return a


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def measured_peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, FALLBACK_HBM_GBS, "fallback"


# fp32 CUDA-core peak for the C1 kernel (no measured fp32 figure exists):
# 148 SMs x 128 FP32 lanes x 2 FLOP (FMA) x 1965 MHz.
NOMINAL_FP32_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def roofline(wl, achieved, peak, peak_kind, traffic):
    """Roofline object of the dominant kernel: bf16 tensor kernels against the
    measured cuBLAS bf16 burst peak, the fp32 CUDA-core kernel (C1) against the
    nominal fp32 FMA peak."""
    if wl.unit == "TOPS":
        return {"bound": "tensor", "kernel": wl.dominant, "achieved": round(achieved, 2),
                "peak": NOMINAL_INT8_TOPS, "unit": "TOPS", "frac": round(achieved / NOMINAL_INT8_TOPS, 4),
                "peak_kind": "nominal dense int8 (datasheet; no measured int8 figure)",
                "traffic": traffic, "traffic_unit": "DRAM bytes per launch (ncu, profiles/)"}
    if wl.unit == "GB/s":
        hbm = measured_peaks()[1]
        return {"bound": "hbm", "kernel": wl.dominant, "achieved": round(achieved, 1),
                "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                "peak_kind": "measured HBM copy (MEASURED_PEAKS.json hbm_gbs)",
                "traffic": traffic, "traffic_unit": "DRAM bytes per launch (ncu, profiles/)"}
    if isinstance(wl, Fp8Gemm):
        return {"bound": "tensor", "kernel": wl.dominant, "achieved": round(achieved, 2),
                "peak": NOMINAL_FP8_TFLOPS, "unit": "TFLOP/s",
                "frac": round(achieved / NOMINAL_FP8_TFLOPS, 4),
                "peak_kind": "nominal dense fp8 (datasheet; no measured fp8 figure)",
                "traffic": traffic, "traffic_unit": "DRAM bytes per launch (ncu, profiles/)"}
    if getattr(wl, "tf32x3", False):
        p = peak / 2  # dense tf32 runs at half the bf16 rate per flop
        return {"bound": "tensor (tf32)", "kernel": wl.dominant, "achieved": round(achieved, 2),
                "peak": round(p, 1), "unit": "TFLOP/s", "frac": round(achieved / p, 4),
                "peak_kind": f"{peak_kind} cuBLAS bf16 burst / 2 (tf32 dense rate); achieved = "
                             "executed tf32 MMA flops (3 x 2MNK) per step",
                "traffic": traffic, "traffic_unit": "DRAM bytes per launch (ncu, profiles/)"}
    fp32 = isinstance(wl, (AttentionF32, GemmF32))
    p = NOMINAL_FP32_TFLOPS if fp32 else peak
    return {"bound": "fp32_cuda_cores" if fp32 else "tensor", "kernel": wl.dominant,
            "achieved": round(achieved, 2), "peak": round(p, 1), "unit": "TFLOP/s",
            "frac": round(achieved / p, 4),
            "peak_kind": ("nominal fp32 FMA, 148 SM x 128 lanes x 2 x 1965 MHz" if fp32
                          else f"{peak_kind} cuBLAS bf16 burst"),
            "traffic": traffic, "traffic_unit": "DRAM bytes per launch (ncu, profiles/)"}


def profiled_traffic(workload):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/<kernel>_<workload>.md, line 'traffic_bytes_per_launch:')."""
    name = {"gemm": "gemm_tc_c2", "attn": "attn_tc_c3", "attn_gqa": "attn_tc_c5",
            "mlp": "gemm_tc_c4", "attn_fp32": "attn_simt_c1", "softmax": "rows_softmax",
            "xent": "rows_xent", "int8": "gemm_s8_int8", "fp8": "gemm_f8_fp8",
            "attn_bwd": "attn_bwd_c3", "gemm_f32": "gemm_tf32x3_f32", "gelu_f32": "gelu_f32"}[workload]
    path = os.path.join(HERE, "profiles", f"{name}.md")
    try:
        with open(path) as f:
            for line in f:
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].strip().split()[0])
    except (OSError, ValueError):
        pass
    return None


def describe(workload, world, extra_l2=None, comm=None):
    """The config object of the JSON line (shared by both arms).  comm: the
    library's communicator, asked which gather route the workload's output
    takes (None: the reference arm)."""
    def how(out_bytes, kernel, what):
        route = comm.gather_route(out_bytes) if comm is not None else "stores"
        return {"stores": f"fused into the {kernel} epilogue as NVLink stores to each rank's {what}",
                "multicast": f"fused into the {kernel} epilogue as NVLink multicast stores (the "
                             f"NVSwitch writes each chunk into every rank's {what})",
                "pull": f"the {kernel} stores this rank's share, then the copy engines pull the "
                        f"other ranks' shares of {what} over NVLink"}[route]
    if workload in ("gemm", "headline"):
        c = {"workload": "C2 fused GEMM+bias+GELU(tanh)", "M": 4096, "N": 4096, "K": 4096,
             "M_per_rank": 4096 // world, "sharding": "rows of M (strong scaling: the global "
             "config split over the ranks)", "dtype_in": "bf16", "accumulate": "fp32",
             "dtype_out": "bf16"}
        if world > 1:
            c["gather"] = ("C gathered into every rank inside the timed step: "
                           + how(4096 * 4096 * 2, "GEMM", "C") + " (jules_dist_gemm_bias_act)")
    elif workload in ("attn", "attn_gqa"):
        gqa = workload == "attn_gqa"
        B, Hq, Hkv, S = (4, 64, 8, 16384) if gqa else (8, 32, 32, 4096)
        c = {"workload": ("C5 GQA causal flash-attention fwd + lse" if gqa else
                          "C3 causal flash-attention fwd + lse"),
             "B": B, "Hq": Hq, "Hkv": Hkv, "S": S, "D": 128,
             "units_per_rank": B * Hkv // world,
             "sharding": "(batch, kv head) units (strong scaling: the global config split over "
                         "the ranks)",
             "flop_convention": "causal = 2*B*Hq*S^2*D"}
        if world > 1:
            c["gather"] = ("O and lse gathered into every rank inside the timed step: "
                           + how(B * Hq * S * 128 * 2, "attention", "O and lse")
                           + " (jules_dist_flash_attention_fwd)")
    elif workload == "mlp":
        c = {"workload": "C4 MLP block LN->GEMM+b+GELU->GEMM+b+residual", "T_per_rank": 16384,
             "d": 4096, "dff": 16384, "global_T": 16384 * world, "sharding": "token rows",
             "eps": 1e-5}
    elif workload == "int8":
        c = {"workload": "int8 GEMM (matmulInt8): s8 x s8 -> s32 -> fp32 * scale + bias",
             "M_per_rank": 8192, "N": 8192, "K": 8192, "global_M": 8192 * world,
             "sharding": "rows of M", "op_convention": "2*M*N*K int8 ops"}
    elif workload == "attn_bwd":
        c = {"workload": "C3-shape causal flash-attention backward (dQ, dK, dV) bf16, from O and lse",
             "B_per_rank": 8, "Hq": 32, "Hkv": 32, "S": 4096, "D": 128, "global_B": 8 * world,
             "sharding": "batch x kv-head-group units",
             "flop_convention": "2.5 x causal forward = 5*B*Hq*S^2*D (5 GEMMs; the kernels "
                                "recompute S and dP for dQ, 7 GEMMs executed)"}
    elif workload == "fp8":
        c = {"workload": "fp8 GEMM + bias + GELU(tanh): e4m3 x e4m3 -> fp32 accumulate -> bf16",
             "M_per_rank": 8192, "N": 8192, "K": 8192, "global_M": 8192 * world,
             "sharding": "rows of M", "flop_convention": "2*M*N*K"}
    elif workload == "softmax":
        c = {"workload": "row softmax (fusedSoftmax), fp32", "M_per_rank": 16384, "N": 4096,
             "global_M": 16384 * world, "sharding": "rows",
             "bytes_convention": "M*N*4 read + M*N*4 written"}
    elif workload == "xent":
        c = {"workload": "fused softmax + cross-entropy (fusedCrossEntropyLoss), fp32 logits",
             "M_per_rank": 4096, "N": 32768, "global_M": 4096 * world, "sharding": "rows",
             "bytes_convention": "logits read + grad written + targets read"}
    elif workload == "gemm_f32":
        c = {"workload": "fp32 GEMM + bias + GELU (tiledMatmulWithActivation's float* path), "
                         "3xTF32 on tensor cores (rel-L2 <= 1e-5 against the reference)",
             "M_per_rank": 2048, "N": 2048, "K": 2048, "sharding": "rows of M"}
    elif workload == "gelu_f32":
        c = {"workload": "fp32 GELU (fusedGelu)", "n_per_rank": 64 << 20,
             "bytes_convention": "n*4 read + n*4 written"}
    else:
        c = {"workload": "C1 fp32 flash-attention fwd, non-causal", "B_per_rank": 1, "H": 8,
             "S": 512, "D": 64, "sharding": "batch"}
    c["parallelism"] = f"shard x{world}"
    if extra_l2:
        c["l2"] = extra_l2
    return c


# ---------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index, interval=0.0005):
        self.ok = False
        self.samples = []
        self.timed_from = None  # index of the first sample inside the timed region
        self.reasons = set()
        self.max_mhz = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass
        self.interval = interval
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self.REASONS.items():
                    if r & bit and k != "gpu_idle":
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(self.interval)

    def start(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def mark_timed(self):
        """The timed region starts now (warm-up samples come before it)."""
        self.timed_from = len(self.samples)

    def stop(self):
        if self._t:
            self._stop.set()
            self._t.join()
        timed = self.samples[self.timed_from:] if self.timed_from is not None else []
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_mhz_timed": statistics.median(timed) if timed else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples), "samples_timed": len(timed),
                "window": "warm-up and timed steps", "source": "nvml" if self.ok else "unavailable"}


# ---------------------------------------------------------------------------
# Workloads.  Each builds rotating input sets (> L2 in total), a device
# step, a host->device->host e2e step, and its FLOP count.
# ---------------------------------------------------------------------------
class Workload:
    name = ""
    dominant = ""
    launches_per_step = 1
    # Work accounting: flops_per_step / flops_dominant count FLOPs for the
    # tensor-core workloads and HBM bytes for the row-wise ones (unit GB/s).
    unit = "TFLOP/s"
    unit_scale = 1e12
    dtype = "bf16"

    def sets_for(self, bytes_per_set):
        return max(2, int((2 * L2_BYTES) // max(bytes_per_set, 1)) + 1)

    def e2e_spec(self):
        """(pinned host inputs, pinned host outputs, run(dev_inputs, dev_outputs)); run calls
        the public API on the current stream."""
        raise NotImplementedError


class E2EPipeline:
    """End-to-end steps through the public API with host buffers: each step
    copies its inputs host -> device, runs, and copies its result device ->
    host.  Two device buffer sets and three streams (H2D, compute, D2H)
    ordered by events, so step i's copies overlap steps i-1 and i+1 the way a
    serving loop overlaps them; every step still moves all of its bytes."""

    def __init__(self, torch, wl):
        self.t = torch
        self.h_in, h_out, self.run = wl.e2e_spec()
        self.h_out = [h_out, [torch.empty_like(h).pin_memory() for h in h_out]]
        self.sets = [([torch.empty_like(h, device="cuda") for h in self.h_in],
                      [torch.empty_like(h, device="cuda") for h in h_out]) for _ in range(2)]
        self.s_in, self.s_comp, self.s_out = (torch.cuda.Stream() for _ in range(3))
        E = torch.cuda.Event
        self.ev_in, self.ev_comp, self.ev_out = ([E(), E()] for _ in range(3))
        for k in range(2):  # first waits are satisfied
            self.ev_comp[k].record(self.s_comp)
            self.ev_out[k].record(self.s_out)
        self.h2d = sum(h.numel() * h.element_size() for h in self.h_in)
        self.d2h = sum(h.numel() * h.element_size() for h in h_out)
        self.i = 0

    def step(self):
        t, k = self.t, self.i % 2
        d_in, d_out = self.sets[k]
        with t.cuda.stream(self.s_in):
            self.s_in.wait_event(self.ev_comp[k])   # step i-2's compute has read d_in
            for h, d in zip(self.h_in, d_in):
                d.copy_(h, non_blocking=True)
            self.ev_in[k].record(self.s_in)
        with t.cuda.stream(self.s_comp):
            self.s_comp.wait_event(self.ev_in[k])
            self.s_comp.wait_event(self.ev_out[k])  # step i-2's D2H has read d_out
            self.run(d_in, d_out)
            self.ev_comp[k].record(self.s_comp)
        with t.cuda.stream(self.s_out):
            self.s_out.wait_event(self.ev_comp[k])
            for h, d in zip(self.h_out[k], d_out):
                h.copy_(d, non_blocking=True)
            self.ev_out[k].record(self.s_out)
        self.i += 1

    def time_steps(self, n):
        """Device time of n steps (first H2D start to last D2H end), ms."""
        t = self.t
        t.cuda.synchronize()
        e0, e1 = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
        e0.record(self.s_in)
        for _ in range(n):
            self.step()
        e1.record(self.s_out)  # after the last D2H, which follows every earlier op
        t.cuda.synchronize()
        return e0.elapsed_time(e1)


class Gemm(Workload):
    """C2: C = GELU(A.W + bias), M=N=K=4096.  With N GPUs the same global
    problem is split by rows of M (strong scaling): each rank computes its
    4096/N rows and the gather of C into every rank is fused into the GEMM
    (jules_dist_gemm_bias_act on shared output buffers), so a step is the
    whole distributed op, gather included."""
    dominant = "gemm_bf16_tc2_kernel (CTA pair)"
    global_work = True

    def __init__(self, jb, torch, rank, world, M=4096, N=4096, K=4096, dist=None):
        self.jb, self.torch = jb, torch
        self.M, self.N, self.K = M, N, K
        self.world, self.dist = world, dist
        if world > 1:
            self.dominant = "gemm_bf16_tc2_kernel (CTA pair) + fused gather to every rank"
            self.launches_per_step = 2  # the GEMM and the one-thread signal/wait kernel
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(1234)  # the same problem on every rank
        per_set = (M * K + K * N + M * N) * 2
        self.nsets = self.sets_for(per_set)
        s = 1.0 / K ** 0.5
        self.A = [((torch.rand((M, K), generator=g, device=dev) * 2 - 1) * s).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        # W and bias are replicated (one copy per rank); distinct copies per set
        # keep every step cold in L2.
        self.W = [((torch.rand((K, N), generator=g, device=dev) * 2 - 1) * s).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.b = [torch.randn(N, generator=g, device=dev) * 0.02 for _ in range(self.nsets)]
        if world > 1:
            self.C = [dist.alloc_shared((M, N), torch.bfloat16) for _ in range(self.nsets)]
        else:
            self.C = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(self.nsets)]
        self.rows = jb.dist_shard(M, world, rank)
        self.flops_per_step = 2.0 * M * N * K  # the whole job's work per step
        self.flops_dominant = 2.0 * (self.rows[1] - self.rows[0]) * N * K  # this rank's GEMM
        self.config = {"l2": f"{self.nsets} rotating input sets ({self.nsets * per_set / 2**20:.0f} MiB > L2)"}

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        if self.world > 1:
            self.dist.gemm_bias_act(self.A[k], self.W[k], self.b[k], act="gelu", out=self.C[k])
        else:
            self.jb.gemm_bias_act(self.A[k], self.W[k], self.b[k], act="gelu", out=self.C[k])
        if ev:
            ev[1].record()

    def compute_only(self, i):
        """This rank's rows without the gather (the compute half of a step)."""
        k = i % self.nsets
        a, b = self.rows
        if not hasattr(self, "Cl"):
            self.Cl = self.torch.empty((b - a, self.N), dtype=self.torch.bfloat16, device="cuda")
        self.jb.gemm_bias_act(self.A[k][a:b], self.W[k], self.b[k], act="gelu", out=self.Cl)

    def release(self):
        if self.world > 1:
            for c in self.C:
                self.dist.free_shared(c)
            self.C = []

    def output(self, i):
        return self.C[i % self.nsets]

    # e2e through the C ABI with host buffers: each step copies A in and C
    # out; W and bias (the replicated weights) are resident, copied once
    # before timing, as in the multi-GPU e2e
    def e2e_spec(self):
        jb = self.jb
        h_in = [self.A[0].cpu().pin_memory()]
        h_out = [self.torch.empty((self.M, self.N), dtype=self.torch.bfloat16).pin_memory()]
        return h_in, h_out, lambda d, o: jb.gemm_bias_act(d[0], self.W[0], self.b[0], act="gelu",
                                                          out=o[0])

    def e2e_dist_spec(self):
        """N > 1: each step copies this rank's rows of A in, runs the sharded
        call (gather fused) and rank 0 reads the whole C back; W and bias are
        replicated once, outside timing."""
        a, b = self.rows
        d_in = self.A[0]
        ins = [(d_in[a:b].cpu().pin_memory(), d_in[a:b])]
        # Two output buffers in turn: while rank 0 reads step s's C, the other
        # ranks may already write step s+1's into the other buffer (they
        # cannot reach step s+2 before rank 0 has signalled s+1, which it
        # does only after its read of step s).
        h_out = self.torch.empty((self.M, self.N), dtype=self.torch.bfloat16).pin_memory()
        outs = [(h_out, self.C[0])]
        state = {"i": 0}

        def run():
            k = state["i"] % 2
            state["i"] += 1
            outs[0] = (h_out, self.C[k])
            self.dist.gemm_bias_act(d_in, self.W[0], self.b[0], act="gelu", out=self.C[k])

        return ins, outs, run


class Attention(Workload):
    """C3 (attn) / C5 (attn_gqa): causal bf16 flash-attention fwd + lse;
    (batch, kv-head group) units sharded across ranks."""
    dominant = "attn_fwd_tc_kernel"

    global_work = True

    def __init__(self, jb, torch, rank, world, gqa=False, dist=None):
        self.jb, self.torch = jb, torch
        self.world, self.dist = world, dist
        if gqa:
            B, Hq, Hkv, S = 4, 64, 8, 16384
            # 32 (b, kv-group) units; each rank owns 32/world of them, run as
            # B_r = 4/world batches when world <= 4, else a head-group slice.
            self.units = 32
        else:
            B, Hq, Hkv, S = 8, 32, 32, 4096
            self.units = B
        D = 128
        self.global_shape = (B, Hq, Hkv, S, D)
        # the global problem on every rank; with N GPUs each computes its
        # (batch, kv head) units and the outputs are gathered (strong scaling)
        self.B, self.Hq, self.Hkv, self.S, self.D = B, Hq, Hkv, S, D
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(77)
        per_set = (B * Hq * S * D * 2 + 2 * B * Hkv * S * D) * 2
        self.nsets = 1 if per_set > L2_BYTES else self.sets_for(per_set)
        self.Q = [torch.randn((B, Hq, S, D), generator=g, device=dev).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        self.Kt = [torch.randn((B, Hkv, S, D), generator=g, device=dev).to(torch.bfloat16)
                   for _ in range(self.nsets)]
        self.V = [torch.randn((B, Hkv, S, D), generator=g, device=dev).to(torch.bfloat16)
                  for _ in range(self.nsets)]
        if world > 1:  # every rank's O and lse writable by all: the gather fused in
            self.O = [dist.alloc_shared((B, Hq, S, D), torch.bfloat16) for _ in self.Q]
            self.L = [dist.alloc_shared((B, Hq, S), torch.float32) for _ in self.Q]
        else:
            self.O = [torch.empty_like(q) for q in self.Q]
            self.L = [torch.empty((B, Hq, S), dtype=torch.float32, device=dev) for _ in self.Q]
        # causal FLOPs, FlashAttention convention: 2 * B*H*S^2*D
        self.flops_per_step = 2.0 * B * Hq * S * S * D
        self.flops_dominant = self.flops_per_step / world
        if world > 1:
            self.dominant = "attn_fwd_tc_kernel + fused gather to every rank"
            self.launches_per_step = 2  # attention and the one-thread signal/wait kernel
        self.config = {"workload": ("C5 GQA causal flash-attention fwd + lse" if gqa else
                                    "C3 causal flash-attention fwd + lse"),
                       "B_per_rank": B, "Hq": Hq, "Hkv": Hkv, "S": S, "D": D,
                       "global_B": B * world, "sharding": "batch x kv-head-group units",
                       "flop_convention": "causal = 2*B*Hq*S^2*D",
                       "l2": f"inputs {per_set / 2**20:.0f} MiB per step (> L2)"
                       if self.nsets == 1 else f"{self.nsets} rotating input sets"}

    def _run(self, Q, K, V, O, L):
        """The C ABI call: causal forward writing O and the fp32 logsumexp
        (sharded over the ranks, O and lse gathered, when N > 1)."""
        jb = self.jb
        if self.world > 1:
            self.dist.flash_attention_fwd(Q, K, V, causal=True, out=O, lse=L)
            return
        rc = jb.lib().jules_flash_attention_fwd(
            jb._ptr(Q), jb._ptr(K), jb._ptr(V), jb._ptr(O), jb._ptr(L), self.B, self.Hq,
            self.Hkv, self.S, self.D, 0.0, 1, jb.DT_BF16, jb._stream(None))
        jb._check(rc, "jules_flash_attention_fwd")

    def release(self):
        if self.world > 1:
            for t in self.O + self.L:
                self.dist.free_shared(t)
            self.O, self.L = [], []

    def compute_only(self, i):
        """This rank's (batch, kv head) units without the gather."""
        units = self.B * self.Hkv
        a, b = self.jb.dist_shard(units, self.world, self.dist.rank)
        G = self.Hq // self.Hkv
        v4 = lambda x, g: x.view(units, g, self.S, self.D)[a:b]
        k = i % self.nsets
        jb = self.jb
        rc = jb.lib().jules_flash_attention_fwd(
            jb._ptr(v4(self.Q[k], G)), jb._ptr(v4(self.Kt[k], 1)), jb._ptr(v4(self.V[k], 1)),
            jb._ptr(v4(self.O[k], G)), jb._ptr(self.L[k].view(units, G, self.S)[a:b]), b - a, G, 1,
            self.S, self.D, 0.0, 1, jb.DT_BF16, jb._stream(None))
        jb._check(rc, "jules_flash_attention_fwd")

    def e2e_dist_spec(self):
        """N > 1: each step copies this rank's units of Q, K, V in, runs the
        sharded call and rank 0 reads the whole O and lse back."""
        t = self.torch
        units = self.B * self.Hkv
        a, b = self.jb.dist_shard(units, self.world, self.dist.rank)
        G = self.Hq // self.Hkv
        q = self.Q[0].view(units, G, self.S, self.D)
        kv = lambda x: x.view(units, 1, self.S, self.D)
        ins = [(q[a:b].cpu().pin_memory(), q[a:b]), (kv(self.Kt[0])[a:b].cpu().pin_memory(), kv(self.Kt[0])[a:b]),
               (kv(self.V[0])[a:b].cpu().pin_memory(), kv(self.V[0])[a:b])]
        outs = [(t.empty_like(self.O[0], device="cpu").pin_memory(), self.O[0]),
                (t.empty_like(self.L[0], device="cpu").pin_memory(), self.L[0])]
        run = lambda: self._run(self.Q[0], self.Kt[0], self.V[0], self.O[0], self.L[0])
        return ins, outs, run

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self._run(self.Q[k], self.Kt[k], self.V[k], self.O[k], self.L[k])
        if ev:
            ev[1].record()

    def output(self, i):
        return self.O[i % self.nsets]

    def e2e_spec(self):
        h_in = [x[0].cpu().pin_memory() for x in (self.Q, self.Kt, self.V)]
        h_out = [self.torch.empty_like(h_in[0]).pin_memory(),
                 self.torch.empty_like(self.L[0], device="cpu").pin_memory()]
        return h_in, h_out, lambda d, o: self._run(d[0], d[1], d[2], o[0], o[1])


class AttentionF32(Workload):
    """C1: fp32 [1,8,512,64] non-causal (CUDA cores)."""
    dominant = "attn_tile_kernel<float, float, 64>"

    def __init__(self, jb, torch, rank, world):
        self.jb, self.torch = jb, torch
        B, H, S, D = 1, 8, 512, 64
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(5 + rank)
        per_set = 4 * B * H * S * D * 4
        self.nsets = self.sets_for(per_set)
        self.Q = [torch.randn((B, H, S, D), generator=g, device=dev) for _ in range(self.nsets)]
        self.Kt = [torch.randn((B, H, S, D), generator=g, device=dev) for _ in range(self.nsets)]
        self.V = [torch.randn((B, H, S, D), generator=g, device=dev) for _ in range(self.nsets)]
        self.O = [torch.empty_like(q) for q in self.Q]
        self.flops_per_step = 4.0 * B * H * S * S * D
        self.flops_dominant = self.flops_per_step
        self.config = {"workload": "C1 fp32 flash-attention fwd, non-causal", "B_per_rank": B,
                       "H": H, "S": S, "D": D, "sharding": "batch",
                       "l2": f"{self.nsets} rotating input sets"}

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self.jb.flash_attention_fwd(self.Q[k], self.Kt[k], self.V[k], causal=False, out=self.O[k],
                                    lse=False)
        if ev:
            ev[1].record()

    def output(self, i):
        return self.O[i % self.nsets]

    def e2e_spec(self):
        jb = self.jb
        h_in = [x[0].cpu().pin_memory() for x in (self.Q, self.Kt, self.V)]
        h_out = [self.torch.empty_like(h_in[0]).pin_memory()]
        return h_in, h_out, lambda d, o: jb.flash_attention_fwd(d[0], d[1], d[2], causal=False,
                                                                 out=o[0], lse=False)


class Mlp(Workload):
    """C4: out = GELU(LN(X).W1 + b1).W2 + b2 + X, T=16384 tokens per rank,
    d=4096, dff=16384 (token rows sharded).  Runs jules_mlp_block_folded:
    a row-statistics pass over X, GEMM1 on the raw rows with the LayerNorm
    applied in its epilogue (weights folded once, outside timing), GEMM2 +
    bias + residual."""
    dominant = ("jules_mlp_block_folded (layernorm_bf16_warp_kernel stats + 2 x "
                "gemm_bf16_tc2_kernel)")
    launches_per_step = 3

    def __init__(self, jb, torch, rank, world, T=16384, d=4096, dff=16384):
        self.jb, self.torch = jb, torch
        self.T, self.d, self.dff = T, d, dff
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(99 + rank)
        self.X = torch.randn((T, d), generator=g, device=dev).to(torch.bfloat16)
        self.gam = 1 + 0.02 * torch.randn(d, generator=g, device=dev)
        self.bet = 0.02 * torch.randn(d, generator=g, device=dev)
        self.W1 = (0.02 * torch.randn((d, dff), generator=g, device=dev)).to(torch.bfloat16)
        self.b1 = 0.02 * torch.randn(dff, generator=g, device=dev)
        self.W2 = (0.02 * torch.randn((dff, d), generator=g, device=dev)).to(torch.bfloat16)
        self.b2 = 0.02 * torch.randn(d, generator=g, device=dev)
        self.out = torch.empty_like(self.X)
        self.folded = jb.mlp_block_fold_weights(self.gam, self.bet, self.W1, self.b1)
        self.ws = torch.empty(int(jb.lib().jules_mlp_block_folded_workspace_bytes(T, d, dff)),
                              dtype=torch.uint8, device=dev)
        self.nsets = 1
        self.flops_per_step = 16.0 * T * d * d * (dff / (4 * d))
        self.flops_dominant = self.flops_per_step
        self.config = {"workload": "C4 MLP block LN->GEMM+b+GELU->GEMM+b+residual",
                       "T_per_rank": T, "d": d, "dff": dff, "global_T": T * world,
                       "sharding": "token rows", "eps": 1e-5,
                       "l2": "inputs 1.4 GB per step (> L2)"}

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self.jb.mlp_block_folded(self.X, self.folded, self.W2, self.b2, out=self.out,
                                 workspace=self.ws)
        if ev:
            ev[1].record()

    def output(self, i):
        return self.out

    def e2e_spec(self):
        jb, t = self.jb, self.torch
        h_in = [self.X.cpu().pin_memory()]   # weights stay resident
        h_out = [t.empty_like(h_in[0]).pin_memory()]
        return h_in, h_out, lambda d, o: jb.mlp_block_folded(d[0], self.folded, self.W2, self.b2,
                                                              out=o[0], workspace=self.ws)


class Int8Gemm(Workload):
    """int8 GEMM, M = N = K = 8192 per rank (rows of M sharded): tcgen05
    kind::i8.  Counted in int8 ops (2*M*N*K), reported as TOPS."""
    unit = "TOPS"
    dtype = "s8"
    dominant = "gemm_s8_tc2_kernel<6>"

    def __init__(self, jb, torch, rank, world, M=8192, N=8192, K=8192):
        self.jb, self.torch = jb, torch
        self.M, self.N, self.K = M, N, K
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(8 + rank)
        per_set = M * K + K * N + M * N * 4
        self.nsets = self.sets_for(per_set)
        self.A = [torch.randint(-128, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
                  for _ in range(self.nsets)]
        self.B = [torch.randint(-128, 128, (K, N), generator=g, device=dev, dtype=torch.int8)
                  for _ in range(self.nsets)]
        self.bias = torch.randn(N, generator=g, device=dev)
        self.C = [torch.empty((M, N), dtype=torch.float32, device=dev) for _ in range(self.nsets)]
        self.flops_per_step = 2.0 * M * N * K
        self.flops_dominant = self.flops_per_step
        self.config = {"l2": f"{self.nsets} rotating input sets ({self.nsets * per_set / 2**20:.0f} MiB > L2)"}

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self.jb.matmul_int8(self.A[k], self.B[k], 0.01, 0.02, self.bias, out=self.C[k])
        if ev:
            ev[1].record()

    def output(self, i):
        return self.C[i % self.nsets]

    def e2e_spec(self):
        jb = self.jb
        h_in = [self.A[0].cpu().pin_memory(), self.B[0].cpu().pin_memory()]
        h_out = [self.torch.empty_like(self.C[0], device="cpu").pin_memory()]
        return h_in, h_out, lambda d, o: jb.matmul_int8(d[0], d[1], 0.01, 0.02, self.bias, out=o[0])


class Fp8Gemm(Workload):
    """fp8 GEMM + bias + GELU, M = N = K = 8192 per rank (rows of M sharded):
    E4M3 operands (the mixed-precision pass's fp8 target), fp32 accumulation
    on tcgen05 kind::f8f6f4, bf16 output."""
    dtype = "e4m3"
    dominant = "gemm_f8_tc2_kernel<6, bf16>"

    def __init__(self, jb, torch, rank, world, M=8192, N=8192, K=8192):
        self.jb, self.torch = jb, torch
        self.M, self.N, self.K = M, N, K
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(9 + rank)
        per_set = M * K + K * N + M * N * 2
        self.nsets = self.sets_for(per_set)
        f8 = torch.float8_e4m3fn
        self.A = [torch.randn((M, K), generator=g, device=dev).to(f8) for _ in range(self.nsets)]
        self.B = [(torch.randn((K, N), generator=g, device=dev) / 16).to(f8)
                  for _ in range(self.nsets)]
        self.bias = 0.02 * torch.randn(N, generator=g, device=dev)
        self.C = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _ in range(self.nsets)]
        self.scale = 1.0 / 8.0
        self.flops_per_step = 2.0 * M * N * K
        self.flops_dominant = self.flops_per_step
        self.config = {"l2": f"{self.nsets} rotating input sets ({self.nsets * per_set / 2**20:.0f} MiB > L2)"}

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self.jb.gemm_fp8(self.A[k], self.B[k], self.bias, act="gelu", scale=self.scale,
                         out=self.C[k])
        if ev:
            ev[1].record()

    def output(self, i):
        return self.C[i % self.nsets]

    def e2e_spec(self):
        jb = self.jb
        h_in = [self.A[0].cpu().pin_memory(), self.B[0].cpu().pin_memory()]
        h_out = [self.torch.empty_like(self.C[0], device="cpu").pin_memory()]
        return h_in, h_out, lambda d, o: jb.gemm_fp8(d[0], d[1], self.bias, act="gelu",
                                                      scale=self.scale, out=o[0])


class AttentionBwd(Workload):
    """Causal flash-attention backward at the C3 shape (B=8, H=32, S=4096,
    D=128, bf16): dQ, dK, dV from Q, K, V, O, dO and lse.  Timed unit: the
    whole jules_flash_attention_bwd call (prep + dK/dV + dQ kernels)."""
    dominant = "jules_flash_attention_bwd (bwd_dkdv_kernel + bwd_dq_kernel + bwd_prep_kernel)"
    launches_per_step = 3

    def __init__(self, jb, torch, rank, world, B=8, H=32, S=4096, D=128):
        self.jb, self.torch = jb, torch
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(77 + rank)
        bf = torch.bfloat16
        mk = lambda: torch.randn((B, H, S, D), generator=g, device=dev).to(bf)
        self.Q, self.K, self.V, self.dO = mk(), mk(), mk(), mk()
        self.O, self.lse = jb.flash_attention_fwd(self.Q, self.K, self.V, causal=True)
        self.grads = (torch.empty_like(self.Q), torch.empty_like(self.K), torch.empty_like(self.V))
        self.ws = torch.empty(jb.lib().jules_flash_attention_bwd_workspace_bytes(B, H, S, D, jb.DT_BF16),
                              dtype=torch.uint8, device=dev)
        self.nsets = 1
        self.flops_per_step = 5.0 * B * H * S * S * D
        self.flops_dominant = self.flops_per_step
        self.config = {"l2": "inputs 1.6 GB per step (> L2)"}

    def step(self, i, ev=None):
        if ev:
            ev[0].record()
        self.jb.flash_attention_bwd(self.Q, self.K, self.V, self.O, self.dO, self.lse, causal=True,
                                    workspace=self.ws, out=self.grads)
        if ev:
            ev[1].record()

    def output(self, i):
        return self.grads[0]

    def e2e_spec(self):
        jb = self.jb
        h_in = [x.cpu().pin_memory() for x in (self.Q, self.K, self.V, self.O, self.dO, self.lse)]
        h_out = [self.torch.empty_like(x, device="cpu").pin_memory() for x in self.grads]
        return h_in, h_out, lambda d, o: jb.flash_attention_bwd(*d, causal=True, workspace=self.ws,
                                                                 out=tuple(o))


class RowWise(Workload):
    """Row softmax (softmax) or fused softmax + cross-entropy (xent), fp32,
    rows sharded across ranks.  HBM-bound: work is counted in bytes."""
    unit = "GB/s"
    unit_scale = 1e9
    dtype = "f32"

    def __init__(self, jb, torch, rank, world, xent=False):
        self.jb, self.torch, self.xent = jb, torch, xent
        M, N = (4096, 32768) if xent else (16384, 4096)
        self.M, self.N = M, N
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(31 + rank)
        per_set = 2 * M * N * 4
        self.nsets = 1 if per_set > L2_BYTES else self.sets_for(per_set)
        self.X = [3 * torch.randn((M, N), generator=g, device=dev) for _ in range(self.nsets)]
        self.Y = [torch.empty_like(x) for x in self.X]
        self.T = [torch.randint(0, N, (M,), generator=g, device=dev, dtype=torch.int32)
                  for _ in range(self.nsets)]
        self.loss = torch.empty((), dtype=torch.float32, device=dev)
        self.flops_per_step = 2.0 * M * N * 4 + (M * 4 if xent else 0)  # bytes
        self.flops_dominant = self.flops_per_step
        self.dominant = ("softmax_stage_kernel<1024, 8, float, true> (cross-entropy)" if xent
                         else "softmax_reg_kernel<256, 4, float, false>")
        self.config = {"l2": f"inputs {per_set / 2**20:.0f} MiB per step (> L2)"
                       if self.nsets == 1 else f"{self.nsets} rotating input sets"}

    def _run(self, x, y, t):
        if self.xent:
            rc = self.jb.lib().jules_cross_entropy_loss(
                self.jb._ptr(x), self.jb._ptr(t), self.jb._ptr(y), self.jb._ptr(self.loss),
                self.M, self.N, self.jb.DT_F32, self.jb._stream(None))
            self.jb._check(rc, "jules_cross_entropy_loss")
        else:
            self.jb.softmax(x, out=y)

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self._run(self.X[k], self.Y[k], self.T[k])
        if ev:
            ev[1].record()

    def output(self, i):
        return self.Y[i % self.nsets]

    def e2e_spec(self):
        h_in = [self.X[0].cpu().pin_memory()] + ([self.T[0].cpu().pin_memory()] if self.xent else [])
        h_out = [self.torch.empty_like(h_in[0]).pin_memory()]
        return h_in, h_out, lambda d, o: self._run(d[0], o[0], d[1] if self.xent else None)


class GemmF32(Workload):
    """The reference's float* GEMM path (tiledMatmulWithActivation with GELU,
    fp32 in and out) at its 1e-5 rel-L2 bar: 3xTF32 on tensor cores
    (jules_gemm_f32_tc: operand split, then the tcgen05 pair GEMM on
    kind::tf32 over K' = 3K).  M = N = K = 2048 per rank.  The exact fp32
    CUDA-core kernel is timed beside it (cuda_core_exact)."""
    dtype = "f32"
    dominant = ("split3_a/w_kernel + gemm_bf16_tc2_kernel<float> (tcgen05 kind::tf32, 3xTF32; "
                "events bracket the split and the GEMM)")
    tf32x3 = True

    def __init__(self, jb, torch, rank, world, M=2048, N=2048, K=2048):
        self.jb, self.torch = jb, torch
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(21 + rank)
        per_set = (M * K + K * N + M * N) * 4
        self.nsets = self.sets_for(per_set)
        s = 1.0 / K ** 0.5
        self.A = [(torch.rand((M, K), generator=g, device=dev) * 2 - 1) * s for _ in range(self.nsets)]
        self.W = [(torch.rand((K, N), generator=g, device=dev) * 2 - 1) * s for _ in range(self.nsets)]
        self.b = torch.randn(N, generator=g, device=dev) * 0.02
        self.C = [torch.empty((M, N), device=dev) for _ in range(self.nsets)]
        self.ws = torch.empty(jb.gemm_f32_tc_workspace_bytes(M, N, K), dtype=torch.uint8, device=dev)
        # two split kernels and one GEMM per 1024-column K chunk
        self.launches_per_step = 2 + (K + 1023) // 1024
        self.flops_per_step = 2.0 * M * N * K
        # executed tf32 MMA work: three products over K
        self.flops_dominant = 3 * self.flops_per_step
        self.config = {"l2": f"{self.nsets} rotating input sets ({self.nsets * per_set / 2**20:.0f} MiB > L2)"}

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self.jb.gemm_f32_tc(self.A[k], self.W[k], self.b, act="gelu", out=self.C[k], workspace=self.ws)
        if ev:
            ev[1].record()

    def extra_measure(self):
        """The exact fp32 CUDA-core GEMM on the same inputs (fp32 FMA
        products), for comparison: TFLOP/s over 10 calls after 3."""
        torch = self.torch
        for i in range(3):
            self.jb.gemm_bias_act(self.A[i % self.nsets], self.W[i % self.nsets], self.b, act="gelu",
                                  out=self.C[i % self.nsets])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(10):
            self.jb.gemm_bias_act(self.A[i % self.nsets], self.W[i % self.nsets], self.b, act="gelu",
                                  out=self.C[i % self.nsets])
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 10
        return {"kernel": "simt::gemm_kernel<float, float> (fp32 CUDA cores, exact products)",
                "ms": round(ms, 4), "tflops": round(self.flops_per_step / (ms * 1e-3) / 1e12, 2)}

    def output(self, i):
        return self.C[i % self.nsets]

    def e2e_spec(self):
        jb = self.jb
        h_in = [self.A[0].cpu().pin_memory(), self.W[0].cpu().pin_memory()]
        h_out = [self.torch.empty_like(self.C[0], device="cpu").pin_memory()]
        return h_in, h_out, lambda d, o: jb.gemm_f32_tc(d[0], d[1], self.b, act="gelu", out=o[0],
                                                        workspace=self.ws)


class GeluF32(Workload):
    """The reference's fusedGelu over 64 Mi fp32 elements (HBM-bound, GB/s)."""
    unit = "GB/s"
    unit_scale = 1e9
    dtype = "f32"
    dominant = "simt::gelu_kernel<float>"

    def __init__(self, jb, torch, rank, world, n=64 << 20):
        self.jb, self.torch = jb, torch
        dev = torch.device("cuda")
        g = torch.Generator(device=dev).manual_seed(22 + rank)
        self.X = [torch.randn(n, generator=g, device=dev) * 3 for _ in range(2)]
        self.Y = [torch.empty_like(x) for x in self.X]
        self.nsets = 2
        self.flops_per_step = 2.0 * n * 4  # bytes read + written
        self.flops_dominant = self.flops_per_step
        self.config = {"l2": "inputs 256 MiB per step (> L2)"}

    def step(self, i, ev=None):
        k = i % self.nsets
        if ev:
            ev[0].record()
        self.jb.gelu(self.X[k], out=self.Y[k])
        if ev:
            ev[1].record()

    def output(self, i):
        return self.Y[i % self.nsets]

    def e2e_spec(self):
        h_in = [self.X[0].cpu().pin_memory()]
        h_out = [self.torch.empty_like(h_in[0]).pin_memory()]
        return h_in, h_out, lambda d, o: self.jb.gelu(d[0], out=o[0])


METRIC = "Flash-attn fwd & fused-GEMM TFLOP/s at 1/2/4/8 B200; % of tensor peak"
# Extra (non-headline) workloads of the row-wise kernels report HBM bytes per second.
ROWS_METRIC = "Row softmax / fused cross-entropy GB/s (HBM bytes moved) per B200"
INT8_METRIC = "int8 GEMM TOPS (matmulInt8) per B200"
FP8_METRIC = "fp8 GEMM + bias + GELU TFLOP/s (mixed-precision matmul at fp8) per B200"
BWD_METRIC = "Flash-attention backward (dQ, dK, dV) TFLOP/s per B200; % of tensor peak"


F32_GEMM_METRIC = "fp32 GEMM + bias + GELU TFLOP/s (the reference's float* API) per B200"
GELU_METRIC = "fp32 GELU GB/s (HBM bytes moved) per B200"


def metric_for(workload):
    if workload in ("softmax", "xent"):
        return ROWS_METRIC
    if workload == "gemm_f32":
        return F32_GEMM_METRIC
    if workload == "gelu_f32":
        return GELU_METRIC
    return {"int8": INT8_METRIC, "fp8": FP8_METRIC, "attn_bwd": BWD_METRIC}.get(workload, METRIC)
# B200 datasheet dense int8 / fp8 tensor throughput (no measured figures on this pool).
NOMINAL_INT8_TOPS = 4500.0
NOMINAL_FP8_TFLOPS = 4500.0
# The reference has no fp8 kernel (its mixed-precision pass only names the
# types), so the fp8 CPU leg times the oracle's restatement ("port").
CPU_KIND = {"fp8": "port", "attn_bwd": "port"}
JSON_OUT = sys.stdout


def emit(line):
    print(json.dumps(line), file=JSON_OUT, flush=True)


# ---------------------------------------------------------------------------
# CPU baseline: the reference's own kernels (oracle/_ref) on the host cores.
# ---------------------------------------------------------------------------
def cpu_reference_sample(workload, reps=3, warm=1):
    """Times the reference CPU path on a bounded sample; returns
    (TFLOP/s, description, threads)."""
    import numpy as np
    sys.path.insert(0, os.path.join(HERE, "oracle"))
    import oracle
    threads = os.cpu_count() or 1
    ref = oracle.Reference()
    ref.set_threads(threads)  # all host threads, whatever OMP_NUM_THREADS says
    g = np.random.default_rng(0)
    if workload in ("gemm", "mlp"):
        if workload == "gemm":
            Ms, N, K = 1024, 4096, 4096
            desc = (f"reference tiledMatmulWithActivation + bias + fusedGelu "
                    f"(FusedKernels.h:378-458,606-627) on {Ms} of the 4096 rows of C2")
        else:
            Ms, N, K = 256, 16384, 4096
            desc = ("reference tiledMatmulWithActivation + bias + fusedGelu on 256 of the "
                    "16384 token rows of C4's GEMM1 (4096->16384); C4 FLOPs scale per row")
        A = (g.uniform(-1, 1, (Ms, K)) / np.sqrt(K)).astype(np.float32)
        W = (g.uniform(-1, 1, (K, N)) / np.sqrt(K)).astype(np.float32)
        b = (0.02 * g.standard_normal(N)).astype(np.float32)
        fn = lambda: ref.gemm_bias_gelu(A, W, b)
        flops = 2.0 * Ms * N * K
    elif workload == "int8":
        Ms, N, K = 16, 8192, 8192
        A = g.integers(-128, 128, (Ms, K)).astype(np.int8)
        B = g.integers(-128, 128, (K, N)).astype(np.int8)
        bias = g.standard_normal(N).astype(np.float32)
        # the scalar build: the AVX-512 build's int8 branches compute a different product
        ref8 = oracle.Reference(variant="avx2")
        ref8.set_threads(threads)
        fn = lambda: ref8.matmul_int8(A, B, 0.01, 0.02, bias)
        flops = 2.0 * Ms * N * K
        desc = (f"reference matmulInt8 (FusedKernels.h:867-1073, scalar branch) on {Ms} of the "
                f"8192 rows; ops 2*M*N*K")
        reps = 2
    elif workload == "fp8":
        Ms, N, K = 16, 8192, 8192
        R = oracle.Restated()
        A = R.fp8_encode(g.standard_normal((Ms, K)).astype(np.float32), "e4m3")
        B = R.fp8_encode((g.standard_normal((K, N)) / 16).astype(np.float32), "e4m3")
        bias = (0.02 * g.standard_normal(N)).astype(np.float32)
        fn = lambda: R.gemm_fp8(A, B, "e4m3", "e4m3", bias, None, "gelu", 1.0 / 8.0)
        flops = 2.0 * Ms * N * K
        desc = (f"oracle restatement orc_gemm_fp8 (oracle/restate.c; the reference has no fp8 "
                f"kernel) on {Ms} of the 8192 rows; FLOPs 2*M*N*K")
        reps = 2
    elif workload == "attn_bwd":
        Sx = 2048
        R = oracle.Restated()
        Q, K_, V, dO = (g.standard_normal((1, 1, Sx, 128), dtype=np.float32) for _ in range(4))
        fn = lambda: R.attention_bwd(Q, K_, V, dO, causal=True)
        flops = 5.0 * Sx * Sx * 128
        desc = (f"oracle restatement orc_attention_bwd (oracle/restate.c, double; the reference "
                f"has no attention backward) on one (b,h) unit at S={Sx}, D=128, causal; "
                f"FLOPs 5*S^2*D")
        reps = 2
    elif workload in ("softmax", "xent"):
        if workload == "softmax":
            Ms, N = 2048, 4096
            X = (3 * g.standard_normal((Ms, N))).astype(np.float32)
            fn = lambda: ref.softmax(X)
            desc = f"reference fusedSoftmax (FusedKernels.h:464-526) on {Ms} of the 16384 rows"
        else:
            Ms, N = 512, 32768
            X = (3 * g.standard_normal((Ms, N))).astype(np.float32)
            T = g.integers(0, N, Ms).astype(np.int32)
            fn = lambda: ref.cross_entropy(X, T)
            desc = f"reference fusedCrossEntropyLoss (FusedKernels.h:766-854) on {Ms} of the 4096 rows"
        flops = 2.0 * Ms * N * 4  # bytes, reported in GB/s below
        reps = 5
        for _ in range(warm):
            fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        dt = (time.perf_counter() - t0) / reps
        return flops / dt / 1e9, desc + f"; {reps} timed reps, {dt * 1e3:.1f} ms each", threads
    elif workload == "gemm_f32":
        Ms, N, K = 512, 2048, 2048
        A = (g.uniform(-1, 1, (Ms, K)) / np.sqrt(K)).astype(np.float32)
        W = (g.uniform(-1, 1, (K, N)) / np.sqrt(K)).astype(np.float32)
        b = (0.02 * g.standard_normal(N)).astype(np.float32)
        fn = lambda: ref.gemm_bias_gelu(A, W, b)
        flops = 2.0 * Ms * N * K
        desc = (f"reference tiledMatmulWithActivation + bias + fusedGelu (FusedKernels.h:378-458,"
                f"606-627) on {Ms} of the 2048 rows")
    elif workload == "gelu_f32":
        n = 16 << 20
        X = (3 * g.standard_normal(n)).astype(np.float32)
        fn = lambda: ref.gelu(X)
        for _ in range(warm):
            fn()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        dt = (time.perf_counter() - t0) / reps
        return (2.0 * n * 4 / dt / 1e9,
                f"reference fusedGelu (FusedKernels.h:606-627) on 16 Mi of the 64 Mi elements; "
                f"{reps} timed reps, {dt * 1e3:.1f} ms each", threads)
    elif workload == "attn_fp32":
        Q, K_, V = (g.standard_normal((1, 8, 512, 64), dtype=np.float32) for _ in range(3))
        fn = lambda: ref.flash_attention(Q, K_, V)
        flops = 4.0 * 8 * 512 * 512 * 64
        desc = "reference flashAttention (FlashAttention.h:130-309), full C1"
        reps = 20
    else:
        # The reference has no causal kernel: its non-causal flashAttention on
        # one (b, h) unit at the config's S, counted at causal FLOPs x2 = the
        # work it actually does.
        S = 4096 if workload == "attn" else 16384
        Sx = min(S, 4096)
        Q, K_, V = (g.standard_normal((1, 1, Sx, 128), dtype=np.float32) for _ in range(3))
        fn = lambda: ref.flash_attention(Q, K_, V)
        flops = 4.0 * Sx * Sx * 128
        reps = 2
        desc = (f"reference flashAttention (non-causal; the reference has no causal mask) on one "
                f"(b,h) unit at S={Sx}, D=128, fp32; non-causal FLOPs 4*S^2*D")
    for _ in range(warm):
        fn()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    dt = (time.perf_counter() - t0) / reps
    return flops / dt / 1e12, desc + f"; {reps} timed reps, {dt * 1e3:.1f} ms each", threads


# ---------------------------------------------------------------------------
def run_reference_arm(args):
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    headline = args.workload == "headline"
    workload = "gemm" if headline else args.workload

    def timed(wkey, steps, warmup):
        """Each step is one bounded sample of the workload on the CPU."""
        for _ in range(warmup):
            cpu_reference_sample(wkey, reps=1, warm=0)
        vals, desc, threads = [], "", os.cpu_count() or 1
        t0 = time.perf_counter()
        for _ in range(steps):
            v, desc, threads = cpu_reference_sample(wkey, reps=1, warm=0)
            vals.append(v)
        return statistics.mean(vals), (time.perf_counter() - t0) / steps, desc, threads

    value, step_s, desc, threads = timed(workload, args.steps, args.warmup)
    rowwise = workload in ("softmax", "xent", "gelu_f32")
    unit = "GB/s" if rowwise else ("TOPS" if workload == "int8" else "TFLOP/s")
    line = {"metric": metric_for(args.workload), "value": round(value, 6), "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(step_s * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": describe(workload, world, "CPU: bounded sample per step"),
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": threads,
                             "kind": CPU_KIND.get(workload, "reference"), "sample": desc},
            "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    if headline:
        # the attention configs (C3, C5): a few samples each, ~1 s of CPU work apiece
        gv, gstep, gdesc, gthreads = timed("attn_gqa", 2, 0)
        line["attn_gqa"] = {"value": round(gv, 6), "unit": "TFLOP/s",
                            "ms_per_step": round(gstep * 1e3, 3), "steps": 2,
                            "config": describe("attn_gqa", world, "CPU: bounded sample per step"),
                            "cpu_baseline": {"value": round(gv, 6), "unit": "TFLOP/s",
                                             "cores": gthreads, "kind": "reference",
                                             "sample": gdesc}}
        av, astep, adesc, athreads = timed("attn", 3, 1)
        line["attn"] = {"value": round(av, 6), "unit": "TFLOP/s",
                        "ms_per_step": round(astep * 1e3, 3), "steps": 3,
                        "config": describe("attn", world, "CPU: bounded sample per step"),
                        "cpu_baseline": {"value": round(av, 6), "unit": "TFLOP/s",
                                         "cores": athreads, "kind": "reference",
                                         "sample": adesc}}
    emit(line)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference_arm(args)

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import jules_b200 as jb
    jb.lib()  # fails loudly when the CUDA library is missing

    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # The communicator of the library's multi-GPU entry points (strong-scaled
    # C2 / C3 / C5); torch.distributed above is the bench's own plumbing
    # (barriers, max over ranks).
    dist_comm = jb.Dist.from_torch() if world > 1 and args.workload in (
        "headline", "gemm", "attn", "attn_gqa") else None

    def make(workload):
        return {"gemm": lambda: Gemm(jb, torch, rank, world, dist=dist_comm),
                "attn": lambda: Attention(jb, torch, rank, world, gqa=False, dist=dist_comm),
                "attn_gqa": lambda: Attention(jb, torch, rank, world, gqa=True, dist=dist_comm),
                "mlp": lambda: Mlp(jb, torch, rank, world),
                "attn_fp32": lambda: AttentionF32(jb, torch, rank, world),
                "softmax": lambda: RowWise(jb, torch, rank, world, xent=False),
                "xent": lambda: RowWise(jb, torch, rank, world, xent=True),
                "int8": lambda: Int8Gemm(jb, torch, rank, world),
                "fp8": lambda: Fp8Gemm(jb, torch, rank, world),
                "attn_bwd": lambda: AttentionBwd(jb, torch, rank, world),
                "gemm_f32": lambda: GemmF32(jb, torch, rank, world),
                "gelu_f32": lambda: GeluF32(jb, torch, rank, world)}[workload]()

    def measure(workload):
        """Warm-up, the K timed steps, the gather, e2e and the CPU leg of one
        workload; returns the fields of its JSON object."""
        wl = make(workload)
        stream = torch.cuda.current_stream()
        # clocks: sampled from the first warm-up step to the end of the timed
        # steps (a short timed region alone gets one or two NVML samples)
        sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                               else local_rank)
        sampler.start()
        for i in range(args.warmup):
            wl.step(i)
        torch.cuda.synchronize()
        if jb.device_error() != 0:
            sampler.stop()
            raise RuntimeError(f"device error during warm-up ({workload})")

        # ---------------- timed region (device) ----------------
        K = args.steps
        dom = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(K)]
        barrier()
        torch.cuda.synchronize()
        sampler.mark_timed()
        t_begin = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_begin.record(stream)
        for i in range(K):
            wl.step(i, dom[i])
        t_end.record(stream)
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        ms_total = max_over_ranks(t_begin.elapsed_time(t_end))
        dom_ms = statistics.mean(a.elapsed_time(b) for a, b in dom)
        dom_ms = max_over_ranks(dom_ms)
        if jb.device_error() != 0:
            raise RuntimeError(f"device error in timed region ({workload})")

        strong = getattr(wl, "global_work", False)
        per_job = 1 if strong else world  # flops_per_step is the whole job's when strong
        tflops_total = wl.flops_per_step * per_job * K / (ms_total * 1e-3) / wl.unit_scale
        peak, hbm, peak_kind = measured_peaks()
        achieved = wl.flops_dominant / (dom_ms * 1e-3) / wl.unit_scale
        traffic = profiled_traffic(workload)

        # ---------------- output gather (N > 1), timed separately ----------------
        gather = None
        compute_only = None
        if world > 1 and strong:
            # the same steps without the gather: this rank's share of the work alone
            for i in range(3):
                wl.compute_only(i)
            torch.cuda.synchronize()
            barrier()
            c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            c0.record(stream)
            for i in range(K):
                wl.compute_only(i)
            c1.record(stream)
            torch.cuda.synchronize()
            cms = max_over_ranks(c0.elapsed_time(c1))
            compute_only = {"value": round(wl.flops_per_step * K / (cms * 1e-3) / wl.unit_scale, 3),
                            "ms_per_step": round(cms / K, 5),
                            "what": "each rank's share without the gather (max over ranks)"}
        elif world > 1:
            out = wl.output(0).contiguous()
            full = torch.empty((world,) + tuple(out.shape), dtype=out.dtype, device="cuda")
            dist.all_gather_into_tensor(full, out)  # warm
            torch.cuda.synchronize()
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record()
            dist.all_gather_into_tensor(full, out)
            g1.record()
            torch.cuda.synchronize()
            gms = max_over_ranks(g0.elapsed_time(g1))
            gather = {"collective": "ncclAllGather of each rank's output shard (not in value)",
                      "bytes_per_rank": out.numel() * out.element_size(), "ms": round(gms, 4)}
            del full

        # ---------------- e2e through the C ABI with host buffers ----------------
        e2e = None
        if not args.no_e2e and world > 1 and strong:
            ins, outs, run = wl.e2e_dist_spec()

            def e2e_step():
                for h, d in ins:
                    d.copy_(h, non_blocking=True)
                run()
                if rank == 0:
                    for h, d in outs:
                        h.copy_(d, non_blocking=True)

            for _ in range(3):
                e2e_step()
            torch.cuda.synchronize()
            Ke = max(4, min(K, 10))
            barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(Ke):
                e2e_step()
            e1.record(stream)
            torch.cuda.synchronize()
            ems = max_over_ranks(e0.elapsed_time(e1))
            barrier()
            h2d = sum(h.numel() * h.element_size() for h, _ in ins) * world  # all ranks' inputs
            d2h = sum(h.numel() * h.element_size() for h, _ in outs)         # rank 0 reads the result
            e2e = {"value": round(wl.flops_per_step * Ke / (ems * 1e-3) / wl.unit_scale, 3),
                   "unit": wl.unit, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                   "steps": Ke,
                   "path": "each rank: pinned host -> cudaMemcpyAsync of its shard of the inputs -> "
                           "sharded public API call (gather included) -> rank 0 cudaMemcpyAsync of "
                           "the whole result -> host; one stream; replicated weights resident"}
        elif not args.no_e2e:
            pipe = E2EPipeline(torch, wl)
            for _ in range(3):
                pipe.step()
            torch.cuda.synchronize()
            Ke = max(4, min(K, 10))
            barrier()
            ems = max_over_ranks(pipe.time_steps(Ke))
            barrier()
            e2e = {"value": round(wl.flops_per_step * world * Ke / (ems * 1e-3) / wl.unit_scale, 3),
                   "unit": wl.unit, "h2d_bytes_per_step": int(pipe.h2d),
                   "d2h_bytes_per_step": int(pipe.d2h), "steps": Ke,
                   "path": "pinned host -> cudaMemcpyAsync (H2D stream) -> public API (compute "
                           "stream) -> cudaMemcpyAsync (D2H stream) -> host; 2 buffer sets, "
                           "consecutive steps overlapped"}
            del pipe

        # ---------------- CPU baseline (rank 0, N == 1) ----------------
        cpu = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            try:
                v, desc, threads = cpu_reference_sample(workload)
                cpu = {"value": round(v, 6), "unit": wl.unit, "cores": threads,
                       "kind": CPU_KIND.get(workload, "reference"), "sample": desc}
            except Exception as ex:  # the GPU number stands without it
                cpu = {"value": None, "unit": wl.unit, "cores": None, "kind": "reference",
                       "sample": f"unavailable: {ex}"}

        res = {
            "value": round(tflops_total, 3), "unit": wl.unit,
            "ms_per_step": round(ms_total / K, 5),
            "dtype": "f32" if workload == "attn_fp32" else wl.dtype,
            "config": describe(workload, world, wl.config.get("l2"), comm=dist_comm),
            "roofline": roofline(wl, achieved, peak, peak_kind, traffic),
            **({"pct_of_dense_bf16_peak_2250": round(100 * tflops_total / world / 2250.0, 2)}
               if wl.unit == "TFLOP/s" and not isinstance(wl, (Fp8Gemm, AttentionF32, GemmF32))
               else {}),
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": K * wl.launches_per_step,
            "cpu_baseline": cpu,
            "scaling": "strong" if strong else "weak",
        }
        if gather:
            res["gather"] = gather
        if compute_only:
            res["compute_only"] = compute_only
        if hasattr(wl, "extra_measure"):
            res["cuda_core_exact"] = wl.extra_measure()
        if hasattr(wl, "release"):
            torch.cuda.synchronize()
            barrier()
            wl.release()
        del wl
        torch.cuda.empty_cache()
        return res

    headline = args.workload == "headline"
    main_res = measure("gemm" if headline else args.workload)
    attn_res = measure("attn") if headline else None
    # C5, the long-context grouped-query config the baseline defines for 8 GPUs
    gqa_res = measure("attn_gqa") if headline else None

    def published_point():
        """The reference's one published attention figure (benchmarks/
        bench_comparison.py:215,219: fp32 flash attention, non-causal,
        [B=2, H=8, S=1024, D=64], 135.416 ms on a 4-core AVX-512 Xeon with
        MKL) against this library's fp32 kernel on the same shape (and the
        bf16 tensor-core kernel beside it).  Device time per call, 50 calls
        after 5 warm-up, rotating inputs."""
        B, H, S, D = 2, 8, 1024, 64
        g = torch.Generator(device="cuda").manual_seed(6)
        res = {"config": "[2, 8, 1024, 64] non-causal, 4*B*H*S^2*D = 4.295 GFLOP",
               "published_ms": 135.416, "published_source": "benchmarks/bench_comparison.py:215,219 "
               "(fp32, 4-core Xeon AVX-512 3.2 GHz, MKL)"}
        for name, dt in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
            qs = [torch.randn((B, H, S, D), generator=g, device="cuda").to(dt) for _ in range(6)]
            o = torch.empty_like(qs[0])
            for i in range(5):
                jb.flash_attention_fwd(qs[i % 6], qs[(i + 1) % 6], qs[(i + 2) % 6], out=o, lse=False)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(50):
                jb.flash_attention_fwd(qs[i % 6], qs[(i + 1) % 6], qs[(i + 2) % 6], out=o, lse=False)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 50
            res[f"{name}_ms"] = round(ms, 4)
            res[f"{name}_speedup_vs_published"] = round(135.416 / ms, 1)
        return res

    pub = published_point() if headline and world == 1 else None
    if rank == 0:
        line = {"metric": metric_for(args.workload), "value": main_res["value"],
                "unit": main_res["unit"], "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": main_res["ms_per_step"],
                "higher_is_better": True, "scaling": main_res["scaling"], "vs_baseline": None,
                "dtype": main_res["dtype"],
                "data": "synthetic (seeded; config shapes and distributions)"}
        for k in ("config", "roofline", "pct_of_dense_bf16_peak_2250", "clocks", "e2e",
                  "gpu_launches", "cpu_baseline", "gather", "compute_only", "cuda_core_exact"):
            if k in main_res:
                line[k] = main_res[k]
        if attn_res:
            # The attention half of the headline metric (config C3), measured in
            # the same process right after the GEMM half; the line's own
            # gpu_launches counts both.
            line["gpu_launches"] += attn_res["gpu_launches"]
            line["attn"] = {k: v for k, v in attn_res.items() if k not in ("dtype",)}
        if gqa_res:
            line["gpu_launches"] += gqa_res["gpu_launches"]
            line["attn_gqa"] = {k: v for k, v in gqa_res.items() if k not in ("dtype",)}
        if pub:
            line["published_attention_point"] = pub
        emit(line)

    if dist_comm is not None:
        torch.cuda.synchronize()
        barrier()
        dist_comm.close()

    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    # The JSON line is the only thing on stdout: keep a private handle on the
    # real stdout and send everything else written to fd 1 (library banners
    # such as NCCL's version line) to stderr.
    JSON_OUT = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    sys.exit(main())
