"""Benchmark of the PyFlameRT MatMul/Gemm hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline workload (the configuration the metric is
quoted on): the quantized int8 linear layer, uint8 activations [512, 4096] x
int8 weights [4096, 4096], int32 accumulation, per-output-channel scales,
requantized to int8.  One step = one pass over one batch.  At N GPUs each rank
processes its own 512-row batch (batch sharding, no collective: weak scaling)
and `value` is the whole-job TOPS: N * 2*M*N*K ops / max-over-ranks time.

Timing: W warm-up steps, then K steps captured in a CUDA graph and replayed
between barriers + synchronizes, timed with CUDA events on the launching
stream; the max over ranks is taken.  The step inputs rotate over enough
copies of (activations, weights, output) that each step's working set has
left L2 (the copies total more than twice the 126 MB L2), so every step reads
its operands from HBM.  `e2e` is the same metric through the public API
with host buffers: pinned-host -> device copy of the activations, the layer,
device -> pinned-host copy of the output, every step.  `e2e.host_link` times
each direction's copies alone on the same lanes; the slower one is the least
a step can take on that box's host link.

The secondary objects report, measured the same way: the CSR SpMM (config 5,
M=1, 90% sparse, 8192 x 8192: the HBM-bound point), the 4096^3 int8 GEMM (the
tensor-peak target), the 4-layer int8 MLP of config 4 (batch 8192 split over
the ranks) and the fp32 Gemm (config 1).  `--impl reference` times the reference's own CPU implementation
(its sources compiled into oracle/_ref) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
M, N, K = 512, 4096, 4096                         # config 2
SPMM_N, SPMM_K, SPMM_S = 8192, 8192, 0.90         # config 5 HBM-bound point (M = 1)
GEMM_M, GEMM_N, GEMM_K = 256, 1024, 1024          # config 1
MLP_BATCH, MLP_HIDDEN, MLP_LAYERS = 8192, 4096, 4  # config 4


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded in profiles/<name>.md by an ncu capture."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    if not os.path.exists(p):
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", open(p).read())
    return float(m.group(1)) if m else None


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons in the background."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.samples = []
        self.proc = None
        self.error = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception as e:  # no nvidia-smi
            self.error = str(e)

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0, t1):
        sel = [p for (t, p) in self.samples if t0 - 0.15 <= t <= t1 + 0.15] or [p for (_, p) in self.samples]
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "note": self.error or "no nvidia-smi samples"}
        mhz = [float(p[1]) for p in sel if p[1].replace(".", "").isdigit()]
        mx = [float(p[2]) for p in sel if p[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for p in sel for i in range(4) if p[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sel),
                "power_w_max": max(float(p[3]) for p in sel if re.match(r"^[0-9.]+$", p[3])) if sel else None}


# --------------------------------------------------------------------------- dist
def dist_init(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        import datetime
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    elif n_gpus > 1:
        raise SystemExit("--gpus N > 1 must be launched with torch.distributed.run (one process per GPU)")
    return world, rank, local


def bind_gpu_local_cpus(local):
    """Keeps this process on the CPUs that NVML reports as local to its GPU
    (a read; only the process's own affinity is set), so pinned host buffers
    are allocated on the GPU's NUMA node and their copies do not cross the
    inter-socket link.  Returns the previous CPU set (to restore), or None if
    nothing was changed (no NVML, or no overlap with the allowed CPUs)."""
    try:
        import pynvml
        import torch
        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, ((os.cpu_count() or 64) + 63) // 64)
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        before = os.sched_getaffinity(0)
        near = cpus & before
        if not near or near == before:
            return None
        os.sched_setaffinity(0, near)
        return before
    except Exception:
        return None


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# --------------------------------------------------------------------------- timing
EAGER = False  # --eager: plain launches, no graph and no soak (for profiler runs)


def graph_time(step_fns, K, W, world, sampler=None, soak=True):
    """W eager warm-up steps; K steps captured in one CUDA graph; a soak replay
    of about a second for the clock sampler (soak=False: none, so the timed
    replay follows the capture at once -- a burst, as a kernel timed in
    isolation runs); then one timed replay between barriers.  Returns
    (ms per step, t_start, t_end) with the max over ranks."""
    import torch
    n = len(step_fns)
    for i in range(W):
        step_fns[i % n]()
    torch.cuda.synchronize()
    if EAGER:
        barrier(world)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.time()
        ev0.record()
        for i in range(K):
            step_fns[i % n]()
        ev1.record()
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(ev0.elapsed_time(ev1) / K, world), t0, time.time()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for i in range(K):
                step_fns[i % n]()
    torch.cuda.synchronize()
    # Soak for ~1 s so the clock samples see the load.  The number of replays
    # is agreed over the ranks first: a graph may hold collectives, and every
    # rank must issue the same collectives in the same order.
    t_soak = time.time()
    g.replay()
    torch.cuda.synchronize()
    one = max(time.time() - t_soak, 1e-4)
    n_soak = int(max_over_ranks(float(max(1, min(10000, int(1.0 / one)))), world)) if soak else 0
    for _ in range(n_soak):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    ev0.record()
    g.replay()
    ev1.record()
    torch.cuda.synchronize()
    t1 = time.time()
    barrier(world)
    ms = ev0.elapsed_time(ev1) / K
    del g
    return max_over_ranks(ms, world), t_soak, t1


def tensor_roofline(achieved, peaks, peak_src, traffic):
    """int8 tensor roofline of a line, one rule for every line: `frac` is
    against the burst peak (2 x the measured bf16 burst figure; a
    multiply-add counts as 2 ops), `frac_of_sustained` against the
    power-capped one."""
    burst = 2.0 * peaks["bf16_tflops"]
    sustained = 2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    return {"bound": "tensor", "achieved": achieved, "peak": burst, "unit": "TFLOP/s", "frac": achieved / burst,
            "frac_of_sustained": achieved / sustained, "traffic": traffic,
            "peak_source": f"int8 dense = 2 x bf16_tflops ({peak_src} MEASURED_PEAKS.json); "
                           f"sustained = 2 x bf16_tflops_sustained"}


# --------------------------------------------------------------------------- workloads
def qlinear_setup(ctx, n_copies):
    import numpy as np
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    q = wl.qlinear_case(M, N, K, seed=2)
    copies = []
    for i in range(n_copies):
        w = pf.QWeight(ctx, q.w, q.w_scale)
        a = torch.from_numpy(q.a).cuda()
        y = torch.empty((M, N), dtype=torch.int8, device="cuda")
        copies.append((w, a, y))
    fns = [(lambda w=w, a=a, y=y: w(a, q.a_scale, q.a_zp, out="int8", y_scale=q.y_scale, y=y))
           for (w, a, y) in copies]
    return q, copies, fns


def qlinear_e2e(ctx, q, w, steps, lanes=3):
    """Through the C ABI's host-buffer entry (pfrt_qlinear_host): every step
    copies its activations from pinned host memory to the device, runs the
    layer and copies its output back to pinned host memory, all enqueued by
    one call.  Steps alternate over `lanes` independent lanes (each its own
    context, stream, weight copy and pinned buffers), so one step's
    device->host copy overlaps the next step's host->device copy and kernel,
    as in a serving loop."""
    import torch

    import pyflamert_b200 as pf
    cur = torch.cuda.current_stream()
    L = []
    for i in range(lanes):
        c = ctx if i == 0 else pf.Context(torch.cuda.current_device())
        L.append(dict(ctx=c, w=w if i == 0 else pf.QWeight(c, q.w, q.w_scale), stream=torch.cuda.Stream(),
                      a_host=torch.from_numpy(q.a).pin_memory(),
                      y_host=torch.empty((M, N), dtype=torch.int8).pin_memory()))

    def step(i):
        ln = L[i % lanes]
        ln["w"].host_call(ln["a_host"], q.a_scale, q.a_zp, ln["y_host"], out="int8", y_scale=q.y_scale,
                          stream=ln["stream"])

    def timed(fn):
        """(device ms per step, host enqueue us per step) of `steps` calls of
        fn(i), the lanes' streams joined to the current stream on both sides."""
        for i in range(5 * lanes):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cur)
        for ln in L:
            ln["stream"].wait_stream(cur)
        h0 = time.perf_counter()
        for i in range(steps):
            fn(i)
        h1 = time.perf_counter()
        for ln in L:
            cur.wait_stream(ln["stream"])
        e1.record(cur)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps, (h1 - h0) * 1e6 / steps

    # The floor of this path on this host link: each direction's copies alone,
    # in the same lanes; with both directions in flight at once (full duplex)
    # a step cannot take less than the slower of the two.
    for ln in L:
        ln["a_dev"] = torch.empty_like(ln["a_host"], device="cuda")
        ln["y_dev"] = torch.zeros_like(ln["y_host"], device="cuda")

    def h2d_only(i):
        ln = L[i % lanes]
        with torch.cuda.stream(ln["stream"]):
            ln["a_dev"].copy_(ln["a_host"], non_blocking=True)

    def d2h_only(i):
        ln = L[i % lanes]
        with torch.cuda.stream(ln["stream"]):
            ln["y_host"].copy_(ln["y_dev"], non_blocking=True)

    h2d_ms, _ = timed(h2d_only)
    d2h_ms, _ = timed(d2h_only)
    ms, enqueue_us = timed(step)
    # every lane's host buffer holds the layer's output
    ref = w(torch.from_numpy(q.a).cuda(), q.a_scale, q.a_zp, out="int8", y_scale=q.y_scale).cpu()
    for ln in L:
        assert torch.equal(ref, ln["y_host"])
    for ln in L[1:]:
        ln["ctx"].check()
        ln["w"].close()
        ln["ctx"].close()
    link = {"h2d_only_ms_per_step": h2d_ms, "d2h_only_ms_per_step": d2h_ms, "enqueue_us_per_step": enqueue_us}
    return ms, M * K, M * N, link


def session_e2e(q, local, steps, warmup, lanes=3):
    """Config 2's layer through the drop-in itself: the reference's
    InferenceSession with device "cuda:<gpu>" (libpfrt_session.so, its own
    session and .pfm loader with the CUDA seam) running a QuantizedMatMul ->
    Quantize graph saved as .pfm, with host (pageable numpy) input and output
    tensors, one synchronous run() per step.  Timed on the host clock around
    the calls (run() returns once the output is in host memory): one session
    alone (the latency of a call), and `lanes` sessions driven by as many
    threads at once (each its own backend and context on this GPU, as a
    serving loop runs them; the GIL is released inside run()), the same
    overlap the e2e object's lanes use.  None when the session library was
    not built (no PyFlameRT sources)."""
    import tempfile
    import threading

    import numpy as np

    from pyflamert_b200 import pfm
    if not os.path.exists(pfm.session_lib_path()):
        return None
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "config2.pfm")
        pfm.save(path, "config2", inputs=[("A", np.uint8, (M, K))], outputs=[("Y", np.int8, (M, N))],
                 initializers={"W": q.w},
                 nodes=[("qmm", "QuantizedMatMul", ["A", "W"], ["t0"],
                         {"a_scale": q.a_scale, "a_zero_point": q.a_zp, "b_scales": q.w_scale}),
                        ("quant", "Quantize", ["t0"], ["Y"], {"scale": q.y_scale, "dtype": "int8"})])
        sess = [pfm.Session(path, f"cuda:{local}") for _ in range(lanes)]
        try:
            feeds = [{"A": q.a.copy()} for _ in range(lanes)]
            first = sess[0].run(feeds[0])[0]
            for i in range(lanes):
                for _ in range(max(3, warmup)):
                    sess[i].run(feeds[i], copy=False)
            t0 = time.perf_counter()
            for _ in range(steps):
                sess[0].run(feeds[0], copy=False)
            one_ms = (time.perf_counter() - t0) * 1e3 / steps
            per = max(1, steps // lanes)
            start = threading.Barrier(lanes + 1)

            def lane(i):
                start.wait()
                for _ in range(per):
                    sess[i].run(feeds[i], copy=False)

            ts = [threading.Thread(target=lane, args=(i,)) for i in range(lanes)]
            for t in ts:
                t.start()
            start.wait()
            t0 = time.perf_counter()
            for t in ts:
                t.join()
            lanes_ms = (time.perf_counter() - t0) * 1e3 / (per * lanes)
        finally:
            for x in sess:
                x.close()
    return lanes_ms, one_ms, first


def spmm_setup(ctx, n_copies):
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    c = wl.spmm_case(1, SPMM_N, SPMM_K, sparsity=SPMM_S, seed=3)
    copies = []
    for i in range(n_copies):
        w = pf.CSR(ctx, c.N, c.K, c.indptr, c.indices, c.values)
        x = torch.from_numpy(c.X).cuda()
        y = torch.empty((1, c.N), dtype=torch.float32, device="cuda")
        copies.append((w, x, y))
    fns = [(lambda w=w, x=x, y=y: w(x, y=y)) for (w, x, y) in copies]
    nnz = c.values.size
    alg_bytes = 8 * nnz + 4 * (c.N + 1) + 4 * c.K + 4 * c.N
    return c, copies, fns, alg_bytes


def spmm_nshard(ctx, args, world, rank, peaks, peak_src):  # noqa: C901
    """Config 5's M=1 point with W's output channels sharded over the ranks
    (strong scaling: the problem is fixed, each rank holds 1/world of W).
    The product path is the fused kernel (pfrt_spmm_allgather): each rank's
    SpMM stores its rows of Y straight into every rank's output over NVLink.
    The same step with NCCL's all_gather_into_tensor after a plain SpMM is
    timed beside it as the library baseline."""
    import numpy as np
    import torch

    from pyflamert_b200 import sharding
    from pyflamert_b200 import workloads as wl
    c = wl.spmm_case(1, SPMM_N, SPMM_K, sparsity=SPMM_S, seed=3)
    nnz = c.values.size
    alg_bytes = 8 * nnz + 4 * (c.N + 1) + 4 * c.K + 4 * c.N
    per_rank = 8 * nnz / world
    n_copies = max(2, math.ceil(2 * L2_BYTES / per_rank))
    x = torch.from_numpy(c.X).cuda()
    fused = [sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, rank, world)
             for _ in range(n_copies)]
    ms, t0_, t1_ = graph_time([(lambda f=f: f(x)) for f in fused], args.steps, args.warmup, world)
    ctx.check()
    y_fused = fused[0](x).cpu().numpy()
    ctx.check()
    for f in fused:
        f.close()
    # NCCL baseline
    objs, fns = [], []
    for i in range(n_copies):
        sh = sharding.NShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, rank, world)
        lb = torch.empty((1, sh.ns), dtype=torch.float32, device="cuda")
        gb = torch.empty((world * sh.ns,), dtype=torch.float32, device="cuda")
        objs.append((sh, lb, gb))
        fns.append(lambda sh=sh, lb=lb, gb=gb: sh(x, gather_buf=gb, local_buf=lb))
    try:
        ms_nccl, _, _ = graph_time(fns, args.steps, args.warmup, world)
    except Exception as e:  # capture of the collective unavailable: plain launches
        global EAGER
        old, EAGER = EAGER, True
        ms_nccl, _, _ = graph_time(fns, args.steps, args.warmup, world)
        EAGER = old
    ctx.check()
    # the fused path's gathered Y equals the NCCL path's (same per-rank kernel
    # and summation order, so bit for bit)
    y_nccl = objs[0][0](x).cpu().numpy()
    same = bool(np.array_equal(y_fused, y_nccl))
    for o in objs:
        o[0].local.close()
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    return {
        "metric": "CSR SpMM HBM GB/s (config 5: M=1, W 8192x8192 90% sparse), W sharded by output channel",
        "value": gbs, "unit": "GB/s", "ms_per_step": ms, "scaling": "strong",
        "parallelism": f"W rows split {world} ways; the all-gather of Y fused into the SpMM kernel "
                       "(NVLink stores to every rank's output)",
        "timing": "K steps in one CUDA graph", "equals_nccl_path": same,
        "nccl_baseline": {"path": "pfrt_spmm + NCCL all_gather_into_tensor per step",
                          "value": alg_bytes / (ms_nccl * 1e-3) / 1e9, "ms_per_step": ms_nccl},
        "roofline": {"bound": "hbm", "achieved": gbs / world, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / world / peaks["hbm_gbs"], "per": "GPU (whole-job bytes / world / time)",
                     "algorithmic_bytes": alg_bytes, "peak_source": f"hbm_gbs ({peak_src} MEASURED_PEAKS.json)"},
        "gpu_launches": args.steps,
    }


SWEEP_MS = (1, 64, 1024, 8192)                    # config 5's batch sizes (at SPMM_S sparsity)
FP32_SIMT_TFLOPS = 148 * 256 * 1.965e9 / 1e12     # derived: 148 SMs x 128 FMA/clk x 2 x max SM clock


def spmm_point(nnz, M, ms, world, peaks):
    """Whole-job figures of one config-5 point and its per-GPU roofline: the
    bound is the larger of the algorithmic bytes over HBM and the flops over
    the FP32 SIMT peak, per GPU (each rank holds 1/world of W and all of X)."""
    flops = 2.0 * nnz * M
    alg_bytes = 8.0 * nnz + 4.0 * (SPMM_N + 1) + 4.0 * M * SPMM_K + 4.0 * M * SPMM_N
    per_gpu_bytes = (8.0 * nnz + 4.0 * (SPMM_N + 1) + 4.0 * M * SPMM_N) / world + 4.0 * M * SPMM_K
    t_hbm = per_gpu_bytes / (peaks["hbm_gbs"] * 1e9)
    t_simt = flops / world / (FP32_SIMT_TFLOPS * 1e12)
    t = ms * 1e-3
    # The tensor-core paths (W densified on chip, or the dense copy) do the
    # dense product as 3xTF32: 3 x 2 M N K tf32 operations, at the tf32 rate
    # (half the measured bf16 rate).
    tf32_tflops = peaks["bf16_tflops"] / 2.0
    t_tc = 6.0 * M * SPMM_N * SPMM_K / world / (tf32_tflops * 1e12)
    return {"M": M, "ms_per_step": ms, "tflops": flops / t / 1e12, "gbs": alg_bytes / t / 1e9,
            "roofline": {"bound": "hbm" if t_hbm >= t_simt else "fp32-simt",
                         "roof_ms": 1e3 * max(t_hbm, t_simt), "frac": max(t_hbm, t_simt) / t,
                         "per": "GPU", "hbm_gbs": peaks["hbm_gbs"], "fp32_simt_tflops": FP32_SIMT_TFLOPS},
            "roofline_dense_3xtf32": {"roof_ms": 1e3 * t_tc, "frac": t_tc / t, "tf32_tflops": tf32_tflops,
                                      "note": "the dense product on the tensor pipe, the bound of the "
                                              "tensor-core paths"}}


def spmm_config3(ctx, args, peaks, peak_src, sampler):
    """Config 3 (the pruned Linear: X [256, 4096] times W^T, W 4096 x 4096 at
    90 % sparsity) through pfrt_spmm's default path, one GPU, rotating over
    copies of W larger than L2 together."""
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    M3, N3, K3 = 256, 4096, 4096
    c = wl.spmm_case(M3, N3, K3, sparsity=0.9, seed=3)
    nnz = int(c.values.size)
    ncopies = int(min(24, max(2, math.ceil(2 * L2_BYTES / (12.0 * nnz)))))
    ws = [pf.CSR(ctx, N3, K3, c.indptr, c.indices, c.values) for _ in range(ncopies)]
    x = torch.from_numpy(c.X).cuda()
    y = torch.empty((M3, N3), dtype=torch.float32, device="cuda")
    fns = [(lambda w=w: w(x, y=y)) for w in ws]
    for f in fns:  # builds each copy's lazily made device state
        f()
    torch.cuda.synchronize()
    ms, t0, t1 = graph_time(fns, args.steps, args.warmup, 1, soak=False)
    ctx.check()
    for w in ws:
        w.close()
    flops = 2.0 * nnz * M3
    alg_bytes = 8.0 * nnz + 4.0 * (N3 + 1) + 4.0 * M3 * K3 + 4.0 * M3 * N3
    tf32 = peaks["bf16_tflops"] / 2.0
    t_tc = 6.0 * M3 * N3 * K3 / (tf32 * 1e12)
    t_hbm = alg_bytes / (peaks["hbm_gbs"] * 1e9)
    return {"metric": "CSR SpMM us per call (config 3: X 256x4096, W 4096x4096 90% sparse)",
            "value": ms * 1e3, "unit": "us", "higher_is_better": False, "ms_per_step": ms,
            "useful_tflops": flops / (ms * 1e-3) / 1e12,
            "path": "pfrt_spmm default (cost model: tensor cores on W's compressed form, the dense copy, "
                    "or the tiled CSR kernel)",
            "roofline": {"bound": "tensor (dense 3xTF32)", "roof_us": 1e6 * t_tc, "frac": t_tc / (ms * 1e-3),
                         "tf32_tflops": tf32, "hbm_roof_us": 1e6 * t_hbm,
                         "peak_source": f"bf16_tflops / 2, hbm_gbs ({peak_src} MEASURED_PEAKS.json)"},
            "clocks": sampler.summary(t0, t1), "gpu_launches": 3 * args.steps,
            "l2": f"{ncopies} copies of W rotated"}


def spmm_structured(ctx, args, peaks, peak_src, sampler):
    """A weight with 2:4 structure along K, as N:M pruning (n = 2, m = 4) of a
    [N, K] weight leaves it (config 5's 8192 x 8192 shape, ~45 % of entries
    kept), at M = 64 and 1024: pfrt_spmm's default path (the structured-sparse
    tensor cores, spmm_sp.cuh) beside the dense copy's 3xTF32 Gemm and the
    tensor-core kernel on W's compressed form, each forced by its switch, on
    the same weight.  One GPU; W's forms (235 MB structured, 512 MB dense)
    are each larger than L2."""
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    Ns = Ks = 8192
    c = wl.structured24_case(8, Ns, Ks, seed=21)
    nnz = int(c.values.size)
    w = pf.CSR(ctx, Ns, Ks, c.indptr, c.indices, c.values)
    envs = ("PFRT_SPMM_SP", "PFRT_SPMM_TC", "PFRT_SPMM_DENSE")
    paths = {"default": {}, "dense": {"PFRT_SPMM_SP": "0", "PFRT_SPMM_DENSE": "1"},
             "tc_compressed": {"PFRT_SPMM_SP": "0", "PFRT_SPMM_TC": "1"}}
    tf32 = peaks["bf16_tflops"] / 2.0
    bf16 = peaks["bf16_tflops"]
    points = []
    saved = {k: os.environ.get(k) for k in envs}
    try:
        for M in (64, 1024):
            x = torch.randn((M, Ks), device="cuda")
            y = torch.empty((M, Ns), dtype=torch.float32, device="cuda")
            fns = [lambda: w(x, y=y)]
            pt = {"M": M}
            for name, env in paths.items():
                for k in envs:
                    os.environ.pop(k, None)
                os.environ.update(env)
                fns[0]()  # builds the path's device form of W outside the capture
                torch.cuda.synchronize()
                ms, t0, t1 = graph_time(fns, args.steps, args.warmup, 1, soak=False)
                ctx.check()
                pt[name + "_us"] = ms * 1e3
                if name == "default":
                    pt["clocks"] = sampler.summary(t0, t1)
            # Roofs: the structured-sparse kernel's six bf16 products on the
            # compressed operands are 6 x M x N x (K / 2) multiply-adds at the
            # dense bf16 rate (a sparse K = 32 MMA takes the time of a dense
            # K = 16 one); the dense path's are 3 tf32 products of M x N x K.
            t_sp = 6.0 * M * Ns * Ks / (bf16 * 1e12)
            pt["useful_tflops"] = 2.0 * nnz * M / (pt["default_us"] * 1e-6) / 1e12
            pt["roofline"] = {"bound": "tensor (sparse bf16 x6)", "roof_us": 1e6 * t_sp,
                              "frac": t_sp / (pt["default_us"] * 1e-6),
                              "dense_3xtf32_roof_us": 1e6 * 6.0 * M * Ns * Ks / (tf32 * 1e12),
                              "peak_source": f"bf16_tflops x 2 for 2:4 sparse MMAs ({peak_src} MEASURED_PEAKS.json)"}
            points.append(pt)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
        w.close()
    return {"metric": "SpMM us per call, 2:4-structured weight (N:M pruning n=2 m=4), 8192 x 8192",
            "unit": "us", "higher_is_better": False, "nnz": nnz,
            "path": "default = structured-sparse tensor cores (tcgen05.mma.sp, bf16 x3 split)",
            "points": points, "gpu_launches_note": "3 launches per step (X packing, kernel, fix-up)"}


def spmm_sweep(ctx, args, world, rank, peaks, peak_src, sampler):  # noqa: C901
    """Config 5's batch sweep (M in 1, 64, 1024, 8192) on its 8192 x 8192
    weight at 90 % sparsity.  One GPU: pfrt_spmm (the kernel its cost model
    picks).  N GPUs: W's output channels split over the ranks, each rank's
    call computes its columns of Y and all-gathers Y over NVLink in the same
    call (pfrt_spmm_allgather; strong scaling: the problem is fixed); the
    single-GPU time of the same point is taken in the same run (every rank
    on its own GPU; rank 0's figure is `single_gpu_ms`), and NCCL's all_gather_into_tensor after the same shard
    SpMM is timed beside it (`nccl_ms`).  Steps rotate over copies of W (and
    windows of X) so each step reads more than L2 holds."""
    import numpy as np
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import sharding
    from pyflamert_b200 import workloads as wl
    c = wl.spmm_case(1, SPMM_N, SPMM_K, sparsity=SPMM_S, seed=3)
    nnz = int(c.values.size)
    Mmax = max(SWEEP_MS)
    g = torch.Generator(device="cuda").manual_seed(77)  # the same X on every rank (X is replicated)
    xbufs = [torch.randn((Mmax, SPMM_K), generator=g, device="cuda", dtype=torch.float32) for _ in range(2)]

    def x_of(i, M):
        xb = xbufs[i % 2]
        off = ((i // 2) * M) % (Mmax - M + 1)
        return xb[off:off + M]

    def copies_for(per_rank_w):
        return int(min(24, max(2, math.ceil(2 * L2_BYTES / (per_rank_w + 4.0 * 64 * SPMM_K)))))

    def time_fns(fns, one_rank=False):
        for f in fns:  # every copy once, eagerly: lazily built state (dense copy, row groups, scratch)
            f()
        torch.cuda.synchronize()
        return graph_time(fns, args.steps, args.warmup, 1 if one_rank else world)

    points = []
    single = {}
    # Every rank times the unsharded point on its own GPU (no collective, so
    # no rank waits on another meanwhile); rank 0's figure is reported.
    if True:
        ws = [pf.CSR(ctx, c.N, c.K, c.indptr, c.indices, c.values) for _ in range(copies_for(8.0 * nnz))]
        y = torch.empty((Mmax, SPMM_N), dtype=torch.float32, device="cuda")
        for M in SWEEP_MS:
            fns = [(lambda w=w, i=i, M=M: w(x_of(i, M), y=y[:M])) for i, w in enumerate(ws)]
            ms, t0, t1 = time_fns(fns, one_rank=True)
            single[M] = (ms, sampler.summary(t0, t1))
        ctx.check()
        for w in ws:
            w.close()
        del y
    if world == 1:
        for M in SWEEP_MS:
            pt = spmm_point(nnz, M, single[M][0], 1, peaks)
            pt["clocks"] = single[M][1]
            points.append(pt)
        return {"metric": "config 5 CSR SpMM sweep (W 8192x8192, 90% sparse), one GPU",
                "path": "pfrt_spmm (row/streaming/tiled CSR kernels or the 3xTF32 dense path, by its cost model)",
                "points": points, "gpu_launches_note": "1-3 launches per step by path"}
    barrier(world)
    sh = sharding.FusedNShardSpMM(ctx, c.N, c.K, c.indptr, c.indices, c.values, rank, world, max_m=Mmax)
    shards = [sh.local] + [sh.shard_copy(c.indptr, c.indices, c.values)
                           for _ in range(copies_for(8.0 * nnz / world) - 1)]
    same = True
    for M in SWEEP_MS:
        fns = [(lambda w=w, i=i, M=M: sh(x_of(i, M), csr=w)) for i, w in enumerate(shards)]
        ms, t0, t1 = time_fns(fns)
        ctx.check()
        pt = spmm_point(nnz, M, ms, world, peaks)
        pt["clocks"] = sampler.summary(t0, t1)
        if rank == 0:
            pt["single_gpu_ms"] = single[M][0]
            pt["speedup_vs_1gpu"] = single[M][0] / ms
            pt["strong_scaling_efficiency"] = single[M][0] / ms / world
        # the NCCL form of the same step: the shard's SpMM, then all_gather_into_tensor and re-layout
        nsh = sharding.NShardSpMM.__new__(sharding.NShardSpMM)
        nsh.N, nsh.K, nsh.rank, nsh.world, nsh.ns, nsh.local = sh.N, sh.K, rank, world, sh.ns, sh.local
        lb = torch.empty((M, sh.ns), dtype=torch.float32, device="cuda")
        gb = torch.empty((world * M * sh.ns,), dtype=torch.float32, device="cuda")
        yo = torch.empty((M, sh.N), dtype=torch.float32, device="cuda")
        nfns = [(lambda w=w, i=i, M=M: (setattr(nsh, "local", w), nsh(x_of(i, M), out=yo, gather_buf=gb,
                                                                       local_buf=lb))) for i, w in enumerate(shards)]
        try:
            pt["nccl_ms"] = time_fns(nfns)[0]
        except Exception as e:  # capture of the collective unavailable
            pt["nccl_ms"] = None
            pt["nccl_note"] = f"not timed: {type(e).__name__}"
        # both forms give the same Y (same shard kernels, so bit for bit)
        xs = x_of(0, M)
        y_fused = sh(xs, csr=shards[0]).clone()
        nsh.local = shards[0]
        nsh(xs, out=yo, gather_buf=gb, local_buf=lb)
        torch.cuda.synchronize()
        same = same and bool(torch.equal(y_fused, yo))
        points.append(pt)
        del lb, gb, yo
    ctx.check()
    for w in shards[1:]:
        w.close()
    sh.close()
    return {"metric": "config 5 CSR SpMM sweep (W 8192x8192, 90% sparse), W sharded by output channel",
            "path": "pfrt_spmm_allgather: each rank's SpMM of its rows of W, then its columns of Y stored "
                    "into every rank's output over NVLink (M = 1: fused into the SpMM kernel)",
            "scaling": "strong", "equals_nccl_path": same, "points": points,
            "peak_source": f"hbm_gbs ({peak_src} MEASURED_PEAKS.json); FP32 SIMT derived"}


def gemm_setup(ctx, n_copies):
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    g = wl.gemm_case(GEMM_M, GEMM_N, GEMM_K, seed=1)
    copies = []
    for i in range(n_copies):
        fw = pf.FWeight(ctx, g.B)
        a = torch.from_numpy(g.A).cuda()
        c = torch.from_numpy(g.C).cuda()
        y = torch.empty((GEMM_M, GEMM_N), dtype=torch.float32, device="cuda")
        copies.append((fw, a, c, y))
    fns = [(lambda fw=fw, a=a, c=c, y=y: fw(a, c, y=y)) for (fw, a, c, y) in copies]
    return g, copies, fns


def cube_setup(ctx, n_copies, D=4096):
    """The 4096^3 int8 GEMM of the tensor-peak target (config 2's layer at
    M = 4096), int8 out, rotating over copies larger than L2 together."""
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    q = wl.qlinear_case(D, D, D, seed=12)
    copies = []
    for i in range(n_copies):
        w = pf.QWeight(ctx, q.w, q.w_scale)
        a = torch.from_numpy(q.a).cuda()
        y = torch.empty((D, D), dtype=torch.int8, device="cuda")
        copies.append((w, a, y))
    fns = [(lambda w=w, a=a, y=y: w(a, q.a_scale, q.a_zp, out="int8", y_scale=q.y_scale, y=y))
           for (w, a, y) in copies]
    return copies, fns, 2.0 * D * D * D


def mlp_setup(ctx, world, rank, n_weight_sets=2):
    """Config 4: MatMul -> Add bias -> Relu -> requantize to uint8, x4 layers,
    hidden 4096, batch 8192 split over the ranks (strong scaling).  Each layer
    is one pfrt_qlinear launch with bias, ReLU and the uint8 requantization in
    its epilogue; layer l+1 reads layer l's uint8 output.  Steps alternate over
    `n_weight_sets` copies of the four weights (128 MiB of weights, plus
    160 MiB of activations per step: more than L2)."""
    import numpy as np
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import sharding
    from pyflamert_b200 import workloads as wl
    x, layers = wl.mlp_case(MLP_BATCH, MLP_HIDDEN, MLP_LAYERS)
    m0, m1 = sharding.batch_slice(MLP_BATCH, rank, world)
    rows = m1 - m0
    sets = []
    for _ in range(n_weight_sets):
        sets.append([(pf.QWeight(ctx, L.w, L.w_scale), torch.from_numpy(L.bias).cuda()) for L in layers])
    acts = [torch.from_numpy(np.ascontiguousarray(x[m0:m1])).cuda()] + \
        [torch.empty((rows, MLP_HIDDEN), dtype=torch.uint8, device="cuda") for _ in layers]

    def step(ws):
        for l, (L, (w, b)) in enumerate(zip(layers, ws)):
            w(acts[l], L.a_scale, L.a_zp, bias=b, relu=True, out="uint8", y_scale=L.y_scale, y=acts[l + 1])

    fns = [(lambda ws=ws: step(ws)) for ws in sets]
    ops_rank = 2.0 * rows * MLP_HIDDEN * MLP_HIDDEN * MLP_LAYERS
    return sets, acts, fns, ops_rank, (m0, m1)


# --------------------------------------------------------------------------- CPU reference
def cpu_reference_rate(budget_s=12.0, threads=None):
    """The reference's own quantized_matmul + quantize_tensor (compiled from its
    sources into oracle/_ref) on a row sample of config 2, all host threads."""
    import numpy as np

    from oracle import pyoracle as po
    from pyflamert_b200 import workloads as wl
    threads = threads or os.cpu_count() or 1
    q = wl.qlinear_case(M, N, K, seed=2)
    # calibrate rows per thread from a 1-row single-thread run
    t = time.time()
    po.ref_quantized_matmul(q.a[:1], q.a_scale, q.a_zp, q.w, 0.0125, 0, out="int8", y_scale=q.y_scale)
    per_row = time.time() - t
    rows = int(max(threads, min(M, threads * max(1, budget_s / per_row // 1))))
    rows = min(rows, M)
    t = time.time()
    po.ref_quantized_matmul(q.a[:rows], q.a_scale, q.a_zp, q.w, 0.0125, 0, out="int8",
                            y_scale=q.y_scale, nthreads=threads)
    dt = time.time() - t
    tops = 2.0 * rows * N * K / dt / 1e12
    return {"value": tops, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
            "sample": f"{rows} of config 2's 512 rows (x 4096 x 4096), reference quantized_matmul "
                      f"+ quantize_tensor, {threads} threads over row slices, {dt:.1f} s"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    steps = args.steps + args.warmup
    # each step: a row sample sized so that all steps end within ~3 minutes
    budget = max(0.05, 180.0 / max(1, steps))
    from oracle import pyoracle as po
    from pyflamert_b200 import workloads as wl
    q = wl.qlinear_case(M, N, K, seed=2)
    t = time.time()
    po.ref_quantized_matmul(q.a[:1], q.a_scale, q.a_zp, q.w, 0.0125, 0, out="int8", y_scale=q.y_scale)
    per_row = time.time() - t
    rows = max(1, min(M, int(threads * budget / per_row)))
    times = []
    for i in range(steps):
        r0 = (i * rows) % (M - rows + 1)
        t = time.time()
        po.ref_quantized_matmul(q.a[r0:r0 + rows], q.a_scale, q.a_zp, q.w, 0.0125, 0, out="int8",
                                y_scale=q.y_scale, nthreads=threads)
        times.append(time.time() - t)
    timed = times[args.warmup:]
    sec = sum(timed) / len(timed)
    tops = 2.0 * rows * N * K / sec / 1e12
    sample = (f"{rows} rows of config 2 (512 x 4096 x 4096) per step, reference quantized_matmul + "
              f"quantize_tensor (its sources compiled into oracle/_ref), {threads} host threads over "
              f"row slices")
    line = {
        "impl": "reference", "metric": "int8 GEMM TOPS (config 2: u8[512,4096] x s8[4096,4096] -> s8, per-channel)",
        "value": tops, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic (seeded, config 2 shapes and distributions)",
        "config": {"workload": "config2_qlinear_int8", "M": M, "N": N, "K": K, "sample_rows": rows},
        "cpu_baseline": {"value": tops, "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": tops, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- profiling
def profile_target(args):
    """One workload, eager launches, no rotation: the small case an ncu capture
    of a single kernel wants (a few tens of MB on the device)."""
    import torch

    import pyflamert_b200 as pf
    from pyflamert_b200 import workloads as wl
    global EAGER
    EAGER = True
    ctx = pf.Context(0)
    t = args.profile_target
    if t in ("qlinear", "qlinear_4096"):
        m = M if t == "qlinear" else 4096
        q = wl.qlinear_case(m, N, K, seed=2)
        w = pf.QWeight(ctx, q.w, q.w_scale)
        a = torch.from_numpy(q.a).cuda()
        y = torch.empty((m, N), dtype=torch.int8, device="cuda")
        fns = [lambda: w(a, q.a_scale, q.a_zp, out="int8", y_scale=q.y_scale, y=y)]
    elif t == "spmm_24":
        # a 2:4 weight (8192 x 8192) at M = 64: the structured-sparse kernel
        c = wl.structured24_case(64, 8192, 8192, seed=21)
        w = pf.CSR(ctx, c.N, c.K, c.indptr, c.indices, c.values)
        x = torch.from_numpy(c.X).cuda()
        y = torch.empty((64, c.N), dtype=torch.float32, device="cuda")
        fns = [lambda: w(x, y=y)]
    elif t in ("spmm_m1", "spmm_cfg3", "spmm_mid", "spmm_m64"):
        c = (wl.spmm_case(1, SPMM_N, SPMM_K, sparsity=SPMM_S, seed=3) if t == "spmm_m1"
             else wl.spmm_case(256, 4096, 4096, sparsity=0.9, seed=3) if t == "spmm_cfg3"
             else wl.spmm_case(64, SPMM_N, SPMM_K, sparsity=SPMM_S, seed=3) if t == "spmm_m64"
             else wl.spmm_case(64, SPMM_N, SPMM_K, sparsity=0.95, seed=3))  # tiled CSR kernel
        w = pf.CSR(ctx, c.N, c.K, c.indptr, c.indices, c.values)
        x = torch.from_numpy(c.X).cuda()
        y = torch.empty((c.X.shape[0], c.N), dtype=torch.float32, device="cuda")
        fns = [lambda: w(x, y=y)]
    else:
        g = wl.gemm_case(GEMM_M, GEMM_N, GEMM_K, seed=1)
        fw = pf.FWeight(ctx, g.B)
        a, cc = torch.from_numpy(g.A).cuda(), torch.from_numpy(g.C).cuda()
        y = torch.empty((GEMM_M, GEMM_N), dtype=torch.float32, device="cuda")
        fns = [lambda: fw(a, cc, y=y)]
    ms, _, _ = graph_time(fns, args.steps, args.warmup, 1)
    ctx.check()
    print(json.dumps({"profile_target": t, "ms_per_step": ms, "note": "eager, not a bench value"}))


# --------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--eager", action="store_true",
                    help="plain launches without CUDA graph or soak (profiler runs; not a bench value)")
    ap.add_argument("--profile-target", default=None,
                    choices=["qlinear", "spmm_m1", "spmm_cfg3", "spmm_mid", "spmm_m64", "spmm_24", "gemm_cfg1",
                             "qlinear_4096"],
                    help="run only this workload, eagerly, for a profiler; prints its ms/step")
    args = ap.parse_args()
    global EAGER
    EAGER = args.eager
    if args.profile_target:
        profile_target(args)
        return
    args.warmup = max(3, args.warmup)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), rank)
        return

    import numpy as np
    import torch

    import pyflamert_b200 as pf
    world, rank, local = dist_init(args.gpus)
    torch.cuda.set_device(local)
    cpus_before = bind_gpu_local_cpus(local)
    ctx = pf.Context(local)
    peaks, peak_src = measured_peaks()
    sampler = ClockSampler(local)
    sampler.start()

    # ---- headline: config 2 quantized int8 linear layer
    per_copy = M * K + N * K + M * N
    n_copies = max(2, math.ceil(2 * L2_BYTES / per_copy))
    q, copies, fns = qlinear_setup(ctx, n_copies)
    ms, t_soak, t_end = graph_time(fns, args.steps, args.warmup, world)
    ctx.check()
    ops = 2.0 * M * N * K
    value = world * ops / (ms * 1e-3) / 1e12
    achieved = ops / (ms * 1e-3) / 1e12
    int8_peak = 2.0 * peaks["bf16_tflops"]
    clocks = sampler.summary(t_soak, t_end)

    e2e_ms, h2d, d2h, link = qlinear_e2e(ctx, q, copies[0][0], max(200, args.steps))
    sess = session_e2e(q, local, max(100, args.steps), args.warmup)
    if sess is not None:
        # the session's output equals the kernel path's (bit for bit)
        y_ref = copies[0][0](torch.from_numpy(q.a).cuda(), q.a_scale, q.a_zp, out="int8", y_scale=q.y_scale).cpu()
        sess_same = bool(np.array_equal(sess[2], y_ref.numpy()))
        sess_ms = max_over_ranks(sess[0], world)
        sess_one_ms = max_over_ranks(sess[1], world)
    e2e_ms = max_over_ranks(e2e_ms, world)
    h2d_ms = max_over_ranks(link["h2d_only_ms_per_step"], world)
    d2h_ms = max_over_ranks(link["d2h_only_ms_per_step"], world)

    line = {
        "metric": "int8 GEMM TOPS (config 2: u8[512,4096] x s8[4096,4096] -> s8, per-channel)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic (seeded, config 2 shapes and distributions)",
        "config": {"workload": "config2_qlinear_int8", "M_per_rank": M, "N": N, "K": K,
                   "global_batch": M * world, "parallelism": f"batch-shard x{world}",
                   "l2": f"inputs rotate over {n_copies} copies ({n_copies * per_copy / 2**20:.0f} MiB > 2x L2)",
                   "timing": "K steps in one CUDA graph, CUDA events, max over ranks"},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": int8_peak, "unit": "TFLOP/s",
                     "frac": achieved / int8_peak, "traffic": profile_traffic("qlinear_config2"),
                     "frac_of_sustained": achieved / (2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])),
                     "peak_source": f"int8 dense = 2 x bf16_tflops ({peak_src} MEASURED_PEAKS.json); "
                                    f"counts a multiply-add as 2 ops",
                     "kernel": "umma_gemm_sk2_kernel<i8, 256> (1 launch per step: 64 clusters of two CTAs, "
                               "K split between them)"},
        "e2e": {"value": world * ops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms, "path": "pfrt_qlinear_host (C ABI, pinned host buffers: copy in, "
                                                "layer, copy out per call); steps alternate over 3 lanes "
                                                "(context, stream, buffers each)",
                "host_link": {"h2d_gbs": h2d / (h2d_ms * 1e-3) / 1e9, "d2h_gbs": d2h / (d2h_ms * 1e-3) / 1e9,
                              "floor_ms_per_step": max(h2d_ms, d2h_ms),
                              "frac_of_floor": max(h2d_ms, d2h_ms) / e2e_ms,
                              "note": "each direction's copies timed alone in the same lanes; floor = the "
                                      "slower direction (both in flight at once)"},
                "host_enqueue_us_per_step": link["enqueue_us_per_step"]},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }

    if sess is not None:
        line["e2e_session"] = {
            "value": world * ops / (sess_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": sess_ms,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "equals_kernel_path": sess_same,
            "ratio_to_e2e": sess_ms / e2e_ms,
            "one_session_ms_per_run": sess_one_ms,
            "path": "the reference's InferenceSession(device=\"cuda:<gpu>\").run on a .pfm of config 2's layer "
                    "(QuantizedMatMul -> Quantize), pageable host input and output Tensors, one synchronous run() "
                    "per step (libpfrt_session.so: the reference session with the CUDA seam -> CudaBackend); "
                    "3 sessions driven by 3 threads at once, as the e2e object's 3 lanes",
            "timing": "host clock around the runs (run() returns once the output is on the host), max over ranks; "
                      "one_session_ms_per_run: one session alone"}

    # ---- secondary: SpMM (HBM-bound point) and fp32 Gemm
    if not args.no_secondary:
        for obj in copies:
            obj[0].close()
        del copies, fns
        # the 4096^3 int8 GEMM (the tensor-peak target): timed as a burst (the
        # kernel alone, as the burst peak is measured), and after a 1 s soak
        # under the power cap as `sustained`
        cc, cfns, cops = cube_setup(ctx, max(2, math.ceil(2 * L2_BYTES / (3 * 4096 * 4096))))
        cms, c0, c1 = graph_time(cfns, args.steps, args.warmup, world, soak=False)
        ctx.check()
        cclk = sampler.summary(c0, c1)
        sms_, s0c, s1c = graph_time(cfns, args.steps, args.warmup, world)
        ctx.check()
        ca = cops / (cms * 1e-3) / 1e12
        csa = cops / (sms_ * 1e-3) / 1e12
        line["int8_4096"] = {
            "metric": "int8 GEMM TOPS (u8[4096,4096] x s8[4096,4096] -> s8, per-channel)",
            "value": world * ca, "unit": "TFLOP/s", "ms_per_step": cms, "scaling": "weak",
            "timing": "burst: K steps in one CUDA graph replayed right after capture (no soak)",
            "roofline": tensor_roofline(ca, peaks, peak_src, profile_traffic("qlinear_4096")),
            "clocks": cclk,
            "sustained": {"value": world * csa, "ms_per_step": sms_, "timing": "the same replay after a 1 s soak",
                          "frac_of_sustained": csa / (2.0 * peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])),
                          "clocks": sampler.summary(s0c, s1c)},
            "gpu_launches": args.steps,
        }
        for obj in cc:
            obj[0].close()
        del cc, cfns
        if world == 1:
            c, sc, sfns, alg_bytes = spmm_setup(ctx, max(2, math.ceil(2 * L2_BYTES / (8 * 6.7e6))))
            sms, s0_, s1_ = graph_time(sfns, args.steps, args.warmup, world)
            ctx.check()
            gbs = alg_bytes / (sms * 1e-3) / 1e9
            sclk = sampler.summary(s0_, s1_)
            line["spmm"] = {
                "metric": "CSR SpMM HBM GB/s (config 5: M=1, W 8192x8192 90% sparse)",
                "value": gbs, "unit": "GB/s", "ms_per_step": sms, "scaling": "single GPU",
                "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": gbs / peaks["hbm_gbs"], "traffic": profile_traffic("spmm_config5_m1"),
                             "algorithmic_bytes": alg_bytes,
                             "peak_source": f"hbm_gbs ({peak_src} MEASURED_PEAKS.json)"},
                "clocks": sclk,
                "gpu_launches": args.steps,
            }
            for obj in sc:
                obj[0].close()
            line["spmm_config3"] = spmm_config3(ctx, args, peaks, peak_src, sampler)
            line["spmm_structured"] = spmm_structured(ctx, args, peaks, peak_src, sampler)
        else:
            line["spmm"] = spmm_nshard(ctx, args, world, rank, peaks, peak_src)
        line["spmm_sweep"] = spmm_sweep(ctx, args, world, rank, peaks, peak_src, sampler)
        # config 4: the 4-layer int8 MLP, batch 8192 split over the ranks
        ms4, acts4, mfns, mops = mlp_setup(ctx, world, rank)[:4]
        mms, m0_, m1_ = graph_time(mfns, args.steps, args.warmup, world)
        ctx.check()
        mclk = sampler.summary(m0_, m1_)
        ma = mops / (mms * 1e-3) / 1e12
        mroof = tensor_roofline(ma, peaks, peak_src, None)
        mroof["per"] = "GPU"
        line["mlp_config4"] = {
            "metric": "int8 MLP TOPS (config 4: 4 x [MatMul -> Add -> Relu -> uint8], hidden 4096, batch 8192)",
            "value": world * ma, "unit": "TFLOP/s", "ms_per_step": mms,
            "scaling": "strong", "parallelism": f"batch 8192 split {world} ways, no collective",
            "roofline": mroof,
            "clocks": mclk,
            "gpu_launches": MLP_LAYERS * args.steps,
        }
        for ws in ms4:
            for w, _ in ws:
                w.close()
        del ms4, acts4, mfns
        g, gc, gfns = gemm_setup(ctx, 2)
        gms, g0_, g1_ = graph_time(gfns, args.steps, args.warmup, world)
        ctx.check()
        flops = 2.0 * GEMM_M * GEMM_N * GEMM_K
        ga = flops / (gms * 1e-3) / 1e12
        tf32x3 = peaks["bf16_tflops"] / 2.0 / 3.0
        line["gemm_f32"] = {
            "metric": "fp32 Gemm TFLOP/s (config 1: [256,1024] x [1024,1024] + bias, 3xTF32)",
            "value": world * ga, "unit": "TFLOP/s", "ms_per_step": gms,
            "roofline": {"bound": "tensor", "achieved": ga, "peak": tf32x3, "unit": "TFLOP/s", "frac": ga / tf32x3,
                         "frac_of_fp32_simt": ga / FP32_SIMT_TFLOPS, "fp32_simt_tflops": FP32_SIMT_TFLOPS,
                         "peak_source": f"3xTF32 effective = bf16_tflops / 2 (tf32 dense) / 3 (products) "
                                        f"({peak_src} MEASURED_PEAKS.json, derived); FP32 SIMT derived "
                                        f"(148 SMs x 256 flop/clk x 1.965 GHz)"},
            "clocks": sampler.summary(g0_, g1_),
            "note": "0.54 GFLOP per call: the working set fits L2 and the call is latency-bound "
                    "(split of A, GEMM with K split 8 ways, reduction)",
            "gpu_launches": 3 * args.steps,
        }

    if cpus_before is not None:
        os.sched_setaffinity(0, cpus_before)  # the CPU baseline uses every host core
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            line["cpu_baseline"] = cpu_reference_rate()
            one = cpu_reference_rate(budget_s=6.0, threads=1)
            line["cpu_baseline"]["single_core"] = {"value": one["value"], "unit": one["unit"], "cores": 1,
                                                   "sample": one["sample"]}
            line["cpu_baseline"]["host_cores"] = os.cpu_count()
            line["cpu_baseline"]["note"] = ("the reference's CPU backend is single-threaded by construction "
                                            "(src/backends/cpu/executor.cpp:10): single_core is 1 core of a "
                                            f"{os.cpu_count()}-core host; value runs it on row slices over all "
                                            "host threads (harness parallelism)")
        except Exception as e:  # the compiled reference is missing
            line["cpu_baseline"] = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "reference",
                                    "sample": f"unavailable: {e}"}
    sampler.stop()
    ctx.close()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
