"""Benchmark of the mHC-lite hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|reference-triton]

Metric: tokens/s fwd+bwd per GPU and % HBM roofline of
K1/K3/K4 at T=65536, C=1024, n=4 (the kernel-level microbench config).  One
step is one forward+backward pass of the hot path over a batch of T tokens:

    K1 fwd -> K3 fwd -> K4 fwd -> K4 bwd -> K3 bwd -> K1 bwd (grad_x and grad_W)

through ``torch.ops.flash_mhc`` (the reference's op API, each op one C-ABI
call), on seeded synthetic inputs with the reference microbench's
distributions (x, lo, upstream grads ~N(0,1) bf16; W ~N(0,0.02) bf16;
h_pre/h_post/H ~N(0,1) f32).  With N > 1 (torchrun, one rank per GPU) every
rank runs its own T-token shard (weak scaling) and the K1 weight gradient is
all-reduced over NCCL, the path's only exchange.

* ``value``: whole-job tokens/s with inputs resident in HBM (max step time over
  ranks, CUDA events on the launching stream at the ends of the timed region).
  Inputs (x alone is 512 MiB) exceed the 126 MB L2, so no flush is needed
  between steps.  Each timed region starts after a barrier and a synchronize,
  then a fixed-length GPU sleep (``--launch-lead-ms``, outside the events) so
  the host can enqueue the region before the GPU reaches it; Python's garbage
  collector is off inside it.  With N > 1 the grad_W all-reduce of step i runs
  on a side stream after step i+1's K4 forward; ``per_gpu`` carries the
  per-GPU figure (BASELINE's metric name says "per GPU").
* ``roofline``: the dominant kernel (K4 backward) -- algorithmic bytes per
  launch (the reference's bytes model, scripts/benchmark_kernels.py:64-105)
  over its CUDA-event duration, measured in a second timed region of the same
  steps with an event pair around every op, against the measured HBM copy
  bandwidth in MEASURED_PEAKS.json.
* ``e2e``: the same step from pinned host buffers, host->device copies of every
  input and device->host copies of every output inside the timed region.
* ``cpu_baseline``: the reference's own CPU implementation of the path (its
  pure-PyTorch block code from the unmodified reference installed in
  ``baseline/_ref``, float32, every host core) on a bounded token sample,
  rank 0 at N = 1 only, run in a child process; ``configs0`` inside it is
  BASELINE configs[0] (the reference's ``MHCLiteBlock`` fwd+bwd on CPU at
  T=4096, C=1024).
* ``--impl reference``: the reference arm: the same reference code on the
  full per-GPU batch (T tokens) per step, rank 0 only.  Where
  ``baseline/_ref`` is missing it falls back to the float32 numpy
  restatement under ``oracle/`` (``kind: "port"``).
* ``block``: ``MHCLiteBlock`` fwd+bwd at BASELINE configs[2] (T=65536 per GPU,
  C=2048, Linear(2048, 2048)); with N > 1 its gradients are all-reduced by
  ``flash_mhc.distributed.BucketedGradReducer`` during the backward.
* ``large``: BASELINE configs[3] per GPU (131,072 tokens, C=4096): the hot-path
  step and the block with the 4096 -> 4096 linear, at every N.
* ``small_batch_graphs`` / ``tiny_inference``: the hot path at T=8192 eager vs
  CUDA-graph replay, and the no-grad block forward at T=1/16/256.
* ``--impl reference-triton``: a comparison line, not the reference arm -- the
  unmodified reference's Triton kernels and block, installed in
  ``baseline/_ref``, timed on this GPU on the same shapes and seeds.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "flash-mhc_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "tokens/s fwd+bwd per GPU and % HBM roofline (K1/K3/K4) at T=65536,C=1024,n=4"
UNIT = "tokens/s"
D_OUT = 32
N_STREAMS = 4


def bytes_model(T: int, C: int, n: int = N_STREAMS, D: int = D_OUT) -> dict:
    """Algorithmic (mandatory) HBM bytes per launch, per kernel.

    The reference's model (scripts/benchmark_kernels.py:64-105) for the six
    kernels; K1's backward here also produces grad_W, so it adds the grad_W
    write (D*nC bf16) to the reference's K1 bwd-dx figure.
    """
    bf, f4 = 2, 4
    nC = n * C
    return {
        "k1_fwd": T * nC * bf + D * nC * bf + T * D * bf + T * f4,
        "k3_fwd": T * n * C * bf + T * n * f4 + T * C * bf,
        "k4_fwd": T * n * C * bf + T * C * bf + T * n * n * f4 + T * n * f4 + T * n * C * bf,
        "k4_bwd": 2 * T * n * C * bf + T * C * bf + T * n * n * f4 + T * n * f4
        + T * n * C * bf + T * C * bf + T * n * n * f4 + T * n * f4,
        "k3_bwd": T * n * C * bf + T * n * f4 + T * C * bf + T * n * C * bf + T * n * f4,
        "k1_bwd": 2 * T * nC * bf + D * nC * bf + 2 * T * D * bf + T * f4 + D * nC * bf,
    }


class _NoGC:
    """Python's garbage collector off inside a timed region (collected just
    before): a collection pause on one rank would otherwise stall that rank's
    launches, and with a per-step collective the other ranks wait too."""

    def __enter__(self):
        import gc

        gc.collect()
        gc.disable()
        return self

    def __exit__(self, *exc):
        import gc

        gc.enable()


def _launch_lead(torch, ms):
    """Keep the GPU busy for ``ms`` (a fixed-length sleep kernel on the current
    stream, bounded by construction) before a timed region's start event, so the
    host can enqueue the region's launches before the GPU reaches them: a host
    stall on one rank (shared host CPUs, NCCL's helper threads) then no longer
    drains that rank's queue, which with a per-step collective would stall every
    rank.  The sleep itself is outside the timed events.  (nvbench's blocking
    kernel serves the same purpose.)"""
    if ms > 0:
        torch.cuda._sleep(int(ms * 2.0e6))  # ~2 GHz SM clock: cycles per ms


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "src": "measured"}
    return {"hbm_gbs": 6650.0, "src": "fallback"}


def dram_traffic() -> dict:
    """Per-launch DRAM bytes per kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if p.exists():
        return json.loads(p.read_text())
    return {}


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples SM clock and throttle reasons of the given GPUs during a region.

    Polls NVML (read-only queries) from a background thread every few ms, so
    even a timed region of a few tens of ms gets samples.
    """

    REASONS = {  # NVML clocks-event reason bits
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "sw_power_cap": 0x4,
    }

    def __init__(self, gpu_indices, period_s=0.005):
        self.idx = list(gpu_indices)
        self.period = period_s
        self.samples = []  # (sm_mhz, max_mhz, reasons_bitmask)
        self._stop = None
        self._thread = None
        self.err = None

    def __enter__(self):
        if not self.idx:
            return self
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in self.idx]
            maxes = [pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM) for h in handles]
        except Exception as e:  # pragma: no cover - depends on the box
            self.err = f"nvml unavailable: {e}"
            return self
        self._stop = threading.Event()

        def loop():
            while not self._stop.is_set():
                for h, mx in zip(handles, maxes):
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, mx, rs))
                    except Exception as e:  # pragma: no cover
                        self.err = str(e)
                self._stop.wait(self.period)

        self._thread = threading.Thread(target=loop, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None,
                    "reasons": [self.err or "no samples"]}
        sm = [s[0] for s in self.samples]
        reasons = set()
        for _, _, rs in self.samples:
            for name, bit in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(s[1] for s in self.samples),
                "sm_min_mhz": min(sm), "samples": len(sm), "source": "nvml",
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# the GPU step
# ---------------------------------------------------------------------------

class HotPath:
    """Inputs and the fwd+bwd step of the hot path on one GPU."""

    # kernels of this library launched per step (8): K1 fwd, K3 fwd, K4 fwd,
    # K4 bwd, K3 bwd, and K1 bwd as prep (gos, s/inv_rms) + the fused
    # grad_x/grad_W kernel + the grad_W reduction
    def __init__(self, T, C, device, seed, torch):
        self.torch = torch
        self.T, self.C = T, C
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        n, D = N_STREAMS, D_OUT
        bf = torch.bfloat16

        def rn(*shape, std=1.0, dtype=bf):
            return (torch.randn(*shape, generator=g, device=device) * std).to(dtype)

        self.inputs = {
            "x": rn(T, n, C), "W": rn(D, n * C, std=0.02), "lo": rn(T, C),
            "h_pre": rn(T, n, dtype=torch.float32), "h_post": rn(T, n, dtype=torch.float32),
            "H": rn(T, n, n, dtype=torch.float32), "g_proj": rn(T, D), "g_pre": rn(T, C),
            "g_post": rn(T, n, C),
        }

    def step(self, inp, events=None, after_k4_fwd=None):
        """One pass; ``events`` (dict name -> list) gets (start, end) event pairs;
        ``after_k4_fwd`` is called once K4's forward is enqueued."""
        torch = self.torch
        ops = torch.ops.flash_mhc
        T, C = self.T, self.C
        x = inp["x"]
        xf = x.reshape(T, N_STREAMS * C)
        outs = {}

        def rec(name, fn):
            if events is None:
                return fn()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            r = fn()
            e.record()
            events.setdefault(name, []).append((s, e))
            return r

        outs["proj"], outs["inv_rms"] = rec("k1_fwd", lambda: ops.fused_rmsnorm_project(xf, inp["W"]))
        outs["layer_input"] = rec("k3_fwd", lambda: ops.fused_pre_map(x, inp["h_pre"]))
        outs["out"] = rec("k4_fwd", lambda: ops.fused_post_res(x, inp["lo"], inp["H"], inp["h_post"]))
        if after_k4_fwd is not None:
            after_k4_fwd()
        (outs["gx4"], outs["glo"], outs["gH"], outs["ghp"]) = rec(
            "k4_bwd", lambda: ops.fused_post_res_backward(inp["g_post"], x, inp["lo"], inp["H"],
                                                          inp["h_post"]))
        outs["gx3"], outs["gh3"] = rec(
            "k3_bwd", lambda: ops.fused_pre_map_backward(inp["g_pre"], x, inp["h_pre"]))
        outs["gx1"], outs["gW"] = rec(
            "k1_bwd", lambda: ops.fused_rmsnorm_project_backward(inp["g_proj"], xf, inp["W"],
                                                                 outs["proj"], outs["inv_rms"]))
        return outs

    # K1f, K3f, K4f, K4b, K3b, K1b main kernel + its grad_W reduce
    LAUNCHES_PER_STEP = 7


def _allreduce_gw(torch, dist, outs):
    buf = outs["gW"].float()
    dist.all_reduce(buf)
    return buf


def _stepper(hp, torch, dist, world):
    """(one_step, join_comm) for the hot path on ``world`` ranks.

    With N > 1 the weight-gradient all-reduce of step i (the path's only
    exchange; nothing in step i+1 reads grad_W) is issued on a side stream
    during step i+1, ordered after that step's K4 forward, so NCCL's kernel runs
    beside the streaming K4/K3 backward instead of competing for SMs and L2
    with the persistent K1 forward that starts the step.  ``join_comm`` issues
    the last step's all-reduce and makes the current stream wait for it; every
    timed region ends with it.
    """
    if world == 1:
        return (lambda events=None: hp.step(hp.inputs, events)), (lambda: None)
    s_comm = torch.cuda.Stream()
    # The previous step's grad_W, not reduced yet.  Only grad_W is kept: holding
    # the whole output set across steps would change the allocator's reuse of
    # the (T, 4, C) output blocks (4 GiB each at configs[3]).
    pending = []

    def launch_pending():
        if not pending:
            return
        prev = pending.pop()
        ready = torch.cuda.Event()
        ready.record()
        s_comm.wait_event(ready)
        with torch.cuda.stream(s_comm):
            prev["gW_all"] = _allreduce_gw(torch, dist, prev)
            prev["gW"].record_stream(s_comm)

    def one_step(events=None):
        outs = hp.step(hp.inputs, events, after_k4_fwd=launch_pending)
        pending.append({"gW": outs["gW"]})
        return outs

    def join_comm():
        launch_pending()
        torch.cuda.current_stream().wait_stream(s_comm)

    return one_step, join_comm


def run_ours(args):
    import torch
    import torch.distributed as dist

    import flash_mhc  # noqa: F401  (registers the ops)
    from flash_mhc import _native

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        opts = dist.ProcessGroupNCCL.Options()
        if args.nccl_max_ctas > 0:
            opts.config.max_ctas = args.nccl_max_ctas
        if args.nccl_nvls_ctas > 0:
            opts.config.nvls_ctas = args.nccl_nvls_ctas
        if args.nccl_cta_policy >= 0:
            opts.config.cta_policy = args.nccl_cta_policy
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev,
                                pg_options=opts)

    if world > 1 and args.compute_priority == "high":
        # Optional: this library's kernels (and the layer's) on a high-priority
        # stream, NCCL's on its default-priority stream, so pending compute
        # CTAs are dispatched before a collective's.  Backward nodes and the
        # gradient hooks run on the stream of their forward, so this covers the
        # block too.  Measured on 2 GPUs: no difference (block 3.50-3.51 ms
        # either way), so it is off by default.
        torch.cuda.set_stream(torch.cuda.Stream(priority=-1))

    T, C = args.T, args.C
    hp = HotPath(T, C, dev, seed=1234 + rank, torch=torch)
    lib_path = str(_native.library_path())
    one_step, join_comm = _stepper(hp, torch, dist, world)

    # --- device-resident timing -------------------------------------------
    for _ in range(args.warmup):
        one_step()
    join_comm()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    # Two timed regions of `steps` steps each.  The first has events only at
    # its ends and gives `value`; the second records an event pair around
    # every op (these records cost ~30 us per step, so they are kept out of the
    # headline) and gives the per-kernel durations behind `kernels` and
    # `roofline`.  The clock sampler runs across both.
    events = {}
    phys = _physical_gpu_indices(world)
    with ClockSampler(phys if rank == 0 else []) as clk, _NoGC():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        _launch_lead(torch, args.launch_lead_ms)
        t0.record()
        for _ in range(args.steps):
            one_step()
        join_comm()
        t1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for _ in range(args.steps):
            one_step(events)
        join_comm()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = t0.elapsed_time(t1) / args.steps
    kern_ms = {k: sum(s.elapsed_time(e) for s, e in v) / len(v) for k, v in events.items()}
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())

    # --- end-to-end from host buffers --------------------------------------
    e2e = None if args.no_e2e else run_e2e(args, hp, one_step, torch, dist, world, dev)
    del hp, one_step, join_comm  # the step closures hold the inputs and last outputs
    torch.cuda.empty_cache()

    # --- the whole block ------------------------------
    block = None if args.no_block else run_block(args, torch, dist, world, dev)

    # --- the large token-sharded config ---------------
    large = None if args.no_large else run_large(args, torch, dist, world, dev)

    # --- small per-GPU batch: eager vs CUDA-graph replay -------------------
    graphs = None if args.no_graphs else run_small_graphs(args, torch, dev)

    # --- tiny-T no-grad inference latency (BASELINE configs[4] shapes) -------
    tiny = None if (args.no_tiny or world > 1) else run_tiny_inference(args, torch, dev)

    if rank == 0:
        peaks = measured_peaks()
        bm = bytes_model(T, C)
        traffic = dram_traffic()
        def traffic_of(k):
            # ncu DRAM bytes per launch, scaled from a small capture; they apply
            # only to the (T, C) they were scaled to
            cap = traffic.get(k, {}) if traffic else {}
            return (cap.get("bytes_per_launch_full")
                    if cap.get("full_T") == T and cap.get("C", C) == C else None)

        kernels = {}
        for k, v in kern_ms.items():
            gbs = bm[k] / (v * 1e-3) / 1e9
            kernels[k] = {"ms": round(v, 5), "bytes": bm[k], "GBps": round(gbs, 1),
                          "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": traffic_of(k)}
        dom = "k4_bwd"
        ach = bm[dom] / (kern_ms[dom] * 1e-3) / 1e9
        tr = traffic_of(dom)
        sum_bytes = sum(bm.values())
        line = {
            "metric": METRIC, "value": round(world * T / (ms * 1e-3), 1), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) x/lo/grads, N(0,0.02) W, N(0,1) f32 coefficients)",
            "config": workload_config(T, C, world),
            "timing": "value: steps timed with events at the region's ends only; "
                      "kernels/roofline: a second region of the same steps with an "
                      "event pair around every op",
            # BASELINE's metric name says "per GPU"; `value` is the whole-job
            # figure the bench contract asks for, and this is the per-GPU one.
            "value_scope": "whole job: tokens/s over all n_gpus GPUs",
            "per_gpu": {"value": round(T / (ms * 1e-3), 1), "unit": "tokens/s per GPU"},
            "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(ach, 1),
                         "peak": peaks["hbm_gbs"], "peak_src": peaks["src"], "unit": "GB/s",
                         "frac": round(ach / peaks["hbm_gbs"], 4),
                         "traffic": tr, "algorithmic_bytes": bm[dom]},
            # algorithmic bytes of the whole step over the step time (gaps included)
            "hot_path_hbm_frac": round(sum_bytes / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
            "kernels": kernels,
            "e2e": e2e,
            "block": block,
            "large": large,
            "small_batch_graphs": graphs,
            "tiny_inference": tiny,
            "gpu_launches": HotPath.LAUNCHES_PER_STEP * args.steps,
            "clocks": clk.summary(),
            "comm": None if world == 1 else {
                "grad_w_allreduce": "f32, on a side stream after the next step's K4 forward",
                "block_grad_allreduce": (f"BucketedGradReducer, {args.block_buckets} bucket(s), "
                                         f"{args.block_reduce_op}"
                                         if args.block_allreduce == "bucketed" else
                                         "allreduce_gradients: one bucket after the backward"),
                "compute_stream_priority": args.compute_priority,
                "nccl_max_ctas": args.nccl_max_ctas or "default",
                "nccl_nvls_ctas": args.nccl_nvls_ctas or "default",
                "nccl_cta_policy": args.nccl_cta_policy if args.nccl_cta_policy >= 0 else "default"},
            "native_lib": os.path.relpath(lib_path, ROOT),
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(args)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _physical_gpu_indices(world):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        try:
            return [int(i) for i in ids[:world]]
        except ValueError:
            pass
    return list(range(world))


def run_tiny_inference(args, torch, dev):
    """Latency of one no-grad MHCLiteBlock forward at tiny token counts
    (T in {1, 16, 256}, C = 768, n = 4 bf16, x ~N(0,1)
    with 1% of channels x100, projection weights ~N(0,0.02), wrapped
    768 -> 768 bias-free linear), eager and replayed from a CUDA graph.
    Microseconds per forward, averaged over 200 back-to-back calls; with one
    forward per graph replay (graph_us) and with 20 forwards captured in one
    graph (graph_x20_us, per forward)."""
    import torch.nn as nn

    from flash_mhc import MHCLiteBlock

    C = 768
    g = torch.Generator(device=dev)
    g.manual_seed(123)
    layer = nn.Linear(C, C, bias=False)
    blk = MHCLiteBlock(4, C, layer).to(dev).to(torch.bfloat16).eval()
    with torch.no_grad():
        blk.W_all.weight.copy_(torch.randn(blk.W_all.weight.shape, generator=g, device=dev) * 0.02)
        layer.weight.copy_(torch.randn(C, C, generator=g, device=dev) * 0.02)
    cols = torch.randperm(C, generator=torch.Generator().manual_seed(5))[: C // 100].to(dev)
    n = 200
    out = {}
    for T in (1, 16, 256):
        x = torch.randn(T, N_STREAMS, C, generator=g, device=dev)
        x[:, :, cols] *= 100.0
        x = x.bfloat16()

        def fwd():
            with torch.no_grad():
                return blk(x)

        def timed(fn):
            for _ in range(10):
                fn()
            torch.cuda.synchronize()
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(n):
                fn()
            e.record()
            torch.cuda.synchronize()
            return s.elapsed_time(e) / n * 1e3

        eager_us = timed(fwd)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fwd()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fwd()
        graph_us = timed(graph.replay)
        del graph
        # 20 forwards in one graph: the device time of a forward without the
        # per-replay launch of the graph itself
        graph20 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph20):
            for _ in range(20):
                fwd()
        graph20_us = timed(graph20.replay) / 20
        del graph20
        out[str(T)] = {"eager_us": round(eager_us, 2), "graph_us": round(graph_us, 2),
                       "graph_x20_us": round(graph20_us, 2)}
    return {"config": {"workload": "MHCLiteBlock no-grad forward (configs[4] tiny-T shapes)",
                       "C": C, "n": N_STREAMS, "layer": "nn.Linear(768, 768, bias=False)",
                       "x": "N(0,1), 1% of channels x100"},
            "calls": n, "latency_per_forward": out}


def run_small_graphs(args, torch, dev):
    """The hot-path step at a small per-GPU batch (the 8-GPU strong-scaling
    shard of the metric batch, T = 65536/8), launched eagerly and replayed
    from a CUDA graph; host launch overhead dominates the eager step here."""
    T = args.small_T
    hp = HotPath(T, args.C, dev, seed=99, torch=torch)
    n = 50

    def timed(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / n

    eager_ms = timed(lambda: hp.step(hp.inputs))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            hp.step(hp.inputs)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        hp.step(hp.inputs)
    graph_ms = timed(graph.replay)
    del graph
    return {"T_per_gpu": T, "C": args.C, "steps": n,
            "eager_ms_per_step": round(eager_ms, 4), "graph_ms_per_step": round(graph_ms, 4),
            "eager_tokens_per_s": round(T / (eager_ms * 1e-3), 1),
            "graph_tokens_per_s": round(T / (graph_ms * 1e-3), 1)}


def run_block(args, torch, dist, world, dev, T=None, C=None, workload=None):
    """MHCLiteBlock fwd+bwd with activation checkpointing:
    T tokens per GPU, C=2048, n=4 bf16, wrapped nn.Linear(C, C, bias=False)
    ~N(0,0.02), upstream grad ~N(0,1).  With N GPUs every parameter gradient
    is all-reduced each step by ``BucketedGradReducer``: the layer's gradient
    starts reducing as soon as the layer's backward has produced it, while the
    block's K3/K2/K1 backward and grad_x combination still run; the block's
    own gradients follow at the end."""
    import torch.nn as nn

    from flash_mhc import MHCLiteBlock
    from flash_mhc.distributed import BucketedGradReducer, allreduce_gradients

    T = T or args.block_T
    C = C or args.block_C
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    layer = nn.Linear(C, C, bias=False)
    blk = MHCLiteBlock(4, C, layer, triton_fused=True, activation_checkpointing=True)
    blk = blk.to(dev).to(torch.bfloat16).train()
    with torch.no_grad():
        layer.weight.copy_((torch.randn(C, C, generator=g, device=dev) * 0.02).bfloat16())
    x = torch.randn(T, N_STREAMS, C, generator=g, device=dev).bfloat16().requires_grad_(True)
    up = torch.randn(T, N_STREAMS, C, generator=g, device=dev).bfloat16()
    reducer = None
    if world > 1 and args.block_allreduce == "bucketed":
        # 2: the layer's bucket reduces during the backward, the block's own at
        # its end; 1: one bucket, reduced when the last gradient arrives
        reducer = BucketedGradReducer(
            blk, buckets=None if args.block_buckets == 2 else [list(blk.parameters())],
            avg_op=args.block_reduce_op == "avg")

    def step():
        blk.zero_grad(set_to_none=True)
        x.grad = None
        out = blk(x)
        out.backward(up)
        if reducer is not None:
            reducer.finish()
        elif world > 1:
            allreduce_gradients(blk)  # one f32 bucket after the backward

    steps = max(1, min(args.steps, 10))
    for _ in range(max(3, min(args.warmup, 5))):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    with _NoGC():
        _launch_lead(torch, args.launch_lead_ms)
        s.record()
        for _ in range(steps):
            step()
        e.record()
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    if reducer is not None:
        reducer.remove()
    flops = 3 * 2 * T * C * C  # the wrapped layer's fwd + 2 bwd GEMMs
    return {"config": {"workload": workload or "MHCLiteBlock fwd+bwd, activation checkpointing "
                                               "(configs[2])",
                       "T_per_gpu": T, "C": C, "n": N_STREAMS,
                       "layer": f"nn.Linear({C}, {C}, bias=False) ~N(0,0.02)",
                       "grad_allreduce": ("none (1 GPU)" if world == 1 else
                                          "allreduce_gradients: one f32 bucket after the backward"
                                          if args.block_allreduce == "after" else
                                          "BucketedGradReducer: layer bucket during the backward, "
                                          "block's own at its end" if args.block_buckets == 2 else
                                          "BucketedGradReducer: one bucket at the end of the backward")},
            "value": round(world * T / (ms * 1e-3), 1), "unit": UNIT, "ms_per_step": round(ms, 4),
            "steps": steps, "layer_gemm_tflops_per_step": round(flops / 1e12, 3)}


def run_large(args, torch, dist, world, dev):
    """BASELINE configs[3], the large token-sharded run, per GPU: 131,072
    tokens per GPU (global T = 131,072 x N; 1,048,576 on 8 GPUs), C = 4096,
    n = 4 bf16.  (1) The hot-path step (same six ops and the grad_W all-reduce
    as the headline, 2 MiB of f32 per step); (2) the MHCLiteBlock fwd+bwd with
    the wrapped 4096 -> 4096 bias-free linear, whose 64 MiB f32 gradient is
    all-reduced with the block's own.  Weak scaling: the per-GPU work is fixed.
    Each (T, 4, C) bf16 tensor holds 4 GiB."""
    T, C = args.large_T, args.large_C
    hp = HotPath(T, C, dev, seed=4321 + int(os.environ.get("RANK", "0")), torch=torch)
    one_step, join_comm = _stepper(hp, torch, dist, world)
    steps = max(1, min(args.steps, 10))
    for _ in range(3):
        one_step()
    join_comm()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    with _NoGC():
        _launch_lead(torch, args.launch_lead_ms)
        s.record()
        for _ in range(steps):
            one_step()
        join_comm()
        e.record()
        torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    del hp, one_step, join_comm
    torch.cuda.empty_cache()
    bm = sum(bytes_model(T, C).values())
    peaks = measured_peaks()
    out = {"config": {"workload": "large token-sharded hot path fwd+bwd (configs[3])",
                      "T_per_gpu": T, "global_T": T * world, "C": C, "n": N_STREAMS,
                      "parallelism": f"token-sharded dp{world}",
                      "l2": "inputs larger than L2 (x alone 4 GiB), no flush"},
           "value": round(world * T / (ms * 1e-3), 1), "unit": UNIT, "ms_per_step": round(ms, 4),
           "steps": steps,
           "hot_path_hbm_frac": round(bm / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)}
    if not args.no_block:
        out["block"] = run_block(args, torch, dist, world, dev, T=T, C=C,
                                 workload="MHCLiteBlock fwd+bwd, activation checkpointing, "
                                          "large token-sharded config (configs[3])")
        torch.cuda.empty_cache()
    return out


def run_e2e(args, hp, one_step, torch, dist, world, dev):
    """Same step from pinned host buffers: every step copies all of its inputs
    host->device and all of its outputs device->host inside the timed region.

    Steps are software-pipelined over three streams (the way a host caller
    would drive the API): the inputs of step i+1 upload on one copy stream
    while step i computes and the outputs of step i-1 download on the other,
    with events ordering each buffer's reuse.  Two device input sets alternate.
    """
    host_in = {k: v.cpu().pin_memory() for k, v in hp.inputs.items()}
    sample = hp.step(hp.inputs)
    host_out = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in sample.items()}
    h2d = sum(v.numel() * v.element_size() for v in host_in.values())
    d2h = sum(v.numel() * v.element_size() for v in host_out.values())
    del sample
    dev_in = [{k: torch.empty_like(v) for k, v in hp.inputs.items()} for _ in range(2)]
    s_in, s_comp, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    for e in ev_free:
        e.record(torch.cuda.current_stream())

    def run(nsteps):
        for i in range(nsteps + 1):
            if i < nsteps:  # upload step i
                b = i % 2
                with torch.cuda.stream(s_in):
                    s_in.wait_event(ev_free[b])
                    for k, v in host_in.items():
                        dev_in[b][k].copy_(v, non_blocking=True)
                    ev_in[b].record(s_in)
            if i >= 1:  # compute step i-1, then download its outputs
                b = (i - 1) % 2
                with torch.cuda.stream(s_comp):
                    s_comp.wait_event(ev_in[b])
                    outs = hp.step(dev_in[b])
                    if world > 1:
                        outs["gW"] = _allreduce_gw(torch, dist, outs).to(outs["gW"].dtype)
                    ev_free[b].record(s_comp)
                    done = torch.cuda.Event()
                    done.record(s_comp)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(done)
                    for k, v in outs.items():
                        if k in host_out:
                            host_out[k].copy_(v, non_blocking=True)
                            v.record_stream(s_out)
        torch.cuda.synchronize()

    steps = max(2, min(args.steps, 8))
    run(max(1, min(args.warmup, 2)))
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with _NoGC():
        start.record(s_in)
        run(steps)
        end.record(s_out)
        torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    wall_ms = (time.perf_counter() - t0) * 1e3 / steps
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    return {"value": round(world * hp.T / (ms * 1e-3), 1), "unit": UNIT, "ms_per_step": round(ms, 3),
            "wall_ms_per_step": round(wall_ms, 3), "steps": steps,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "api": "torch.ops.flash_mhc (ctypes -> C ABI), pinned host buffers, "
                   "copies pipelined across steps on two copy streams"}


# ---------------------------------------------------------------------------
# CPU baselines.  The reference's own CPU implementation of the path is its
# pure-PyTorch block code (src/flash_mhc/block.py:82-148), run from the
# unmodified reference installed in baseline/_ref; the float32 numpy
# restatement under oracle/ stands in only when that install is missing.
# ---------------------------------------------------------------------------

REF_DIR = ROOT / "baseline" / "_ref"


def _reference_installed() -> bool:
    return (REF_DIR / "flash_mhc" / "__init__.py").is_file()


def _import_reference():
    """Import the reference package from baseline/_ref instead of this
    repository's (both are named ``flash_mhc`` and define the same
    torch.library namespace, so this process must not have imported ours)."""
    mod = sys.modules.get("flash_mhc")
    if mod is not None and REF_DIR.resolve() not in Path(mod.__file__).resolve().parents:
        raise RuntimeError("this repository's flash_mhc is imported in this process; "
                           "the reference must run in a process of its own")
    sys.path[:] = [p for p in sys.path
                   if Path(p or ".").resolve() not in (ROOT, ROOT / "flash-mhc_b200")]
    sys.path.insert(0, str(REF_DIR))
    import flash_mhc as ref  # the reference package

    if REF_DIR.resolve() not in Path(ref.__file__).resolve().parents:
        raise RuntimeError(f"expected the reference from {REF_DIR}, got {ref.__file__}")
    return ref


def _host_cores() -> int:
    return len(os.sched_getaffinity(0))


def _ref_cpu_hot_path(ref, T, C, steps, warmup, seed=1234):
    """The hot-path step through the reference's own pure-PyTorch code, float32
    on the host cores: ``_mhc_pre_map_pytorch`` (K1 as F.rms_norm + F.linear,
    K2, K3; block.py:82-110) and ``_mhc_post_res_pytorch`` (K4; block.py:112-124)
    forward, then one autograd backward from upstream gradients of the layer
    input and the block output (K4, K3, K2 and K1 backward, including the
    projection-weight gradient).  Inputs have the GPU arm's distributions;
    ``W_all`` keeps the reference's default init.  Returns per-step seconds."""
    import torch
    import torch.nn as nn

    torch.manual_seed(seed)
    blk = ref.MHCLiteBlock(N_STREAMS, C, nn.Identity())  # the layer itself is not called
    x = torch.randn(T, N_STREAMS, C).requires_grad_(True)
    lo = torch.randn(T, C).requires_grad_(True)
    g_pre = torch.randn(T, C)
    g_post = torch.randn(T, N_STREAMS, C)

    def step():
        blk.zero_grad(set_to_none=True)
        x.grad = None
        lo.grad = None
        layer_input, H_merged, h_post = blk._mhc_pre_map_pytorch(x)
        out = blk._mhc_post_res_pytorch(x, lo, H_merged, h_post)
        torch.autograd.backward([layer_input, out], [g_pre, g_post])

    for _ in range(warmup):
        step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    return times


def _ref_cpu_configs0(ref, iters=5):
    """the reference's ``MHCLiteBlock`` forward+backward on
    the CPU (its pure-PyTorch path, block.py:126-148), float32, n=4, C=1024,
    T=4096, x ~N(0,1), wrapped nn.Linear(1024, 1024, bias=False) ~N(0,0.02),
    default coefficient-projection init, no activation checkpointing, seed 0.
    One warm-up iteration, then the median of ``iters``."""
    import torch
    import torch.nn as nn

    T, C = 4096, 1024
    torch.manual_seed(0)
    layer = nn.Linear(C, C, bias=False)
    with torch.no_grad():
        layer.weight.normal_(0.0, 0.02)
    blk = ref.MHCLiteBlock(N_STREAMS, C, layer).train()
    x = torch.randn(T, N_STREAMS, C).requires_grad_(True)
    up = torch.randn(T, N_STREAMS, C)

    def step():
        blk.zero_grad(set_to_none=True)
        x.grad = None
        blk(x).backward(up)  # CPU input: the reference dispatches to _forward_pytorch

    step()
    ts = []
    for _ in range(iters):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    med = statistics.median(ts)
    return {"value": round(T / med, 1), "unit": UNIT, "ms_per_iter": round(med * 1e3, 2),
            "iters": iters, "cores": _host_cores(), "kind": "reference",
            "workload": "configs[0]: MHCLiteBlock fwd+bwd, pure-PyTorch path, float32, T=4096, "
                        "C=1024, n=4, Linear(1024, 1024, bias=False) ~N(0,0.02), default init, "
                        "seed 0",
            "source": "unmodified reference in baseline/_ref, MHCLiteBlock.forward on CPU "
                      "(src/flash_mhc/block.py:126-148)"}

def _cpu_worker(args):
    import numpy as np
    from oracle import mhc_oracle as O

    T, C, seed, reps = args
    rng = np.random.default_rng(seed)
    x = O.bf16_round(rng.standard_normal((T, 4, C)))
    W = O.bf16_round(rng.standard_normal((32, 4 * C)) * 0.02)
    lo = O.bf16_round(rng.standard_normal((T, C)))
    H = rng.standard_normal((T, 4, 4)).astype(np.float32)
    hq = rng.standard_normal((T, 4)).astype(np.float32)
    hp = rng.standard_normal((T, 4)).astype(np.float32)
    gp = O.bf16_round(rng.standard_normal((T, 32)))
    g3 = O.bf16_round(rng.standard_normal((T, C)))
    g4 = O.bf16_round(rng.standard_normal((T, 4, C)))
    t0 = time.perf_counter()
    for _ in range(reps):
        O.hot_path_step_f32(x, W, lo, H, hq, hp, gp, g3, g4)
    return time.perf_counter() - t0


class CpuPool:
    """A spawn process pool (one process per core) running the float32 numpy
    restatement (the fallback when the reference is not installed)."""

    def __init__(self, C, workers):
        import multiprocessing as mp

        self.C, self.workers = C, workers
        os.environ.setdefault("OMP_NUM_THREADS", "1")
        os.environ.setdefault("OPENBLAS_NUM_THREADS", "1")
        self.pool = mp.get_context("spawn").Pool(workers)
        self.pool.map(_cpu_worker, [(8, C, 0, 1)] * workers)  # imports, first touch

    def run(self, tokens_per_worker, reps, seed=100):
        """Wall seconds of every worker running ``reps`` steps of its tokens."""
        t0 = time.perf_counter()
        self.pool.map(_cpu_worker, [(tokens_per_worker, self.C, seed + i, reps)
                                    for i in range(self.workers)])
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()


def workload_config(T, C, world):
    """The ``config`` object both arms print (the same workload)."""
    return {"workload": "kernel-level hot path fwd+bwd (configs[1] shapes)",
            "T_per_gpu": T, "C": C, "n": N_STREAMS, "D": D_OUT,
            "step": "K1f,K3f,K4f,K4b,K3b,K1b(dx+dW)" + (",allreduce(gW)" if world > 1 else ""),
            "parallelism": f"token-sharded dp{world}",
            "l2": f"inputs larger than L2 (x alone {T * N_STREAMS * C * 2 / 2**20:.0f} MiB), "
                  "no flush"}


def run_reference(args):
    """The reference arm: the reference's own CPU implementation of the path
    on this box's host cores (rank 0 only; other ranks exit without work).

    With the reference installed in baseline/_ref, each step is
    ``_ref_cpu_hot_path`` over ``--ref-tokens`` tokens (default: the full
    per-GPU batch, T) with every host core (torch intra-op threads), plus the
    configs[0] block timing.  Without it, the float32 numpy restatement on one
    spawn process per core over a bounded token sample (``kind: "port"``).
    """
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    cores = _host_cores()
    T, C = args.T, args.C
    if _reference_installed() and args.ref_kind == "reference":
        ref = _import_reference()
        import torch

        torch.set_num_threads(cores)
        tok = min(args.ref_tokens or T, T)
        times = _ref_cpu_hot_path(ref, tok, C, args.steps, args.warmup)
        ms = 1e3 * sum(times) / len(times)
        kind = "reference"
        sample = (f"{tok} of the {T} tokens per step" if tok < T else f"the full {T}-token batch") + (
            f", float32, torch intra-op threads = {cores}: the reference's pure-PyTorch "
            "_mhc_pre_map_pytorch + _mhc_post_res_pytorch forward and autograd backward "
            "(baseline/_ref, src/flash_mhc/block.py:82-124)")
        source = "unmodified reference installed in baseline/_ref (pure-PyTorch path on CPU)"
        configs0 = None if args.no_configs0 else _ref_cpu_configs0(ref)
    else:
        tpw = args.cpu_tokens_per_worker
        pool = CpuPool(C, cores)
        try:
            for i in range(args.warmup):
                pool.run(64, 1, seed=10 + i)
            times = [pool.run(tpw, 1, seed=1000 + 97 * i) for i in range(args.steps)]
        finally:
            pool.close()
        tok = cores * tpw
        ms = 1e3 * sum(times) / len(times)
        kind = "port"
        sample = (f"{tok} of the {T} tokens per step ({cores} spawn processes x {tpw}), "
                  "float32 numpy restatement of the reference algorithm (oracle/)")
        source = ("baseline/_ref not installed" if not _reference_installed()
                  else "numpy restatement requested (--ref-kind port)")
        configs0 = None
    value = tok / (ms * 1e-3)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 1), "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) x/lo/grads; the reference's default W_all init)",
        "config": workload_config(T, C, world),
        "cpu_baseline": {"value": round(value, 1), "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample, "source": source},
        "e2e": {"value": round(value, 1), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    if configs0 is not None:
        line["cpu_baseline"]["configs0"] = configs0
    print(json.dumps(line), flush=True)


def cpu_baseline(args):
    """``cpu_baseline`` of the GPU arm (rank 0, N = 1): the reference arm run in
    a child process (this process has imported this repository's flash_mhc,
    whose torch.library namespace the reference's would clash with) on a
    bounded token sample, with the GPU hidden from it."""
    import subprocess

    cmd = [sys.executable, str(Path(__file__).resolve()), "--impl", "reference",
           "--steps", str(args.cpu_reps), "--warmup", "1", "--T", str(args.T), "--C", str(args.C),
           "--ref-tokens", str(args.cpu_ref_tokens),
           "--cpu-tokens-per-worker", str(args.cpu_tokens_per_worker)]
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", RANK="0", WORLD_SIZE="1")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900, cwd=ROOT)
    if r.returncode != 0:
        return {"value": None, "unit": UNIT, "cores": _host_cores(), "kind": "reference",
                "sample": None, "error": (r.stderr or r.stdout)[-500:]}
    cb = json.loads(r.stdout.strip().splitlines()[-1])["cpu_baseline"]
    cb["steps"] = args.cpu_reps
    return cb


def run_reference_triton(args):
    """The reference's own Triton kernels on this GPU (a comparison line).

    Imports the unmodified reference from ``baseline/_ref`` (pip-installed from
    the reference's source tree) instead of this repository's package -- both
    are named ``flash_mhc`` -- and times (1) the same six-op step as
    ``HotPath`` through the reference's ops, K1's weight gradient taken as the
    reference's autograd takes it (``ops.py:683-684``: a bf16 matmul of
    ``go * inv_rms`` with x), and (2) the reference's ``MHCLiteBlock``
    (triton_fused, activation checkpointing) at the block config.  Rank 0 only.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    ref_dir = ROOT / "baseline" / "_ref"
    line = {"impl": "reference-triton", "metric": METRIC, "unit": UNIT}
    if not (ref_dir / "flash_mhc").is_dir():
        line["unavailable"] = "baseline/_ref holds no installed reference package"
        print(json.dumps(line), flush=True)
        return
    sys.path[:] = [p for p in sys.path if Path(p).resolve() not in (ROOT, ROOT / "flash-mhc_b200")]
    sys.path.insert(0, str(ref_dir))
    import torch
    import torch.nn as nn
    import flash_mhc as ref  # the reference package
    if ref_dir.resolve() not in Path(ref.__file__).resolve().parents:
        raise RuntimeError(f"expected the reference from {ref_dir}, got {ref.__file__}")
    ops = torch.ops.flash_mhc
    dev = "cuda"
    T, C, n, D = args.T, args.C, N_STREAMS, D_OUT
    g = torch.Generator(device=dev)
    g.manual_seed(1234)

    def rn(*shape, std=1.0, dt=torch.bfloat16):
        return (torch.randn(*shape, generator=g, device=dev) * std).to(dt)

    x = rn(T, n, C)
    W = rn(D, n * C, std=0.02)
    lo = rn(T, C)
    hp, hq, H = rn(T, n, dt=torch.float32), rn(T, n, dt=torch.float32), rn(T, n, n, dt=torch.float32)
    gp, g3, g4 = rn(T, D), rn(T, C), rn(T, n, C)
    xf = x.reshape(T, n * C)

    def k1_bwd(proj, inv):
        gx = ops.fused_rmsnorm_project_bwd_dx(gp, xf, W, proj, inv)
        gW = torch.matmul((gp * inv[:, None]).to(xf.dtype).t(), xf)
        return gx, gW

    def step(ev=None):
        def rec(k, f):
            if ev is None:
                return f()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            r = f()
            e.record()
            ev.setdefault(k, []).append((s, e))
            return r
        proj, inv = rec("k1_fwd", lambda: ops.fused_rmsnorm_project(xf, W))
        rec("k3_fwd", lambda: ops.fused_pre_map(x, hp))
        rec("k4_fwd", lambda: ops.fused_post_res(x, lo, H, hq))
        rec("k4_bwd", lambda: ops.fused_post_res_backward(g4, x, lo, H, hq))
        rec("k3_bwd", lambda: ops.fused_pre_map_backward(g3, x, hp))
        rec("k1_bwd", lambda: k1_bwd(proj, inv))

    t_tune = time.time()
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    tune_s = time.time() - t_tune
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(_physical_gpu_indices(1)) as clk:
        s.record()
        for _ in range(args.steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / args.steps
        ev = {}
        for _ in range(5):
            step(ev)
        torch.cuda.synchronize()
    kernels = {k: round(sum(a.elapsed_time(b) for a, b in v) / len(v), 4) for k, v in ev.items()}
    line.update({
        "value": round(T / (ms * 1e-3), 1), "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4), "higher_is_better": True,
        "dtype": "bf16", "data": "synthetic (same seeds and distributions as impl ours)",
        "config": {"workload": "kernel-level hot path fwd+bwd (configs[1] shapes)",
                   "T_per_gpu": T, "C": C, "n": n, "D": D},
        "kernels_ms": kernels,
        "clocks": clk.summary(),
        "autotune": os.environ.get("FLASH_MHC_TRITON_AUTOTUNE", "default"),
        "warmup_s_incl_autotune": round(tune_s, 1),
        "source": "unmodified reference installed in baseline/_ref, torch.ops.flash_mhc (Triton)",
    })
    del x, W, lo, hp, hq, H, gp, g3, g4, xf
    if not args.no_block:
        Tb, Cb = args.block_T, args.block_C
        layer = nn.Linear(Cb, Cb, bias=False)
        blk = ref.MHCLiteBlock(n, Cb, layer, triton_fused=True, activation_checkpointing=True)
        blk = blk.to(dev).to(torch.bfloat16).train()
        with torch.no_grad():
            layer.weight.copy_(rn(Cb, Cb, std=0.02))
        xb = rn(Tb, n, Cb).requires_grad_(True)
        up = rn(Tb, n, Cb)

        def bstep():
            blk.zero_grad(set_to_none=True)
            xb.grad = None
            blk(xb).backward(up)

        for _ in range(3):
            bstep()
        torch.cuda.synchronize()
        with ClockSampler(_physical_gpu_indices(1)) as bclk:
            s.record()
            for _ in range(10):
                bstep()
            e.record()
            torch.cuda.synchronize()
        bms = s.elapsed_time(e) / 10
        line["block"] = {"config": {"workload": "MHCLiteBlock fwd+bwd, activation checkpointing "
                                                "(configs[2])", "T_per_gpu": Tb, "C": Cb, "n": n},
                         "value": round(Tb / (bms * 1e-3), 1), "unit": UNIT,
                         "ms_per_step": round(bms, 4), "steps": 10, "clocks": bclk.summary()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-triton"], default="ours",
                    help="reference: the CPU reference arm; reference-triton: the reference's "
                         "own Triton kernels on this GPU from baseline/_ref (comparison line)")
    ap.add_argument("--T", type=int, default=65536, help="tokens per GPU")
    ap.add_argument("--C", type=int, default=1024)
    ap.add_argument("--cpu-tokens-per-worker", type=int, default=1024,
                    help="tokens per spawn process of the numpy fallback")
    ap.add_argument("--cpu-reps", type=int, default=3, help="timed steps of cpu_baseline")
    ap.add_argument("--cpu-ref-tokens", type=int, default=16384,
                    help="tokens per step of the reference code in cpu_baseline")
    ap.add_argument("--ref-tokens", type=int, default=0,
                    help="tokens per step of the reference arm (0: the full per-GPU batch)")
    ap.add_argument("--ref-kind", choices=["reference", "port"], default="reference",
                    help="reference arm: the reference's own code (baseline/_ref) or the numpy port")
    ap.add_argument("--no-configs0", action="store_true",
                    help="reference arm: skip the configs[0] block timing")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-block", action="store_true", help="skip the MHCLiteBlock measurement")
    ap.add_argument("--block-T", type=int, default=65536, help="tokens per GPU for the block")
    ap.add_argument("--block-C", type=int, default=2048)
    ap.add_argument("--no-graphs", action="store_true", help="skip the small-batch graph measurement")
    ap.add_argument("--no-tiny", action="store_true", help="skip the tiny-T inference latency")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the host-buffer e2e leg (its pinned buffers grow with --T/--C)")
    ap.add_argument("--small-T", type=int, default=8192)
    ap.add_argument("--no-large", action="store_true",
                    help="skip the large token-sharded config (configs[3])")
    ap.add_argument("--large-T", type=int, default=131072, help="tokens per GPU, configs[3]")
    ap.add_argument("--large-C", type=int, default=4096)
    ap.add_argument("--launch-lead-ms", type=float, default=20.0,
                    help="GPU sleep before each timed region's start event (0: none)")
    ap.add_argument("--block-allreduce", choices=["bucketed", "after"], default="bucketed",
                    help="with N > 1: BucketedGradReducer, or one bucket after the backward "
                         "(allreduce_gradients)")
    ap.add_argument("--block-reduce-op", choices=["sum", "avg"], default="sum",
                    help="with N > 1: NCCL SUM + scale, or NCCL AVG, for the block's gradients")
    ap.add_argument("--block-buckets", type=int, choices=[1, 2], default=2,
                    help="with N > 1: gradient buckets of the block's all-reduce")
    ap.add_argument("--compute-priority", choices=["high", "default"], default="default",
                    help="with N > 1: the stream priority of the compute stream (NCCL keeps "
                         "the default priority)")
    ap.add_argument("--nccl-max-ctas", type=int, default=0,
                    help="NCCL communicator max_ctas (0: NCCL's default)")
    ap.add_argument("--nccl-cta-policy", type=int, default=-1,
                    help="NCCL communicator cta_policy (-1: NCCL's default)")
    ap.add_argument("--nccl-nvls-ctas", type=int, default=0,
                    help="NCCL communicator nvls_ctas (0: NCCL's default)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        print("note: the timing rules ask for >= 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-triton":
        run_reference_triton(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
