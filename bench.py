#!/usr/bin/env python
"""Attention-forward benchmark (driver contract: one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C4]
                    [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...     (N > 1)

Workload: BASELINE config C4 -- attention forward b=32 s=4096 h=64 d=128
bf16, O + LSE -- the configuration the 1/2/4/8-GPU TFLOPS metric is quoted
on.  The headline is non-causal; the causal variant is timed in the same run
and reported under "variants".  Each rank owns a fixed (batch x head) shard
of that size (32 x 64 independent units), so per-GPU work is fixed as N grows
(weak scaling, no data-path collective; the global batch is 32*N).

  value   whole-job TFLOPS with inputs resident in HBM, device-timed with
          CUDA events, max over ranks.  FLOPs = 4*b*h*s^2*d, halved causal.
  e2e     the same metric through the public API with pinned HOST buffers:
          q/k/v host->device, flash_attn_func, O/LSE device->host, all
          inside the timed region.
  roofline  the kernel's own launch duration (events around each launch on
          its stream) against the measured dense bf16 peak.
  cpu_baseline  fp32 torch math attention on the host cores (the oracle),
          on a bounded sample of (batch, head) slices; N = 1 only.

--impl reference runs the reference's own implementation of this path --
its SM80 kernel, compiled from its sources into oracle/_ref/ -- through its
extension's forward(q, k, v, causal) on the same shards, timed the same way.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(REPO, "flash-attention-cute_b200")
for _p in (REPO, PKG_DIR):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

CONFIGS = {
    "C1": dict(batch=2, seqlen=1024, heads=8, head_dim=64, dtype="float16", causal=False),
    "C2": dict(batch=8, seqlen=2048, heads=16, head_dim=128, dtype="bfloat16", causal=True),
    "C3": dict(batch=16, seqlen=4096, heads=32, head_dim=64, dtype="float16", causal=False),
    "C4": dict(batch=32, seqlen=4096, heads=64, head_dim=128, dtype="bfloat16", causal=False),
    # Long-context causal attention; sharded by zigzag context parallelism
    # (NCCL K/V all-gather) under torchrun, strong scaling.
    "C5": dict(batch=1, seqlen=131072, heads=32, head_dim=128, dtype="bfloat16", causal=True),
    # Profiling case for ncu: C4's per-unit shape with 64 (batch, head) units;
    # q/k/v/o = 256 MiB (> L2) so DRAM counters stay meaningful.
    "C4s": dict(batch=4, seqlen=4096, heads=16, head_dim=128, dtype="bfloat16", causal=False),
}
FALLBACK_PEAK_TFLOPS = 1590.0
THROTTLE_BITS = {
    0x4: "sw_power_cap",
    0x8: "hw_slowdown",
    0x20: "sync_boost",
    0x40: "sw_thermal_slowdown",
    0x80: "hw_thermal_slowdown",
    0x100: "hw_power_brake_slowdown",
}


def flops(b, s, h, d, causal):
    f = 4.0 * b * h * s * s * d
    return f / 2 if causal else f


# ----------------------------------------------------------------- helpers
def load_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["bf16_tflops"]), float(pk.get("bf16_tflops_sustained", 0) or 0), "measured"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, 0.0, "fallback"


def profiled_traffic(config_name, causal):
    """DRAM bytes per launch from the committed ncu summary, if any."""
    path = os.path.join(REPO, "profiles", "traffic_per_launch.txt")
    key = f"{config_name}{'_causal' if causal else ''}"
    try:
        for line in open(path):
            parts = line.split()
            if len(parts) >= 2 and parts[0] == key:
                return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    def __init__(self, device_index, period_s=0.02):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._th = None
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            # Map the CUDA device to its NVML handle by UUID (looking handles
            # up by PCI bus id crashed inside NVML on these hosts).
            h = None
            try:
                want = str(torch.cuda.get_device_properties(device_index).uuid).lower().replace("gpu-", "")
                for i in range(pynvml.nvmlDeviceGetCount()):
                    cand = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(cand)
                    u = (u.decode() if isinstance(u, bytes) else str(u)).lower().replace("gpu-", "")
                    if u == want:
                        h = cand
                        break
            except Exception:
                h = None
            if h is None:
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._h = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
        self.period = period_s

    def _run(self):
        nv = self._nv
        get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or getattr(
            nv, "nvmlDeviceGetCurrentClocksThrottleReasons"
        )
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(get_reasons(self._h))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._h is not None:
            self._th = threading.Thread(target=self._run, daemon=True)
            self._th.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._th is not None:
            self._th.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {
            "sm_mhz": statistics.median(self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": [n for b, n in THROTTLE_BITS.items() if self.reasons & b],
            "samples": len(self.samples),
        }


class Dist:
    def __init__(self, gpus):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if gpus != self.world:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}: launch N>1 through torchrun")
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.pg = None
        if self.world > 1:
            import torch.distributed as dist

            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=self.dev)
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier()

    def max(self, x):
        if self.pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.barrier()
            self.pg.destroy_process_group()


# --------------------------------------------------------------- measurement
def make_shard(cfg, rank, device, seed=0):
    dtype = getattr(torch, cfg["dtype"])
    b, s, h, d = cfg["batch"], cfg["seqlen"], cfg["heads"], cfg["head_dim"]
    g = torch.Generator(device=device).manual_seed(seed + 1000 * rank)
    return [torch.randn((b, s, h, d), generator=g, device=device, dtype=torch.float32).to(dtype) for _ in range(3)]


def fits_in_l2(args) -> bool:
    """True when the step's input tensors together fit in this GPU's L2."""
    size = sum(t.numel() * t.element_size() for t in args if isinstance(t, torch.Tensor))
    return size <= torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size


def l2_note(args) -> str:
    size = sum(t.numel() * t.element_size() for t in args if isinstance(t, torch.Tensor))
    if fits_in_l2(args):
        return (f"inputs ({size / 2**20:.0f} MiB) fit in L2: a buffer of twice the L2 size is written before "
                "every step, outside the event pair that times the step")
    return f"inputs larger than L2 (q/k/v = {size / 2**30:.2f} GiB per step), no flush"


def device_timed(fn, args, steps, warmup, dist_, clocks=None):
    """Returns (ms per step (max over ranks), mean per-launch device ms on
    this rank).

    Inputs larger than L2: the K steps run back to back between one pair of
    events, with nothing else recorded inside (a per-step event costs host time
    that shows at small sizes); the per-launch duration comes from a second,
    separately bracketed pass with an event pair around each launch.
    Inputs that fit in L2: before each step a buffer of twice the L2 size is
    written (evicting the previous step's lines), outside an event pair around
    the step alone; ms per step is the mean of those pairs."""
    for _ in range(warmup):
        fn(*args)
    torch.cuda.synchronize()
    dist_.barrier()
    torch.cuda.synchronize()
    ctx = clocks if clocks is not None else _Null()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    if fits_in_l2(args):
        flush = torch.empty(2 * torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size,
                            dtype=torch.uint8, device="cuda")
        with ctx:
            for e0, e1 in evs:
                flush.fill_(1)
                e0.record()
                fn(*args)
                e1.record()
            torch.cuda.synchronize()
        dist_.barrier()
        per_launch = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
        return dist_.max(per_launch), per_launch
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ctx:
        start.record()
        for _ in range(steps):
            fn(*args)
        end.record()
        torch.cuda.synchronize()
    dist_.barrier()
    torch.cuda.synchronize()
    total = start.elapsed_time(end)
    for e0, e1 in evs:
        e0.record()
        fn(*args)
        e1.record()
    torch.cuda.synchronize()
    dist_.barrier()
    per_launch = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    return dist_.max(total) / steps, per_launch


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def _e2e_step_count(call, min_steps, dist_, target_s=0.25):
    """Steps for a timed region of about target_s, at least min_steps, the
    same on every rank: one more warm call, timed on the host, sets it."""
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    call()
    torch.cuda.synchronize()
    el = dist_.max(time.perf_counter() - t0)
    return max(min_steps, min(1000, int(target_s / max(el, 1e-6))))


def e2e_timed(fn, host_in, dev_in, host_out_fn, min_steps, dist_):
    """Per step: H2D of q/k/v from pinned memory, the call, D2H of outputs.
    Returns (ms per step, steps timed)."""
    qh, kh, vh = host_in
    qd, kd, vd = dev_in

    def step():
        qd.copy_(qh, non_blocking=True)
        kd.copy_(kh, non_blocking=True)
        vd.copy_(vh, non_blocking=True)
        out = fn(qd, kd, vd)
        host_out_fn(out)

    step()
    steps = _e2e_step_count(step, min_steps, dist_)
    torch.cuda.synchronize()
    dist_.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    dist_.barrier()
    return dist_.max(start.elapsed_time(end)) / steps, steps


def e2e_streamed(call, min_steps, dist_):
    """Per step: one blocking host-to-host call (it copies q/k/v in and O/LSE
    out).  Returns (ms per step, steps timed)."""
    call()
    steps = _e2e_step_count(call, min_steps, dist_)
    torch.cuda.synchronize()
    dist_.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        call()
    end.record()
    torch.cuda.synchronize()
    dist_.barrier()
    return dist_.max(start.elapsed_time(end)) / steps, steps


def cpu_baseline(cfg, budget_s=12.0):
    """fp32 math attention (the oracle) on the host cores, on (batch, head)
    slices of the workload until ~budget_s of CPU work has run."""
    from oracle.attention_oracle import make_inputs, math_attention

    s, d, causal = cfg["seqlen"], cfg["head_dim"], cfg["causal"]
    dtype = getattr(torch, cfg["dtype"])
    q, k, v = make_inputs(1, s, 1, d, dtype, seed=99)
    math_attention(q[:, :256], k[:, :256], v[:, :256], causal)  # warm-up
    done, t0 = 0, time.perf_counter()
    while True:
        math_attention(q, k, v, causal)
        done += 1
        el = time.perf_counter() - t0
        if el >= budget_s or done >= 64:
            break
    tf = done * flops(1, s, 1, d, causal) / el / 1e12
    units = cfg["batch"] * cfg["heads"]
    return {
        "value": round(tf, 4),
        "unit": "TFLOPS",
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"{done} of {units} (batch, head) slices (s={s}, d={d}, causal={causal}) in fp32 torch "
        f"math on {torch.get_num_threads()} host threads, {el:.1f} s; throughput extrapolates linearly in slices",
        "ms_per_step_extrapolated": round(el / done * units * 1e3, 1),
    }


def build_fn(impl, cfg, causal):
    if impl == "ours":
        from flash_attention import flash_attn_func

        def fn(q, k, v):
            return flash_attn_func(q, k, v, causal, return_lse=True)

        return fn, "flash_attention (sm_100a tcgen05 kernel) via flash_attn_func, O + LSE"
    from oracle.build_ref import load_module

    ref = load_module()

    def fn(q, k, v):
        return ref.forward(q, k, v, causal)

    return fn, "reference SM80 kernel (its own csrc, compiled for sm_100a) via _C.forward, O only"


def cp_launches(a, b):
    """Kernel launches of rank 0 per C5 step (attention + LSE-merge kernels)."""
    if a.gpus == 1:
        return 1
    if a.cp_schedule == "gather":
        return 2
    world = a.gpus
    pa, pb = 0, 2 * world - 1
    attn = 1 + (1 if pa > 0 else 0) + 2 + (1 if pb > world else 0)
    return attn + 2 * b


def run_context_parallel(a, dist_):
    """C5: every rank builds the same seeded full q/k/v, keeps its zigzag
    shard and runs the context-parallel forward (all-gather of K/V + two
    kernel calls); the whole job is one causal attention over the sequence."""
    from flash_attention import flash_attn_func
    from flash_attention.distributed import context_parallel_attention, zigzag_shard

    cfg = CONFIGS["C5"]
    b, s, h, d = cfg["batch"], cfg["seqlen"], cfg["heads"], cfg["head_dim"]
    q, k, v = make_shard(cfg, 0, dist_.dev)  # identical on every rank
    if dist_.world > 1:
        q, k, v = (zigzag_shard(t, dist_.world, dist_.rank) for t in (q, k, v))

        overlap = a.cp_schedule == "overlap"
        workspace = {}

        def fn(q_, k_, v_):
            return context_parallel_attention(q_, k_, v_, True, overlap=overlap, workspace=workspace)
    else:

        def fn(q_, k_, v_):
            return flash_attn_func(q_, k_, v_, True, return_lse=True)

    fl = flops(b, s, h, d, True)  # whole job
    peak, _, peak_src = load_peaks()
    clocks = ClockSampler(dist_.local) if not a.no_clocks else None
    ms, launch_ms = device_timed(fn, (q, k, v), a.steps, a.warmup, dist_, clocks)
    value = fl / (ms * 1e-3) / 1e12
    if dist_.rank == 0:
        line = {
            "metric": "attn fwd TFLOPS (whole job) & fraction of measured B200 dense bf16 peak",
            "value": round(value, 2),
            "unit": "TFLOPS",
            "n_gpus": a.gpus,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic: i.i.d. N(0,1) q/k/v from a seeded generator (no dataset involved)",
            "config": {
                "workload": f"C5: causal attention b={b} s={s} h={h} d={d} bf16, O + LSE, one sequence over "
                f"{a.gpus} GPU(s)",
                "seq_len": s,
                "parallelism": (
                    "zigzag context parallelism: 2N chunks, NCCL all-gather of K and V, kernel on global positions"
                    + (", gather in two async halves hidden behind local-key compute, fp32 partials LSE-merged"
                       if a.cp_schedule == "overlap" else ", gather then compute")
                )
                if a.gpus > 1
                else "single GPU",
                "l2": l2_note((q, k, v)) + " on each rank",
                "flops_per_step_total": fl,
            },
            "impl": a.impl,
            "roofline": {
                "bound": "tensor",
                "achieved_per_gpu": round(value / a.gpus, 2),
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": round(value / a.gpus / peak, 4),
                "peak_source": f"{peak_src} dense bf16 GEMM (burst)",
            },
            "gpu_launches": a.steps * cp_launches(a, b),
            "clocks": clocks.summary() if clocks is not None else None,
        }
        print(json.dumps(line), flush=True)
    dist_.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="C4", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3, help="minimum e2e steps (more for short steps)")
    ap.add_argument("--no-variants", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-clocks", action="store_true", help="skip NVML clock sampling")
    ap.add_argument("--cp-schedule", default="gather", choices=["overlap", "gather"],
                    help="C5 on N>1 GPUs: gather K/V first (measured faster at N=2), or overlap the gather "
                    "with compute on the local keys and merge fp32 partials")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)

    dist_ = Dist(a.gpus)
    if a.config == "C5":
        if a.impl == "reference":
            if dist_.rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no context-parallel "
                                  "path (single-GPU only); compare C5 at N=1 through --config C5 on one GPU"}))
            dist_.close()
            return
        run_context_parallel(a, dist_)
        return
    cfg = dict(CONFIGS[a.config])
    b, s, h, d = cfg["batch"], cfg["seqlen"], cfg["heads"], cfg["head_dim"]
    ref_available = True
    if a.impl == "reference":
        try:
            build_fn("reference", cfg, False)
        except Exception as e:
            ref_available = False
            ref_error = str(e)
    if a.impl == "reference" and not ref_available:
        # The checker copy of the reference kernel is missing: time the CPU
        # port of its algorithm instead (rank 0 only).
        if dist_.rank == 0:
            cb = cpu_baseline(cfg)
            line = {
                "impl": "reference",
                "metric": "attn fwd TFLOPS (whole job)",
                "value": cb["value"],
                "unit": "TFLOPS",
                "n_gpus": a.gpus,
                "steps": a.steps,
                "warmup": a.warmup,
                "higher_is_better": True,
                "cpu_baseline": cb,
                "e2e": {"value": cb["value"], "unit": "TFLOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "note": f"reference kernel not built ({ref_error}); CPU port of its algorithm timed instead",
            }
            print(json.dumps(line), flush=True)
        dist_.close()
        return

    q, k, v = make_shard(cfg, dist_.rank, dist_.dev)
    fl = flops(b, s, h, d, cfg["causal"])
    peak, peak_sustained, peak_src = load_peaks()

    fn, desc = build_fn(a.impl, cfg, cfg["causal"])
    clocks = ClockSampler(dist_.local) if not a.no_clocks else None
    ms, launch_ms = device_timed(fn, (q, k, v), a.steps, a.warmup, dist_, clocks)
    l2_of_step = l2_note((q, k, v))
    value = fl * a.gpus / (ms * 1e-3) / 1e12
    achieved = fl / (launch_ms * 1e-3) / 1e12

    variants = {}
    if not a.no_variants and a.config in ("C3", "C4", "C4s"):
        fn_c, _ = build_fn(a.impl, cfg, True)
        ms_c, launch_c = device_timed(fn_c, (q, k, v), a.steps, a.warmup, dist_)
        fl_c = flops(b, s, h, d, True)
        variants[f"{a.config}_causal"] = {
            "value": round(fl_c * a.gpus / (ms_c * 1e-3) / 1e12, 2),
            "unit": "TFLOPS",
            "ms_per_step": round(ms_c, 4),
            "roofline_frac": round(fl_c / (launch_c * 1e-3) / 1e12 / peak, 4),
        }

    if not a.no_variants and a.impl == "ours" and a.config in ("C2", "C3", "C4", "C4s"):
        # the backward pass (no counterpart in the reference): FLOPs counted
        # as 2.5x the forward's, the usual convention (5 GEMMs against 2)
        from flash_attention._C import forward_with_lse
        from flash_attention.backward import flash_attn_backward

        for causal_b in sorted({cfg["causal"], True}):
            o_b, lse_b = forward_with_lse(q, k, v, causal_b)
            do_b = torch.randn_like(q)
            ms_b, _ = device_timed(lambda q_, k_, v_: flash_attn_backward(do_b, q_, k_, v_, o_b, lse_b, causal_b),
                                   (q, k, v), max(3, a.steps // 4), a.warmup, dist_)
            fl_b = 2.5 * flops(b, s, h, d, causal_b)
            variants[f"{a.config}_backward{'_causal' if causal_b else ''}"] = {
                "value": round(fl_b * a.gpus / (ms_b * 1e-3) / 1e12, 2),
                "unit": "TFLOPS (2.5x forward FLOPs)",
                "ms_per_step": round(ms_b, 4),
            }
            del o_b, lse_b, do_b

    # e2e through the public call with host buffers.
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty_like(qh).pin_memory()
    lseh = torch.empty((b, h, s), dtype=torch.float32).pin_memory()
    qd, kd, vd = (torch.empty_like(t) for t in (q, k, v))
    del q, k, v

    def host_out(out):
        if isinstance(out, tuple):
            oh.copy_(out[0], non_blocking=True)
            lseh.copy_(out[1], non_blocking=True)
        else:
            oh.copy_(out, non_blocking=True)

    if a.impl == "ours":
        # the library's public call for host-resident tensors: batch chunks
        # stream through the GPU with H2D, kernel and D2H overlapped
        from flash_attention import flash_attn_func_host

        del qd, kd, vd
        ms_e2e, e2e_steps = e2e_streamed(lambda: flash_attn_func_host(qh, kh, vh, cfg["causal"], out=oh, lse_out=lseh),
                              a.e2e_steps, dist_)
        e2e_how = ("pinned host q/k/v -> flash_attn_func_host -> pinned host O + LSE: batch chunks stream through "
                   "the GPU, H2D / kernel / D2H of different chunks overlapped on three streams")
    else:
        ms_e2e, e2e_steps = e2e_timed(fn, (qh, kh, vh), (qd, kd, vd), host_out, a.e2e_steps, dist_)
        e2e_how = "pinned host q/k/v -> device, the public call, O (+LSE) -> pinned host; one stream"
    h2d = 3 * qh.numel() * qh.element_size()
    d2h = oh.numel() * oh.element_size() + (lseh.numel() * 4 if a.impl == "ours" else 0)
    e2e_value = fl * a.gpus / (ms_e2e * 1e-3) / 1e12

    cpu = None
    if dist_.rank == 0 and a.gpus == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(cfg)
        if a.impl == "reference":
            cpu = dict(cpu)

    if dist_.rank == 0:
        traffic = profiled_traffic(a.config, cfg["causal"]) if a.impl == "ours" else None
        line = {
            "metric": "attn fwd TFLOPS (whole job) & fraction of measured B200 dense bf16 peak",
            "value": round(value, 2),
            "unit": "TFLOPS",
            "n_gpus": a.gpus,
            "steps": a.steps,
            "warmup": a.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16" if cfg["dtype"] == "bfloat16" else "fp16",
            "data": "synthetic: i.i.d. N(0,1) q/k/v from a seeded generator (no dataset involved)",
            "config": {
                "workload": f"{a.config}: attention forward b={b} s={s} h={h} d={d} {cfg['dtype']} "
                f"{'causal' if cfg['causal'] else 'non-causal'}, O + LSE, per GPU",
                "batch_per_gpu": b,
                "global_batch": b * a.gpus,
                "seq_len": s,
                "heads": h,
                "head_dim": d,
                "causal": cfg["causal"],
                "parallelism": f"batch x head sharding over {a.gpus} GPU(s), no collective",
                "l2": l2_of_step,
                "flops_per_step_per_gpu": fl,
            },
            "impl": a.impl,
            "path": desc,
            "roofline": {
                "bound": "tensor",
                "achieved": round(achieved, 2),
                "peak": peak,
                "unit": "TFLOP/s",
                "frac": round(achieved / peak, 4),
                "peak_source": f"{peak_src} dense bf16 GEMM (burst)" + ("" if peak_src == "measured" else ", fallback"),
                "frac_of_sustained_peak": round(achieved / peak_sustained, 4) if peak_sustained else None,
                "traffic": traffic,
                "launch_ms": round(launch_ms, 4),
                "algorithmic_flops_per_launch": fl,
            },
            "e2e": {
                "value": round(e2e_value, 2),
                "unit": "TFLOPS",
                "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "ms_per_step": round(ms_e2e, 3),
                "steps": e2e_steps,
                "how": e2e_how,
            },
            "gpu_launches": a.steps if a.impl == "ours" else 0,
            "clocks": clocks.summary() if clocks is not None else None,
            "variants": variants,
            "cpu_baseline": cpu,
        }
        if a.impl == "reference":
            line["gpu_launches"] = 0
            line["reference_kernel_launches"] = a.steps
            line["cpu_baseline"] = {
                "value": round(value, 2),
                "unit": "TFLOPS",
                "cores": 1,
                "kind": "reference",
                "sample": "the full workload on the GPU: the reference's implementation of this path is a "
                "CUDA kernel (no CPU path exists); one host thread launches it",
            }
            if cpu is not None:
                line["cpu_fp32_math"] = cpu
        print(json.dumps(line), flush=True)
    dist_.close()


if __name__ == "__main__":
    main()
