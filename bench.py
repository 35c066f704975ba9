"""Benchmark of the fused attention forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload c4] [--impl ours|reference]

A step is one forward pass of the workload's attention (every shape of the
workload, one kernel launch each).  Default workload: the causal
long-context configuration B=1, H=64, L=16384, D=128, fp16 -- the one the
metric quotes at 1/2/4/8 GPUs -- with the 64 (batch*head) slices sharded
contiguously over the ranks (strong scaling: the total work is fixed, each
rank runs the kernel on its own heads, no collective in the timed region).

Inputs: i.i.d. N(0,1)*scale values drawn slice by slice, one CPU generator per
(tensor, batch, head) seeded from --seed (``workloads.make_qkv``), so a rank
draws exactly the heads it owns, the same values at every N, and the tests
and the parity check below regenerate exactly these inputs.

Timing: W untimed warm-up steps, then K steps, each bracketed by CUDA events
on the launching stream; between timed steps a 256 MiB buffer is rewritten to
flush L2 (outside the events); a barrier and a device synchronise on both
sides of the timed region; the per-rank total is reduced with MAX.

Reported on the line:
  value         whole-job TFLOP/s (algorithmic FLOPs of all ranks / max time)
  e2e           the same metric through the public API for host-resident
                tensors, ``rocm_attn_b200.attn_forward_pinned`` (which calls
                ``attn_forward`` per chunk of heads): H2D of q/k/v, the forward
                and D2H of O, all inside the timed region, overlapped chunk by
                chunk on three streams
  roofline      tensor-bound: TFLOP/s of the kernel launches vs the measured
                dense bf16 GEMM peak; traffic from the committed ncu summary
  parity        max abs error of the timed step's output against the CPU
                oracle (torch SDPA math, fp32) on a subset of heads and rows
  per_config    N = 1: every other benchmark configuration (C1, C2, C3, the C5
                sweep, the UnifoLM preset set) timed the same way, each with
                its parity check and the same-box GPU comparators the
                reference's benchmark offers (torch SDPA per backend, and
                flash_attn_func when importable), run only for their times
  cpu_baseline  rank 0 at N=1: the reference path (torch SDPA as the
                reference's _sdpa_fallback runs it) on the host cores, fp32,
                on a bounded sample of the same workload's heads
  clocks        NVML samples taken during the timed region
  --nvtx        one NVTX range per shape launch, for profiler timelines
  gather        N > 1 only: the NCCL all-gather that assembles the full O
                on every rank, timed on its own after the timed region
``--impl reference`` times that CPU reference path alone on the same
workload (rank 0; other ranks exit without work).  It never imports the
CUDA package: ``workloads.py`` is loaded by path.
"""
from __future__ import annotations

import argparse
import dataclasses
import importlib.util
import json
import os
import statistics
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def _load_workloads():
    """``rocm_attn_b200/workloads.py`` (pure Python: shapes, seeded inputs,
    sharding), loaded by path so that importing it does not run the package's
    ``__init__``, which loads the CUDA extension.  The reference arm thus maps
    none of this repository's native libraries."""
    name = "rocm_attn_bench_workloads"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(REPO, "rocm_attn_b200", "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


W = _load_workloads()
DTYPES, WORKLOADS, Shape, Workload = W.DTYPES, W.WORKLOADS, W.Shape, W.Workload

METRIC = "attention fwd ms/iter and TFLOPS (% of B200 fp16 TC peak) at 1/2/4/8 GPUs"
SPEC_DENSE_FP16_TFLOPS = 2250.0
FALLBACK_HBM_GBS = 6650.0  # earlier measurement on this pool, used without MEASURED_PEAKS.json
MAX_SM_CLOCK_HZ = 1.965e9  # B200 clocks.max.sm, the clock the MUFU fraction is quoted at
FALLBACK_PEAK_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20
L2_NOTE = "a 256 MiB buffer rewritten between timed steps, outside the timed region"
PER_CONFIG = ("c1", "c2", "c3", "c4", "c5", "unifolm")
# The reference benchmark's defaults for its back-to-back loop
# (benchmark/bench_attention.py:162-163).
WARM_ITERS, WARM_WARMUP = 50, 10


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="c4", choices=sorted(WORKLOADS) + ["custom"])
    ap.add_argument("--shapes", default=None,
                    help="custom workload: 'B,H,Lq,D' or 'B,H,Lq,Lk,D' entries separated by ';' "
                         "(the reference benchmark's --shapes syntax); implies --workload custom")
    ap.add_argument("--causal", action="store_true", help="custom workload: causal masking")
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16"], help="custom workload dtype")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample-seconds", type=float, default=12.0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true", help="skip the per-configuration table (N=1)")
    ap.add_argument("--no-parity", action="store_true", help="skip the oracle check of the timed inputs")
    ap.add_argument("--nvtx", action="store_true",
                    help="wrap every shape's launch in an NVTX range named after the shape (for nsys/ncu timelines); "
                         "host-side only, off by default")
    ap.add_argument("--graph", action="store_true",
                    help="capture one step (all shapes of the workload) in a CUDA graph and time its replays: "
                         "removes the per-launch host overhead of small-shape workloads")
    return ap.parse_args(argv)


# ---------------------------------------------------------------- helpers

def measured_peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_PEAK_TFLOPS, FALLBACK_PEAK_TFLOPS, "fallback"


def measured_hbm_gbs():
    """Measured HBM copy bandwidth (GB/s) and whether it was measured."""
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(workload_key: str, rank_heads: int, total_heads: int):
    """DRAM bytes per launch of the attention kernel, from the committed ncu
    summary (profiles/attn_fwd_traffic.txt: '<workload> <heads> <bytes>' lines,
    measured on `heads` slices), scaled to this launch's head count."""
    p = os.path.join(REPO, "profiles", "attn_fwd_traffic.txt")
    try:
        with open(p) as f:
            for line in f:
                parts = line.split()
                if len(parts) == 3 and parts[0] == workload_key:
                    return float(parts[2]) * rank_heads / float(parts[1])
    except OSError:
        pass
    return None


def config_of(w, seed: int) -> dict:
    """The workload as both arms report it (identical dicts)."""
    return {"workload": w.name, "shapes": [dataclasses.asdict(s) for s in w.shapes], "causal": w.causal,
            "input_dtype": w.dtype, "inputs": f"N(0,1)*{w.value_scale:g} per (tensor, batch, head) slice",
            "seed": seed, "l2": L2_NOTE}


class ClockSampler:
    """Samples SM clock, max clock and clock-event (throttle) reasons of one
    GPU every few milliseconds through NVML while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.dev = device_index
        self.period = period_s
        self.samples = []
        self._stop = threading.Event()
        self.max_mhz = None
        self.error = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.dev)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        except Exception as e:  # NVML missing: report no samples rather than fail the bench
            self._nvml = None
            self.error = repr(e)
        return self

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((float(sm), int(reasons)))
            except Exception as e:
                self.error = repr(e)
                return
            time.sleep(self.period)

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._thread.join(timeout=2)
            try:
                self._nvml.nvmlShutdown()
            except Exception:
                pass

    def summary(self):
        reasons = sorted({name for _, r in self.samples for bit, name in self.REASONS.items() if r & bit})
        out = {"sm_mhz": statistics.median([c for c, _ in self.samples]) if self.samples else None,
               "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples), "source": "nvml"}
        if self.error and not self.samples:
            out["error"] = self.error
        return out


def local_shapes(workload, world: int, rank: int):
    """Per-shape (batch*head) range owned by this rank.  Each shape is viewed
    as [1, B*H, L, D]; the slices of a rank are contiguous."""
    return [(s, W.shard_range(s.bh, world, rank)) for s in workload.shapes]


def make_local_inputs(workload, shards, seed, device):
    """q, k, v [1, len(range), L, D] per shape for the rank's (batch*head)
    slices, drawn slice by slice from the seeded CPU generators."""
    dtype = DTYPES[workload.dtype]
    out = []
    for s, r in shards:
        if len(r) == 0:
            out.append(None)
            continue
        out.append(W.make_qkv(s, dtype, seed=seed, value_scale=workload.value_scale, bh_range=r, device=device))
    return out


def check_rows(L: int) -> list:
    """Query rows the parity check covers: the first and the last 128 (the
    longest causal rows), or every row of a short sequence."""
    if L <= 256:
        return list(range(L))
    return list(range(128)) + list(range(L - 128, L))


def parity_of(workload, shards, inputs, outs, causal: bool):
    """Max abs error of ``outs`` against the CPU oracle (torch SDPA math,
    fp32) on the first and last local head of each shape, over
    :func:`check_rows`.  The oracle is the checker here; nothing it computes
    is timed or returned as output."""
    import oracle

    dtype = DTYPES[workload.dtype]
    worst = 0.0
    finite = True
    checked = []
    for (s, r), t, o in zip(shards, inputs, outs):
        if t is None:
            continue
        q, k, v = t
        heads = sorted({0, len(r) - 1})
        rows = check_rows(s.Lq)
        for h in heads:
            ref = oracle.sdpa_rows_fp32(q[:, h:h + 1], k[:, h:h + 1], v[:, h:h + 1], rows, causal=causal)
            got = o[:, h:h + 1, rows].float().cpu()
            finite = finite and bool(torch.isfinite(got).all())
            worst = max(worst, oracle.max_abs_err(got, ref))
        checked.append(f"{len(heads)} heads x {len(rows)} rows of {s.B}x{s.H}x{s.Lq}x{s.Lk}x{s.D}")
    tol = oracle.ATOL[dtype]
    return {"max_abs_err": worst, "tolerance": tol, "finite": finite, "ok": finite and worst <= tol,
            "oracle": "torch SDPA math fp32 on CPU", "checked": "; ".join(checked)}


def time_steps(fn, steps: int, warmup: int, flush, stream):
    """Per-step milliseconds of ``fn`` (CUDA events on ``stream``, L2 flushed
    between steps outside the events)."""
    for _ in range(max(3, warmup)):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        flush.fill_(float(i))
        starts[i].record(stream)
        fn()
        ends[i].record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in zip(starts, ends)]


def time_back_to_back(fn, iters: int, warmup: int, stream):
    """Mean milliseconds per call of ``fn`` run ``iters`` times back to back
    with a warm L2, the way the reference's benchmark times every backend
    (``benchmark/bench_attention.py:47-57``: ``warmup`` calls, then a loop of
    ``iters`` calls between two synchronisations; there by wall clock, here
    by CUDA events on ``stream``)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / iters


# ---------------------------------------------------------------- reference arm

def cpu_reference_sample(workload, seconds: float, seed: int):
    """Times the reference's CPU path (oracle.reference_sdpa_path: the
    reference's _sdpa_fallback restated, fp32, all host threads) on whole
    (batch*head) slices of the workload's seeded inputs until about
    `seconds` have elapsed.  Returns (TFLOP/s, cores, sample description)."""
    import oracle  # CPU reference leg only

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    dtype = DTYPES[workload.dtype]
    flops = 0.0
    t_total = 0.0
    done = []
    for i, s in enumerate(workload.shapes):
        per_head = s.flops(workload.causal) / s.bh
        n = 0
        for f in range(s.bh):
            q, k, v = W.make_qkv(s, dtype, seed=seed, value_scale=workload.value_scale, bh_range=[f])
            q, k, v = (t.float() for t in (q, k, v))
            t0 = time.perf_counter()
            oracle.reference_sdpa_path(q, k, v, causal=workload.causal)
            t_total += time.perf_counter() - t0
            flops += per_head
            n += 1
            if t_total >= seconds * (i + 1) / len(workload.shapes):
                break
        done.append(f"{n}/{s.bh} heads of {s.B}x{s.H}x{s.Lq}x{s.Lk}x{s.D}")
    return flops / t_total / 1e12, cores, "; ".join(done) + f" in {t_total:.1f}s (torch SDPA fp32, CPU)"


def run_reference_arm(args, rank, world):
    w = WORKLOADS[args.workload]
    if rank != 0:
        return None
    per_step = []
    sample = None
    cores = os.cpu_count() or 1
    budget = max(2.0, min(30.0, 120.0 / max(1, args.steps + args.warmup)))
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32)
    for i in range(args.warmup + args.steps):
        flush.fill_(float(i))  # the host caches start cold at every step, as the GPU arm's L2 does
        tf, cores, sample = cpu_reference_sample(w, budget, args.seed)
        if i >= args.warmup:
            per_step.append(tf)
    value = statistics.median(per_step)
    ms = w.flops() / (value * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": config_of(w, args.seed),
        "method": "bounded sample of whole heads per step on the host cores; ms_per_step extrapolated to the "
                  "whole workload",
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample,
                         "what": "the reference's _sdpa_fallback (python/rocm_attn_op/__init__.py:7-26) restated "
                                 "for CPU tensors (oracle.reference_sdpa_path); the reference's own Python package "
                                 "cannot be installed without its HIP extension"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# ---------------------------------------------------------------- our arm

def time_gather(w, shards, step, world, rank, dev, stream, reps: int = 5):
    """Times ``sharding.gather_heads`` (NCCL all_gather_into_tensor of every
    rank's O slices into the full [B, H, Lq, D] O) with CUDA events, max over
    ranks.  Every rank makes the same collective calls in the same order."""
    import torch.distributed as dist
    from rocm_attn_b200.sharding import gather_heads

    outs = iter(step())
    local = []
    for s, r in shards:
        local.append(next(outs) if len(r) > 0 else
                     torch.empty((1, 0, s.Lq, s.D), dtype=DTYPES[w.dtype], device=dev))
    for (s, _), o in zip(shards, local):  # warm-up (communicator set-up)
        gather_heads(o, s.B, s.H, world, rank)
    torch.cuda.synchronize(dev)
    dist.barrier()
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(reps):
        for (s, _), o in zip(shards, local):
            gather_heads(o, s.B, s.H, world, rank)
    g1.record(stream)
    torch.cuda.synchronize(dev)
    t = torch.tensor([g0.elapsed_time(g1) / reps], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    full_bytes = sum(2 * s.bh * s.Lq * s.D for s in w.shapes)
    algbw = full_bytes / (ms * 1e-3) / 1e9
    return {"collective": "NCCL all_gather_into_tensor of O (sharding.gather_heads)", "ms": round(ms, 4),
            "bytes_gathered": int(full_bytes), "algbw_gbs": round(algbw, 1),
            "busbw_gbs": round(algbw * (world - 1) / world, 1), "reps": reps,
            "nccl_version": ".".join(str(x) for x in torch.cuda.nccl.version())}


def comparator_fns(w, inputs):
    """Same-box GPU comparators on the same inputs, as the reference's
    benchmark offers them (benchmark/bench_attention.py:103-145): torch SDPA
    restricted to each backend -- FLASH first is what the reference's wrapper
    runs on a CUDA device (python/rocm_attn_op/__init__.py:7-26) -- SDPA with
    its default choice, and flash_attn_func when the package imports.  They
    are timed only."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    def sdpa(backend):
        def fn():
            for t in inputs:
                if backend is None:
                    F.scaled_dot_product_attention(t[0], t[1], t[2], is_causal=w.causal)
                else:
                    with sdpa_kernel(backend):
                        F.scaled_dot_product_attention(t[0], t[1], t[2], is_causal=w.causal)
        return fn

    fns = {"sdpa_flash": sdpa(SDPBackend.FLASH_ATTENTION), "sdpa_efficient": sdpa(SDPBackend.EFFICIENT_ATTENTION),
           "sdpa_cudnn": sdpa(SDPBackend.CUDNN_ATTENTION), "sdpa_default": sdpa(None)}
    try:
        from flash_attn import flash_attn_func
        blhd = [tuple(x.transpose(1, 2).contiguous() for x in t) for t in inputs]

        def fa():
            for q, k, v in blhd:
                flash_attn_func(q, k, v, causal=w.causal)
        fns["flash_attn_func"] = fa
    except Exception:
        pass
    return fns


def per_config_table(args, dev, stream, flush, headline: dict):
    """Every benchmark configuration on this GPU (N = 1): ours timed like the
    headline, the parity check of its output, and the comparators."""
    import rocm_attn_op

    burst, _, peak_kind = measured_peaks()
    hbm, _ = measured_hbm_gbs()
    table = {}
    for key in PER_CONFIG:
        w = WORKLOADS[key]
        row = {"workload": w.name}
        try:
            shards = local_shapes(w, 1, 0)
            reuse = key == args.workload and headline
            inputs = headline["inputs"] if reuse else make_local_inputs(w, shards, args.seed, dev)
            steps = 20 if w.flops() > 2e11 else 50

            def ours():
                return [rocm_attn_op.attn_forward(t[0], t[1], t[2], causal=w.causal) for t in inputs]

            if reuse:  # the headline's own timing
                ms, min_ms = headline["ms"], headline["min_ms"]
            else:
                samples = time_steps(ours, steps, args.warmup, flush, stream)
                ms, min_ms = statistics.median(samples), min(samples)
            warm_ms = time_back_to_back(ours, WARM_ITERS, WARM_WARMUP, stream)
            tf = w.flops() / (ms * 1e-3) / 1e12
            byts = sum(s.io_bytes() for s in w.shapes)
            row.update({"ms": round(ms, 4), "min_ms": round(min_ms, 4), "warm_ms": round(warm_ms, 4),
                        "warm_tflops": round(w.flops() / (warm_ms * 1e-3) / 1e12, 2),
                        "tflops": round(tf, 2), "frac_of_measured_peak": round(tf / burst, 4),
                        "frac_of_spec_2250": round(tf / SPEC_DENSE_FP16_TFLOPS, 4),
                        "hbm_gbs": round(byts / (ms * 1e-3) / 1e9, 1),
                        "frac_of_measured_hbm": round(byts / (ms * 1e-3) / 1e9 / hbm, 4)})
            # Roofline of the workload shape by shape: each shape bound by
            # the slower of its FLOPs at the measured GEMM peak and its bytes
            # at the measured HBM bandwidth (a mixed list has shapes of both
            # kinds), summed; the fraction is that time over the measured one.
            roof_ms = sum(max(s.flops(w.causal) / (burst * 1e12), s.io_bytes() / (hbm * 1e9)) for s in w.shapes) * 1e3
            row.update({"shape_roofline_ms": round(roof_ms, 4), "frac_of_shape_roofline": round(roof_ms / ms, 4)})
            # Softmax exponentials (one per unmasked score) and, for the
            # tensor-core kernel's share on the MUFU (three quarters; the rest
            # is a polynomial on the FMA pipes), the fraction of the MUFU's
            # 16 ex2 per clock per SM at the maximum SM clock: D=64 is bound
            # by them.
            exps = sum(s.bh * s.unmasked_pairs(w.causal) for s in w.shapes)
            mufu_peak = 16.0 * torch.cuda.get_device_properties(dev).multi_processor_count * MAX_SM_CLOCK_HZ
            row.update({"exp_count": exps, "exp_per_s": round(exps / (ms * 1e-3), 1),
                        "mufu_frac_at_max_clock": round(0.75 * exps / (ms * 1e-3) / mufu_peak, 4)})
            if len(w.shapes) > 1:
                # the same sequence as one call of the batch entry point
                # (grouped tensor-core grids), and both sequences replayed
                # from CUDA graphs; the batch must equal the per-shape calls
                def batched():
                    return rocm_attn_op.attn_forward_batch([t[0] for t in inputs], [t[1] for t in inputs],
                                                           [t[2] for t in inputs], causal=w.causal)

                bms = statistics.median(time_steps(batched, steps, args.warmup, flush, stream))
                a, b = ours(), batched()
                torch.cuda.synchronize()
                row["batch"] = {"ms": round(bms, 4), "tflops": round(w.flops() / (bms * 1e-3) / 1e12, 2),
                                "equal_to_per_shape_calls": all(torch.equal(x, y) for x, y in zip(a, b))}
                del a, b
                for name, fn in (("graph_ms", ours), ("batch_graph_ms", batched)):
                    graph = torch.cuda.CUDAGraph()
                    fn()
                    torch.cuda.synchronize()
                    with torch.cuda.graph(graph):
                        fn()
                    gms = statistics.median(time_steps(graph.replay, steps, args.warmup, flush, stream))
                    row[name] = round(gms, 4)
                    del graph
                row["frac_of_shape_roofline_batch_graph"] = round(roof_ms / row["batch_graph_ms"], 4)
            if reuse and headline.get("parity") is not None:
                row["parity"] = headline["parity"]
            elif not args.no_parity:
                outs = ours()
                torch.cuda.synchronize()
                row["parity"] = parity_of(w, shards, inputs, outs, w.causal)
                del outs
            comps = {}
            for name, fn in comparator_fns(w, inputs).items():
                try:
                    cms = statistics.median(time_steps(fn, steps, args.warmup, flush, stream))
                    cwarm = time_back_to_back(fn, WARM_ITERS, WARM_WARMUP, stream)
                    comps[name] = {"ms": round(cms, 4), "tflops": round(w.flops() / (cms * 1e-3) / 1e12, 2),
                                   "ours_speedup": round(cms / ms, 3), "warm_ms": round(cwarm, 4),
                                   "warm_ours_speedup": round(cwarm / warm_ms, 3)}
                except Exception as e:  # backend not available for this shape or device
                    comps[name] = {"error": str(e).splitlines()[0][:160]}
                torch.cuda.synchronize()
            row["comparators"] = comps
            del inputs
        except Exception as e:
            row["error"] = repr(e)[:300]
        table[key] = row
        torch.cuda.empty_cache()
    return {"peak_kind": f"{peak_kind} bf16 dense GEMM (burst) {burst} TFLOP/s; HBM {hbm} GB/s",
            "timing": f"ms: median of 20 steps (50 for workloads under 0.2 TFLOP), {L2_NOTE}; min_ms: the "
                      f"fastest of those steps; warm_ms: mean of {WARM_ITERS} calls back to back after "
                      f"{WARM_WARMUP} warm-up calls, L2 warm (the reference benchmark's loop)", "rows": table}


def run_ours(args, rank, world, local_rank):
    import rocm_attn_op  # public API (drop-in name)

    w = WORKLOADS[args.workload]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    shards = local_shapes(w, world, rank)
    inputs = make_local_inputs(w, shards, args.seed, dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    dist = torch.distributed if world > 1 else None

    names = [f"attn {s.B}x{s.H}x{s.Lq}x{s.Lk}x{s.D}{' causal' if w.causal else ''} rows {r.start}-{r.stop}"
             for s, r in shards]

    def step():
        outs = []
        for t, name in zip(inputs, names):
            if t is None:
                continue
            if args.nvtx:
                torch.cuda.nvtx.range_push(name)
            outs.append(rocm_attn_op.attn_forward(t[0], t[1], t[2], causal=w.causal))
            if args.nvtx:
                torch.cuda.nvtx.range_pop()
        return outs

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    assert rocm_attn_op.check_status(local_rank) == 0, "kernel watchdog fired during warm-up"
    run = step
    graph = None
    if args.graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize(dev)
        run = graph.replay

    # ---- timed region (device time, per step events, L2 flushed between steps)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev.index) as clk:
        for i in range(args.steps):
            flush.fill_(float(i))
            starts[i].record(stream)
            run()
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
        if dist:
            dist.barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = sum(step_ms)
    t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    rank_ms = None
    if dist:
        every = torch.zeros(world, dtype=torch.float64, device=dev)
        dist.all_gather_into_tensor(every, t)
        rank_ms = [round(float(x) / args.steps, 4) for x in every.cpu()]
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_total_ms = float(t.item())
    ms_per_step = max_total_ms / args.steps
    tflops = w.flops() / (ms_per_step * 1e-3) / 1e12
    assert rocm_attn_op.check_status(local_rank) == 0, "kernel watchdog fired during timing"
    if graph is not None:
        del graph

    # ---- parity of the timed inputs (oracle as checker, outside the timed region)
    parity = None
    if not args.no_parity:
        outs = iter(step())
        local_outs = [next(outs) if t is not None else None for t in inputs]
        torch.cuda.synchronize(dev)
        parity = parity_of(w, shards, inputs, local_outs, w.causal)
        del local_outs, outs

    # ---- roofline of the kernel on this rank (one launch per shape per step)
    local_flops = sum(s.flops(w.causal) * len(r) / s.bh for s, r in shards)
    local_heads = sum(len(r) for _, r in shards)
    kernel_tflops = local_flops / (statistics.mean(step_ms) * 1e-3) / 1e12
    burst, sustained, peak_kind = measured_peaks()
    traffic = profiled_traffic(args.workload, local_heads, sum(s.bh for s in w.shapes)) if len(w.shapes) == 1 \
        else None
    local_bytes = sum(s.io_bytes() * len(r) / s.bh for s, r in shards)
    hbm, hbm_kind = measured_hbm_gbs()
    if local_flops / max(local_bytes, 1.0) >= burst * 1e12 / (hbm * 1e9):
        # arithmetic intensity above the ridge: bound by the tensor cores
        roofline = {"bound": "tensor", "achieved": round(kernel_tflops, 2), "peak": burst, "unit": "TFLOP/s",
                    "frac": round(kernel_tflops / burst, 4), "peak_kind": f"{peak_kind} bf16 dense GEMM (burst)",
                    "frac_of_spec_2250": round(kernel_tflops / SPEC_DENSE_FP16_TFLOPS, 4)}
    else:
        # below the ridge (e.g. the UnifoLM short-sequence set): bound by HBM
        gbs = local_bytes / (statistics.mean(step_ms) * 1e-3) / 1e9
        roofline = {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm, "unit": "GB/s",
                    "frac": round(gbs / hbm, 4), "peak_kind": f"{hbm_kind} HBM copy bandwidth"}
    roofline.update({"traffic": traffic, "algorithmic_bytes": local_bytes,
                     "algorithmic_flops": local_flops})

    # ---- the all-gather that assembles the full O on every rank (N > 1 only;
    # outside the timed region, reported on its own)
    gather = time_gather(w, shards, step, world, rank, dev, stream) if dist else None

    # ---- every benchmark configuration with same-box comparators (N = 1)
    per_config = None
    if world == 1 and not args.no_per_config:
        with ClockSampler(dev.index) as clk_table:
            per_config = per_config_table(args, dev, stream, flush,
                                          {"ms": ms_per_step, "min_ms": min(step_ms), "inputs": inputs,
                                           "parity": parity})
        per_config["clocks"] = clk_table.summary()

    # ---- end to end through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e:
        host_in = []
        h2d = d2h = 0
        for t in inputs:
            if t is None:
                continue
            hq, hk, hv = (x.cpu().pin_memory() for x in t)
            ho = torch.empty(t[0].shape, dtype=t[0].dtype).pin_memory()
            host_in.append((hq, hk, hv, ho))
            h2d += sum(x.numel() * x.element_size() for x in (hq, hk, hv))
            d2h += ho.numel() * ho.element_size()
        del inputs
        torch.cuda.empty_cache()

        import rocm_attn_b200

        def e2e_step():
            # host q/k/v -> device -> attention -> host O, with the two copy
            # directions and the kernel overlapped chunk by chunk
            for hq, hk, hv, ho in host_in:
                rocm_attn_b200.attn_forward_pinned(hq, hk, hv, causal=w.causal, out=ho, device=dev)

        for _ in range(max(3, args.warmup)):  # warm-up: pipeline buffers, streams, host paths
            e2e_step()
        torch.cuda.synchronize(dev)
        n_e2e = max(3, min(args.steps, 10))
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if dist:
            dist.barrier()
        torch.cuda.synchronize(dev)
        ev0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
        e_ms = torch.tensor([ev0.elapsed_time(ev1) / n_e2e], dtype=torch.float64, device=dev)
        if dist:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        e2e = {"value": round(w.flops() / (float(e_ms.item()) * 1e-3) / 1e12, 3), "unit": "TFLOP/s",
               "ms_per_step": round(float(e_ms.item()), 3), "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": int(d2h), "steps": n_e2e,
               "api": "rocm_attn_b200.attn_forward_pinned (host->device, attention and device->host overlapped "
                      "over chunks of heads)"}

    clocks = clk.summary()
    line = {
        "metric": METRIC, "value": round(tflops, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
        "config": config_of(w, args.seed),
        "sharding": "contiguous (batch*head) slices per rank, no collective in the timed region",
        "cuda_graph": bool(args.graph),
        "frac_of_spec_dense_fp16": round(tflops / world / SPEC_DENSE_FP16_TFLOPS, 4),
        "rank_ms_per_step": rank_ms,
        "parity": parity,
        "e2e": e2e,
        "gather": gather,
        "gpu_launches": args.steps * sum(1 for _, r in shards if len(r) > 0),
        "roofline": roofline,
        "clocks": clocks,
        "per_config": per_config,
    }
    return line


def main(argv=None):
    args = parse_args(argv)
    if args.shapes:
        WORKLOADS["custom"] = Workload("custom-" + args.shapes.replace(";", "_") + ("-causal" if args.causal else "")
                                       + "-" + args.dtype, tuple(W.parse_shapes(args.shapes)), args.dtype,
                                       args.causal)
        args.workload = "custom"
    elif args.workload == "custom":
        raise SystemExit("--workload custom needs --shapes")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE", file=sys.stderr)
    dist = None
    if world > 1 and args.impl == "ours":
        import datetime
        torch.cuda.set_device(local_rank)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local_rank))
        dist = torch.distributed
    try:
        if args.impl == "reference":
            line = run_reference_arm(args, rank, world)
        else:
            line = run_ours(args, rank, world, local_rank)
            if rank == 0 and world == 1 and not args.no_cpu_baseline:
                tf, cores, sample = cpu_reference_sample(WORKLOADS[args.workload], args.cpu_sample_seconds,
                                                         args.seed)
                line["cpu_baseline"] = {"value": round(tf, 4), "unit": "TFLOP/s", "cores": cores, "kind": "port",
                                        "sample": sample}
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
