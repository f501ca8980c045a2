#!/usr/bin/env python
"""Benchmark of the fused Cayley + quaternion selective scan (forward) on B200.

Workload (config 3 of the hot path): per GPU batch=4, seq_len=2048, d_inner=1536,
d_state=64; x ~ N(0,1) [4,2048,1536] is the real part of S; delta =
softplus(N(-3,1)); Lambda: Re = -exp(U(ln 1e-3, ln 1e-1)), Im ~ N(0, 0.5);
B_t, C_t shared by all channels [4,2048,64,4] ~ N(0,1)/8; D = 1. fp32 by default
(``--dtype bf16`` for bf16 inputs, state always fp32; ``--layout perchannel`` for
the reference block's per-channel B/C [4,2048,1536,64,4]).

One step = one fused scan launch over the whole batch (inputs resident in HBM).
With N GPUs (torchrun, one process per GPU) every rank scans its own batch of 4
(weak scaling over batch, no collective on the data path); the step time is the
max over ranks. Prints one JSON line (rank 0).

``--impl reference`` times the reference's sequential PyTorch CPU path (restated
in ``oracle/``) on the host cores instead, on a bounded time-prefix of the same
workload per step.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

BATCH, SEQ, CHANNELS, STATE = 4, 2048, 1536, 64
METRIC = "quaternion SSM scan forward tokens/s (config 3: B=4/GPU, T=2048, D=1536, N=64)"
# algorithmic FLOPs per (b, t, d, n) element of the fused forward with a real
# signal: Cayley from (delta, Lambda) 15, q (x) h 28, x*B 4, + 4, C (x) h 28, sum over n 4
FLOPS_PER_ELEM_SREAL = 83
FLOPS_PER_ELEM_SQUAT = 83 - 4 + 28  # B (x) S instead of x*B


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--dtype", choices=["fp32", "bf16"], default="fp32")
    ap.add_argument("--layout", choices=["shared", "perchannel"], default="shared")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-budget-s", type=float, default=15.0,
                    help="seconds of CPU work for the cpu_baseline sample")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the forward+backward and per-channel-layout sub-measurements")
    ap.add_argument("--only", choices=["fwd", "fwd_bwd", "perchannel", "perchannel_fwd_bwd"],
                    default=None,
                    help="run only this sub-measurement and print it (profiling aid)")
    ap.add_argument("--prof-batch", type=int, default=None,
                    help="--only perchannel_fwd_bwd: batch rows (a small case for profilers)")
    ap.add_argument("--prof-seq", type=int, default=None,
                    help="--only perchannel_fwd_bwd: sequence length (a small case for profilers)")
    ap.add_argument("--prof-channels", type=int, default=None,
                    help="--workload fused_parts: scan channels of the projections (a small "
                         "case for profilers)")
    ap.add_argument("--segments", type=int, default=4,
                    help="config5 on >1 GPU: time segments whose all-gather overlaps the "
                         "scan of the next segment")
    ap.add_argument("--decode-batch", type=int, default=4,
                    help="decode workload: sequences decoded together per GPU")
    ap.add_argument("--gather", choices=["peer", "nccl", "multicast"], default="peer",
                    help="config5 on >1 GPU: how y is assembled on every rank (multicast: "
                         "NVLink SHARP multimem stores, where the platform has them)")
    ap.add_argument("--shard", choices=["channel", "time"], default="channel",
                    help="config5 on >1 GPU: channel shards with y all-gathered, or time "
                         "shards exchanging range summaries (y then all-gathered too)")
    ap.add_argument("--workload", choices=["config3", "config5", "config2", "decode", "block_glue",
                                           "config4_block", "fused_parts"],
                    default="config3",
                    help="config5: B=1, T=65536, D=1536, N=64, bf16, channel-sharded over the "
                         "GPUs with an NCCL all-gather of y (strong scaling)")
    return ap.parse_args()


# ----------------------------------------------------------------- plumbing

def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if (args.impl == "b200" and torch.cuda.is_available()) else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        kw = {"device_id": torch.device(f"cuda:{local}")} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300), **kw)
    return world, rank, local


def barrier(world):
    if world > 1:
        dist.barrier()


def make_inputs(dev, dtype, layout, seed, batch=None, seq=None):
    """Config-3 inputs (batch/seq override the config's 4 x 2048, for the small
    cases that profiler captures use)."""
    BATCH_, SEQ_ = batch or BATCH, seq or SEQ
    g = torch.Generator(device=dev).manual_seed(seed)
    f32 = torch.float32
    x = torch.randn(BATCH_, SEQ_, CHANNELS, generator=g, device=dev, dtype=f32)
    delta = torch.nn.functional.softplus(
        torch.randn(BATCH_, SEQ_, CHANNELS, generator=g, device=dev, dtype=f32) - 3.0)
    lam = torch.empty(CHANNELS, STATE, 4, device=dev, dtype=f32)
    u = torch.rand(CHANNELS, STATE, generator=g, device=dev, dtype=f32)
    lam[..., 0] = -torch.exp(u * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    lam[..., 1:] = 0.5 * torch.randn(CHANNELS, STATE, 3, generator=g, device=dev, dtype=f32)
    bc_shape = (BATCH_, SEQ_, STATE, 4) if layout == "shared" else (BATCH_, SEQ_, CHANNELS, STATE, 4)
    Bm = torch.randn(*bc_shape, generator=g, device=dev, dtype=f32) / math.sqrt(STATE)
    Cm = torch.randn(*bc_shape, generator=g, device=dev, dtype=f32) / math.sqrt(STATE)
    Dk = torch.ones(CHANNELS, device=dev, dtype=f32)
    cast = torch.bfloat16 if dtype == "bf16" else f32
    return dict(delta=delta.to(cast), Lambda=lam, B=Bm.to(cast), C=Cm.to(cast), x=x.to(cast), D=Dk)


def algorithmic_bytes(inp, y_bytes):
    return sum(t.numel() * t.element_size() for t in inp.values()) + y_bytes


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
              "timestamp")

    def __init__(self, dev):
        self.proc = None
        self.path = None
        try:
            self.uuid = str(torch.cuda.get_device_properties(dev).uuid)
        except Exception:
            self.uuid = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="mqc_clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            # let the sampler start up before the timed region begins
            t_end = time.time() + 3.0
            while time.time() < t_end and Path(self.path).stat().st_size == 0:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        self.window = [time.time(), None]

    def mark_end(self):
        """End of the timed region (samples after it are not counted)."""
        self.window[1] = time.time()

    def stop(self):
        if self.proc is None:
            return None
        if self.window[1] is None:
            self.mark_end()
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            if self.uuid and self.uuid.replace("GPU-", "") not in parts[1]:
                continue
            rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        # keep the samples taken between the start of the warm-up and the end of
        # the timed region (all of them if the timestamps cannot be read)
        inside = []
        for r in rows:
            try:
                ts = datetime.datetime.strptime(r[10], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except (IndexError, ValueError):
                inside = rows
                break
            if self.window[0] - 0.05 <= ts <= self.window[1] + 0.05:
                inside.append(r)
        rows = inside or rows

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None

        sm = [num(r[2]) for r in rows if num(r[2]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[6:10]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(rows[0][3]), "samples": len(rows),
                "reasons": sorted(reasons)}


def timed(fn, steps, warmup, world, stream):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    return e0.elapsed_time(e1)


def max_over_ranks(val, world, dev):
    if world == 1:
        return val
    t = torch.tensor([val], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def fp32_peak_tflops(dev):
    """FP32 FMA peak measured now (same clocks as the timed region)."""
    import ctypes

    from mambaqc_b200 import _lib
    out = torch.zeros(1, device=dev)
    n = ctypes.c_int64(0)
    stream = torch.cuda.current_stream(dev)
    iters = 4096
    for _ in range(2):
        _lib.call("mqc_probe_fp32_fma", out.data_ptr(), iters, ctypes.byref(n), stream.cuda_stream)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    e0.record(stream)
    for _ in range(reps):
        _lib.call("mqc_probe_fp32_fma", out.data_ptr(), iters, ctypes.byref(n), stream.cuda_stream)
    e1.record(stream)
    torch.cuda.synchronize()
    sec = e0.elapsed_time(e1) / 1e3 / reps
    return 2.0 * n.value / sec / 1e12


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ----------------------------------------------------------- CPU reference leg

def cpu_reference_sample(budget_s, dtype_name, layout, seed=0):
    """The reference's sequential fp32 PyTorch path (oracle restatement) on a
    time-prefix of the config-3 workload; returns (tokens/s, sample description, threads)."""
    from oracle import ref
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    slab = 8
    lam = torch.empty(CHANNELS, STATE, 4)
    lam[..., 0] = -torch.exp(torch.empty(CHANNELS, STATE).uniform_(math.log(1e-3), math.log(1e-1),
                                                                   generator=g))
    lam[..., 1:] = 0.5 * torch.randn(CHANNELS, STATE, 3, generator=g)
    Dk = torch.ones(CHANNELS)
    h = None
    steps = 0
    t_start = time.perf_counter()
    while steps < SEQ:
        x = torch.randn(BATCH, slab, CHANNELS, generator=g)
        delta = torch.nn.functional.softplus(torch.randn(BATCH, slab, CHANNELS, generator=g) - 3.0)
        shape = (BATCH, slab, STATE, 4) if layout == "shared" else (BATCH, slab, CHANNELS, STATE, 4)
        Bm = torch.randn(*shape, generator=g) / 8
        Cm = torch.randn(*shape, generator=g) / 8
        _, h = ref.ssm_scan_cayley(delta, lam, Bm, Cm, x, Dk, h0=h, t_slab=slab)
        steps += slab
        if time.perf_counter() - t_start > budget_s:
            break
    elapsed = time.perf_counter() - t_start
    sample = (f"first {steps} of {SEQ} timesteps of config 3 (B={BATCH}, D={CHANNELS}, "
              f"N={STATE}, {layout} B/C, fp32), Cayley + sequential recurrence")
    return BATCH * steps / elapsed, sample, threads, steps, elapsed


# ----------------------------------------------------------------- main legs

def config3_dict(world, layout):
    """The `config` object of the config-3 line; both arms print this same dict."""
    return {"workload": "config3_fused_scan_forward", "batch_per_gpu": BATCH,
            "global_batch": BATCH * world, "seq_len": SEQ, "d_inner": CHANNELS,
            "d_state": STATE, "layout": layout, "signal": "real x",
            "parallelism": f"dp{world} (batch shards, no data-path collective)",
            "l2": "inputs larger than L2 (310+ MB per step)"}


def run_reference(args, world, rank):
    """The reference arm: the reference's sequential fp32 PyTorch CPU path (the
    oracle restatement) on the host cores. Each step is a bounded time-prefix of
    the config-3 workload; `ms_per_step` is the wall time actually spent per
    timed step and `value` the tokens of the timed steps over that time."""
    if rank != 0:
        return 0
    per_step_budget = min(args.cpu_budget_s, max(0.5, 150.0 / max(1, args.steps + args.warmup)))
    tokens = 0
    seconds = 0.0
    info = None
    for i in range(args.warmup + args.steps):
        v, sample, threads, steps, elapsed = cpu_reference_sample(per_step_budget, args.dtype,
                                                                 args.layout, seed=i)
        if i >= args.warmup:
            tokens += BATCH * steps
            seconds += elapsed
            info = (sample, threads, steps)
    value = tokens / seconds
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * seconds / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.dtype == "fp32" else "bf16 inputs, f32 state",
        "data": "synthetic (seeded, config-3 distributions)",
        "config": config3_dict(world, args.layout),
        "timed": {"seconds": seconds, "tokens": tokens,
                  "tokens_per_step": tokens / args.steps,
                  "note": "each step scans a time-prefix of the config-3 batch for a bounded "
                          "wall time; ms_per_step is that measured time"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": info[1], "kind": "port",
                         "sample": f"{info[0]}; last timed step: {info[2]} timesteps"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# DRAM bytes (read + write) of one launch of the dominant kernel, taken from the
# ncu capture summarised in profiles/scan_fwd_packed_config3.md
# (dram__bytes_read.sum + dram__bytes_write.sum), keyed by (dtype, layout). This
# run does not measure it (no profiler runs inside the bench); None where no
# capture exists.
NCU_TRAFFIC_BYTES = {("fp32", "shared"): 119.57e6 + 151.86e6}
NCU_TRAFFIC_SOURCE = ("ncu capture of the same kernel and workload, summarised in "
                      "profiles/scan_fwd_packed_config3.md; not measured by this run")


def launches_per_scan(dtype: str) -> int:
    """Kernels one channel-shared fused scan call launches: the B/C pre-pass and
    the scan, plus the bf16 -> fp32 widening of delta and x for bf16 inputs."""
    return 2 if dtype == "fp32" else 4


def run_b200(args, world, rank, local):
    from mambaqc_b200 import _lib
    from mambaqc_b200.kernels import ssm_scan_cayley

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if args.only is not None:
        stream = torch.cuda.current_stream(dev)
        if args.only == "fwd":
            inp = make_inputs(dev, args.dtype, args.layout, seed=1234 + rank)
            ms = timed(lambda: ssm_scan_cayley(inp["delta"], inp["Lambda"], inp["B"], inp["C"],
                                               inp["x"], inp["D"]),
                       args.steps, args.warmup, world, stream)
            _lib.check_device_status(dev)
            res = {"ms_per_step": max_over_ranks(ms / args.steps, world, dev)}
        elif args.only == "fwd_bwd":
            inp = make_inputs(dev, args.dtype, args.layout, seed=1234 + rank)
            res = run_fwd_bwd(args, inp, dev, world, stream, ssm_scan_cayley)
        elif args.only == "perchannel_fwd_bwd":
            res = run_perchannel_fwd_bwd(args, dev, world, stream, ssm_scan_cayley,
                                         measured_peaks()[0], args.dtype, args.prof_batch,
                                         args.prof_seq)
        else:
            res = run_perchannel(args, dev, world, stream, ssm_scan_cayley, measured_peaks()[0])
        if rank == 0:
            print(json.dumps({"only": args.only, **res}), flush=True)
        return 0
    inp = make_inputs(dev, args.dtype, args.layout, seed=1234 + rank)
    stream = torch.cuda.current_stream(dev)
    out = {}

    def step():
        out["y"] = ssm_scan_cayley(inp["delta"], inp["Lambda"], inp["B"], inp["C"], inp["x"],
                                   inp["D"])

    step()
    torch.cuda.synchronize()
    _lib.check_device_status(dev)
    y_bytes = out["y"].numel() * out["y"].element_size()

    clocks = ClockSampler(dev)
    clocks.start()
    ms_total = timed(step, args.steps, args.warmup, world, stream)
    clocks.mark_end()
    clk = clocks.stop()
    _lib.check_device_status(dev)
    ms_step_local = ms_total / args.steps
    ms_step = max_over_ranks(ms_step_local, world, dev)
    tokens = BATCH * SEQ * world
    value = tokens / (ms_step / 1e3)

    # roofline of the dominant kernel (the packed scan; the step also runs the small
    # B/C pre-pass, and for bf16 inputs the widening of delta and x, which the
    # achieved figures include): FP32 bound, with the HBM view beside it
    elems = BATCH * SEQ * CHANNELS * STATE
    flops = elems * FLOPS_PER_ELEM_SREAL
    abytes = algorithmic_bytes(inp, y_bytes)
    sec = ms_step_local / 1e3
    peaks, peak_kind = measured_peaks()
    fp32_peak = fp32_peak_tflops(dev)
    roofline = {"bound": "fp32", "achieved": flops / sec / 1e12, "peak": fp32_peak,
                "unit": "TFLOP/s", "frac": flops / sec / 1e12 / fp32_peak,
                "peak_source": "FP32 FMA probe (mqc_probe_fp32_fma) run by bench.py, same clocks",
                "algorithmic_flops_per_launch": flops,
                "traffic": NCU_TRAFFIC_BYTES.get((args.dtype, args.layout)),
                "traffic_source": NCU_TRAFFIC_SOURCE}
    roofline_hbm = {"bound": "hbm", "achieved": abytes / sec / 1e9, "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "frac": abytes / sec / 1e9 / peaks["hbm_gbs"],
                    "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                    "algorithmic_bytes_per_launch": abytes,
                    "traffic": NCU_TRAFFIC_BYTES.get((args.dtype, args.layout)),
                    "traffic_source": NCU_TRAFFIC_SOURCE}

    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, inp, dev, world, stream, ssm_scan_cayley)

    extras = {}
    # the work the hot path shards over GPUs, measured at every N: config 3 as one
    # 8192-token problem split over the ranks, and config 5 with its y exchange
    if args.layout == "shared":
        del inp, out
        torch.cuda.empty_cache()
        extras["config3_strong"] = config3_strong_measure(args, world, rank, local)
        extras["config5"] = config5_measure(args, world, rank, local, gather=args.gather)
        torch.cuda.empty_cache()
        inp = make_inputs(dev, args.dtype, args.layout, seed=1234 + rank)
        out = {}
    if not args.no_extras:
        extras["fwd_bwd"] = run_fwd_bwd(args, inp, dev, world, stream, ssm_scan_cayley)
        if args.layout == "shared":
            del inp, out
            torch.cuda.empty_cache()
            extras["perchannel_fwd"] = run_perchannel(args, dev, world, stream, ssm_scan_cayley,
                                                      peaks)
            extras["perchannel_fwd_bwd"] = run_perchannel_fwd_bwd(
                args, dev, world, stream, ssm_scan_cayley, peaks, "bf16")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, sample, threads, steps, elapsed = cpu_reference_sample(args.cpu_budget_s, args.dtype,
                                                                 args.layout)
        cpu = {"value": v, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{sample}; {elapsed:.1f} s on {threads} threads"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32" if args.dtype == "fp32" else "bf16 inputs, f32 state",
            "data": "synthetic (seeded, config-3 distributions)",
            "config": config3_dict(world, args.layout),
            "roofline": roofline, "roofline_hbm": roofline_hbm,
            "gpu_launches": args.steps * launches_per_scan(args.dtype), "clocks": clk,
            "e2e": e2e, "cpu_baseline": cpu,
            **extras,
        }
        print(json.dumps(line), flush=True)
    return 0


def run_e2e(args, inp, dev, world, stream, op):
    """Same metric through the public API with host buffers: every step hands the
    inputs in pinned host memory to ``ssm_scan_cayley_from_host`` and gets y back
    in pinned host memory -- all host<->device copies inside the timed region
    (pipelined over time segments by the API)."""
    from mambaqc_b200.kernels.ssm_fused import _host_segments
    from mambaqc_b200.kernels import ssm_scan_cayley_from_host

    host = {k: v.cpu().pin_memory() for k, v in inp.items()}
    y_host = torch.empty(BATCH, SEQ, CHANNELS, 4, dtype=inp["delta"].dtype).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = y_host.numel() * y_host.element_size()
    bufs = {}

    def step():
        ssm_scan_cayley_from_host(host["delta"], host["Lambda"], host["B"], host["C"],
                                  host["x"], host["D"], device=dev, out=y_host, _bufs=bufs)

    steps = max(3, min(args.steps, 10))
    ms = timed(step, steps, max(3, min(args.warmup, 3)), world, stream) / steps
    ms = max_over_ranks(ms, world, dev)
    return {"value": BATCH * SEQ * world / (ms / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms,
            "steps": steps,
            "gpu_launches_per_step": _host_segments(SEQ) * launches_per_scan(args.dtype),
            "path": "mambaqc_b200.kernels.ssm_scan_cayley_from_host: pinned host inputs -> "
                    "device (copy stream), fused scan per time segment of the whole batch "
                    f"({_host_segments(SEQ)} segments chained through the final state), "
                    "y -> pinned host (third stream)"}


# Algorithmic FLOPs per (b, t, d, n) element of the scan backward with a real
# signal: lambda = conj(C) (x) dy + carry 32, carry = conj(q) (x) lambda 28,
# dq = lambda (x) conj(h_prev) 28, the Cayley map 15 and its vector-Jacobian
# product 42, ddelta <dz, Lambda> 7, dLambda += delta dz 8, dB = x lambda 4,
# dx <B, lambda> 7, dC = dy (x) conj(h) 28. The recomputation of the states
# from the forward's checkpoints (36 more) is not counted.
BWD_FLOPS_PER_ELEM_SREAL = 199


def run_fwd_bwd(args, inp, dev, world, stream, op):
    """Forward + backward of the fused scan (config 3 names both): one step = the
    forward with checkpoints plus the backward for a fixed upstream gradient.
    The backward alone is timed with CUDA events around the autograd backward and
    reported against the FP32 FMA peak (channel-shared B/C: FP32-bound)."""
    leaves = {k: (v.detach().requires_grad_() if k != "D" else v) for k, v in inp.items()}
    gy = torch.randn(BATCH, SEQ, CHANNELS, 4, device=dev, dtype=inp["delta"].dtype)
    bwd = []

    def step():
        for v in leaves.values():
            v.grad = None
        y = op(leaves["delta"], leaves["Lambda"], leaves["B"], leaves["C"], leaves["x"],
               leaves["D"])
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        y.backward(gy)
        e1.record(stream)
        bwd.append((e0, e1))

    steps = max(3, min(args.steps, 10))
    ms = timed(step, steps, max(3, min(args.warmup, 3)), world, stream) / steps
    torch.cuda.synchronize()
    ms_bwd = sum(a.elapsed_time(b) for a, b in bwd[-steps:]) / steps
    ms = max_over_ranks(ms, world, dev)
    ms_bwd = max_over_ranks(ms_bwd, world, dev)
    flops = BATCH * SEQ * CHANNELS * STATE * BWD_FLOPS_PER_ELEM_SREAL
    peak = fp32_peak_tflops(dev)
    # kernels per step: scan forward, scan backward, plus torch's zero-fill of the
    # shared dB/dC accumulators, the casts and the sums over batch
    return {"value": BATCH * SEQ * world / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "backward_ms": ms_bwd, "steps": steps,
            "what": "scan forward (with checkpoints) + backward, "
                    + ("fp32" if inp["delta"].dtype == torch.float32 else "bf16 inputs"),
            "roofline": {"bound": "fp32", "kernel": "ssm_scan_bwd_packed_kernel (the backward)",
                         "achieved": flops / (ms_bwd / 1e3) / 1e12, "peak": peak,
                         "unit": "TFLOP/s", "frac": flops / (ms_bwd / 1e3) / 1e12 / peak,
                         "algorithmic_flops_per_launch": flops,
                         "flops_per_element": BWD_FLOPS_PER_ELEM_SREAL,
                         "peak_source": "FP32 FMA probe run by bench.py"}}


def perchannel_bwd_bytes(inp):
    """Algorithmic bytes of one per-channel scan backward: B, C, delta, x and dy
    read once; dB, dC, ddelta, dx written once; Lambda read and its per-batch
    partials written once. The forward's state checkpoints, which the backward
    also reads, are an artefact of recomputation and are not counted."""
    es = inp["B"].element_size()
    bc = inp["B"].numel() * es
    per_tc = inp["delta"].numel() * inp["delta"].element_size()
    lam = inp["Lambda"].numel() * 4
    return 4 * bc + 2 * per_tc + 2 * per_tc + per_tc * 4 + lam + BATCH * lam


def run_perchannel_fwd_bwd(args, dev, world, stream, op, peaks, dtype_name, batch=None,
                           seq=None):
    """Forward (with the backward's state checkpoints) + backward of the scan in
    the reference block's per-channel B/C layout [4,2048,1536,64,4], the config-4
    training case. HBM-bound: B, C, dB and dC each cross HBM once in the
    backward. Reports the step and the backward alone (CUDA events around the
    autograd backward on the launching stream), each against the measured HBM
    bandwidth."""
    bsz, seqlen = batch or BATCH, seq or SEQ
    inp = make_inputs(dev, dtype_name, "perchannel", seed=2468, batch=bsz, seq=seqlen)
    leaves = {k: v.detach().requires_grad_() for k, v in inp.items()}
    gy = torch.randn(bsz, seqlen, CHANNELS, 4, device=dev).to(inp["delta"].dtype)
    bwd_ms = []

    def step(record=False):
        for v in leaves.values():
            v.grad = None
        y = op(leaves["delta"], leaves["Lambda"], leaves["B"], leaves["C"], leaves["x"],
               leaves["D"])
        if record:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
        y.backward(gy)
        if record:
            e1.record(stream)
            bwd_ms.append((e0, e1))

    steps = max(3, min(args.steps, 10))
    ms = timed(lambda: step(True), steps, max(3, min(args.warmup, 3)), world, stream) / steps
    torch.cuda.synchronize()
    bwd = [a.elapsed_time(b) for a, b in bwd_ms[-steps:]]
    ms_bwd = sum(bwd) / len(bwd)
    es = inp["B"].element_size()
    fwd_bytes = (2 * inp["B"].numel() * es + 2 * inp["delta"].numel() * inp["delta"].element_size()
                 + inp["Lambda"].numel() * 4 + inp["delta"].numel() * 4 * es)
    bwd_bytes = perchannel_bwd_bytes(inp)
    hbm = peaks["hbm_gbs"]
    ms_max = max_over_ranks(ms, world, dev)
    ms_bwd_max = max_over_ranks(ms_bwd, world, dev)
    res = {
        "value": bsz * seqlen * world / (ms_max / 1e3), "unit": "tokens/s", "ms_per_step": ms_max,
        "backward_ms": ms_bwd_max, "steps": steps, "batch": bsz, "seq_len": seqlen,
        "dtype": "bf16 inputs, f32 state" if dtype_name == "bf16" else "f32",
        "what": "per-channel B/C scan forward (with checkpoints) + backward",
        "roofline": {"bound": "hbm", "kernel": "ssm_scan_bwd_pc_kernel (the backward)",
                     "achieved": bwd_bytes / (ms_bwd / 1e3) / 1e9, "peak": hbm, "unit": "GB/s",
                     "frac": bwd_bytes / (ms_bwd / 1e3) / 1e9 / hbm,
                     "algorithmic_bytes_per_launch": bwd_bytes, "traffic": None,
                     "peak_source": "MEASURED_PEAKS.json hbm_gbs"},
        "roofline_step": {"bound": "hbm", "achieved": (fwd_bytes + bwd_bytes) / (ms / 1e3) / 1e9,
                          "peak": hbm, "unit": "GB/s",
                          "frac": (fwd_bytes + bwd_bytes) / (ms / 1e3) / 1e9 / hbm,
                          "algorithmic_bytes_per_step": fwd_bytes + bwd_bytes},
    }
    del inp, leaves, gy
    torch.cuda.empty_cache()
    return res


def run_perchannel(args, dev, world, stream, op, peaks):
    """The reference block's layout: per-channel B/C [4,2048,1536,64,4]. HBM-bound:
    the roofline is the measured copy bandwidth."""
    inp = make_inputs(dev, args.dtype, "perchannel", seed=4321)
    out = {}

    def step():
        out["y"] = op(inp["delta"], inp["Lambda"], inp["B"], inp["C"], inp["x"], inp["D"])

    step()
    torch.cuda.synchronize()
    y_bytes = out["y"].numel() * out["y"].element_size()
    steps = max(3, min(args.steps, 10))
    ms = timed(step, steps, max(3, min(args.warmup, 3)), world, stream) / steps
    abytes = algorithmic_bytes(inp, y_bytes)
    gbs = abytes / (ms / 1e3) / 1e9
    ms_max = max_over_ranks(ms, world, dev)
    res = {"value": BATCH * SEQ * world / (ms_max / 1e3), "unit": "tokens/s", "ms_per_step": ms_max,
           "steps": steps,
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": abytes}}
    del inp, out
    torch.cuda.empty_cache()
    return res


C5_SEQ = 65536


def config5_measure(args, world, rank, local, gather="peer"):
    """Config 5 (B=1, T=65536, D=1536, N=64, bf16 inputs, fp32 state),
    channel-sharded over the ranks: every rank holds D/world channels of
    delta/x/Lambda/D and the shared B/C, scans them time-parallel, and the
    output y [1, T, D, 4] is assembled on every rank. ``gather="peer"``: each
    scanned time segment is pushed straight into its channel columns of every
    rank's output over NVLink (no permute), under the scan of the next segment;
    ``"nccl"``: NCCL all_gather_into_tensor per segment plus a permute. One step
    = local scan + exchange; max over ranks. Returns the measurement dict."""
    from mambaqc_b200.kernels import ssm_scan_cayley
    from mambaqc_b200.kernels.sharded import ssm_scan_cayley_channel_sharded
    from mambaqc_b200.kernels.ssm_fused import auto_time_chunks

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if CHANNELS % world:
        raise SystemExit(f"{CHANNELS} channels do not split over {world} GPUs")
    dl = CHANNELS // world
    g = torch.Generator(device=dev).manual_seed(77)  # same B/C on every rank
    bf = torch.bfloat16
    Bm = (torch.randn(1, C5_SEQ, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)).to(bf)
    Cm = (torch.randn(1, C5_SEQ, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)).to(bf)
    g.manual_seed(1000 + rank)  # this rank's channels
    x = torch.randn(1, C5_SEQ, dl, generator=g, device=dev).to(bf)
    delta = torch.nn.functional.softplus(
        torch.randn(1, C5_SEQ, dl, generator=g, device=dev) - 3.0).to(bf)
    lam = torch.empty(dl, STATE, 4, device=dev)
    u = torch.rand(dl, STATE, generator=g, device=dev)
    lam[..., 0] = -torch.exp(u * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    lam[..., 1:] = 0.5 * torch.randn(dl, STATE, 3, generator=g, device=dev)
    Dk = torch.ones(dl, device=dev)
    nc = auto_time_chunks(1, C5_SEQ, dl, STATE, dev)
    # the fused peer exchange runs in the scan kernel itself (one call, no segments)
    segs = args.segments if (world > 1 and gather == "nccl") else 1
    stream = torch.cuda.current_stream(dev)
    out = {}

    def step():
        out["y"] = ssm_scan_cayley_channel_sharded(
            delta, lam, Bm, Cm, x, Dk, time_chunks="auto" if segs > 1 else nc, segments=segs,
            gather=gather)

    def scan_only():
        out["yl"] = ssm_scan_cayley(delta, lam, Bm, Cm, x, Dk, time_chunks=nc)

    with torch.no_grad():
        step()
        torch.cuda.synchronize()
        assert out["y"].shape == (1, C5_SEQ, CHANNELS, 4)
        steps = max(3, min(args.steps, 20))
        ms = timed(step, steps, max(3, args.warmup), world, stream) / steps
        ms_max = max_over_ranks(ms, world, dev)
        ms_scan = timed(scan_only, steps, 3, world, stream) / steps
        ms_scan_max = max_over_ranks(ms_scan, world, dev)
    del out
    elems = C5_SEQ * CHANNELS * STATE
    used = gather
    how = {"multicast": "every y quaternion stored once by the scan kernel with multimem.st to "
                        "the multicast address of a symmetric-memory output (NVLink SHARP: "
                        "NVSwitch writes all ranks' buffers; "
                        "mqc_ssm_scan_fwd_chunked_multicast), ordered by two 1-element NCCL "
                        "all-reduces",
           "peer": "every y value stored by the scan kernel into all ranks' outputs over NVLink "
                   "(mqc_ssm_scan_fwd_chunked_peer, CUDA IPC buffers), ordered by two "
                   "1-element NCCL all-reduces",
           "nccl": "NCCL all_gather_into_tensor of y per time segment plus a permute, "
                   "overlapped with the scan of the next segment"}.get(used, used)
    return {
        "value": C5_SEQ / (ms_max / 1e3), "unit": "tokens/s", "ms_per_step": ms_max,
        "steps": steps, "scaling": "strong", "n_gpus": world,
        "dtype": "bf16 inputs, f32 state",
        "config": {"workload": "config5_channel_sharded", "batch": 1, "seq_len": C5_SEQ,
                   "d_inner": CHANNELS, "d_state": STATE, "channels_per_gpu": dl,
                   "time_chunks": nc, "segments": segs,
                   "parallelism": f"channel shards x{world}" + (
                       f", y exchange: {how}" if world > 1 else "")},
        "scan_only_ms": ms_scan_max,
        "exchange_exposed_ms": ms_max - ms_scan_max,
        "scan_fp32_tflops_per_gpu": elems / world * FLOPS_PER_ELEM_SREAL / (ms_scan_max / 1e3) / 1e12,
    }


def run_config5(args, world, rank, local):
    """`--workload config5`: the config-5 measurement as its own JSON line."""
    res = config5_measure(args, world, rank, local, gather=args.gather)
    if rank == 0:
        line = {
            "metric": "config5 long-sequence scan forward tokens/s (B=1, T=65536, D=1536, N=64, "
                      "channel-sharded, y assembled on every rank)",
            "value": res["value"], "unit": "tokens/s", "n_gpus": world, "steps": res["steps"],
            "warmup": max(3, args.warmup), "ms_per_step": res["ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": res["dtype"], "data": "synthetic (seeded, config-3 distributions)",
            "config": res["config"], "scan_only_ms": res["scan_only_ms"],
            "exchange_exposed_ms": res["exchange_exposed_ms"],
            "scan_fp32_tflops_per_gpu": res["scan_fp32_tflops_per_gpu"],
        }
        print(json.dumps(line), flush=True)
    return 0


def config3_strong_measure(args, world, rank, local):
    """Config 3 as one problem of 8192 tokens (B=4, T=2048, D=1536, N=64, shared
    B/C, fp32) split over the ranks: batch shards while the ranks divide the
    batch (4/world rows each), then batch 4-way x channel world/4-way (at 8 GPUs:
    one batch row and 768 channels per rank). Each rank scans its shard with no
    collective on the data path; tokens/s = 8192 / max-rank time."""
    from mambaqc_b200.kernels import ssm_scan_cayley

    dev = torch.device(f"cuda:{local}")
    bs = math.gcd(BATCH, world)
    cs = world // bs
    if CHANNELS % cs:
        raise SystemExit(f"{CHANNELS} channels do not split {cs} ways")
    rows, dl = BATCH // bs, CHANNELS // cs
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    f32 = torch.float32
    x = torch.randn(rows, SEQ, dl, generator=g, device=dev, dtype=f32)
    delta = torch.nn.functional.softplus(torch.randn(rows, SEQ, dl, generator=g, device=dev) - 3)
    lam = torch.empty(dl, STATE, 4, device=dev)
    u = torch.rand(dl, STATE, generator=g, device=dev)
    lam[..., 0] = -torch.exp(u * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    lam[..., 1:] = 0.5 * torch.randn(dl, STATE, 3, generator=g, device=dev)
    Bm = torch.randn(rows, SEQ, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)
    Cm = torch.randn(rows, SEQ, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)
    Dk = torch.ones(dl, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = {}

    def step():
        out["y"] = ssm_scan_cayley(delta, lam, Bm, Cm, x, Dk)

    steps = max(3, min(args.steps, 20))
    with torch.no_grad():
        ms = timed(step, steps, max(3, min(args.warmup, 5)), world, stream) / steps
    ms_max = max_over_ranks(ms, world, dev)
    del out
    return {"value": BATCH * SEQ / (ms_max / 1e3), "unit": "tokens/s", "ms_per_step": ms_max,
            "steps": steps, "scaling": "strong", "n_gpus": world, "dtype": "f32",
            "config": {"workload": "config3_fused_scan_forward", "global_batch": BATCH,
                       "seq_len": SEQ, "d_inner": CHANNELS, "d_state": STATE, "layout": "shared",
                       "shard": {"batch_rows_per_gpu": rows, "channels_per_gpu": dl,
                                 "batch_ways": bs, "channel_ways": cs},
                       "parallelism": "batch x channel shards, no data-path collective"}}


def run_config5_time(args, world, rank, local):
    """Config 5 split by time: rank r holds steps [r*T/G, (r+1)*T/G) of all D
    channels. One step = range summary (state-only pass) + all-gather of the
    summaries + carry + scan of the range from its start state, then an NCCL
    all-gather of y so that every rank holds y [1, T, D, 4], as in the
    channel-sharded form; the time without that gather is reported beside it."""
    from mambaqc_b200.kernels.sharded import ssm_scan_cayley_time_sharded

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if C5_SEQ % world:
        raise SystemExit(f"{C5_SEQ} steps do not split over {world} GPUs")
    tl = C5_SEQ // world
    g = torch.Generator(device=dev).manual_seed(77)
    bf = torch.bfloat16
    Bm = (torch.randn(1, tl, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)).to(bf)
    Cm = (torch.randn(1, tl, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)).to(bf)
    g.manual_seed(1000 + rank)
    x = torch.randn(1, tl, CHANNELS, generator=g, device=dev).to(bf)
    delta = torch.nn.functional.softplus(
        torch.randn(1, tl, CHANNELS, generator=g, device=dev) - 3.0).to(bf)
    g.manual_seed(99)  # Lambda is the same on every rank
    lam = torch.empty(CHANNELS, STATE, 4, device=dev)
    u = torch.rand(CHANNELS, STATE, generator=g, device=dev)
    lam[..., 0] = -torch.exp(u * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    lam[..., 1:] = 0.5 * torch.randn(CHANNELS, STATE, 3, generator=g, device=dev)
    Dk = torch.ones(CHANNELS, device=dev)
    stream = torch.cuda.current_stream(dev)
    y_full = torch.empty(world, tl, CHANNELS, 4, dtype=bf, device=dev)
    out = {}

    def scan_only():
        out["y"], out["hT"] = ssm_scan_cayley_time_sharded(delta, lam, Bm, Cm, x, Dk)

    def step():
        scan_only()
        if world > 1:
            dist.all_gather_into_tensor(y_full, out["y"][0])
        else:
            y_full[0].copy_(out["y"][0])

    with torch.no_grad():
        step()
        torch.cuda.synchronize()
        steps = max(3, min(args.steps, 20))
        ms_max = max_over_ranks(timed(step, steps, max(3, args.warmup), world, stream) / steps,
                                world, dev)
        ms_scan_max = max_over_ranks(timed(scan_only, steps, 3, world, stream) / steps, world,
                                     dev)
    if rank == 0:
        line = {
            "metric": "config5 long-sequence scan forward tokens/s (B=1, T=65536, D=1536, N=64, "
                      "time-sharded, y all-gathered)",
            "value": C5_SEQ / (ms_max / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms_max,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 inputs, f32 state", "data": "synthetic (seeded, config-3 distributions)",
            "config": {"workload": "config5_time_sharded", "batch": 1, "seq_len": C5_SEQ,
                       "d_inner": CHANNELS, "d_state": STATE, "steps_per_gpu": tl,
                       "parallelism": f"time shards x{world}: range summary, NCCL all-gather of "
                                      "the summaries (P, E), carry, range scan; then an NCCL "
                                      "all-gather of y"},
            "without_y_gather_ms": ms_scan_max,
        }
        print(json.dumps(line), flush=True)
    return 0


def run_config2(args, world, rank, local):
    """Config 2: the quaternion primitives on their own, each timed with one pair
    of CUDA events around K back-to-back launches (replays of a CUDA graph of the
    public calls, so host call overhead is not in the kernel figures). Primitives
    whose data fit in L2 rotate over enough independent input/output sets
    (together larger than L2) that every launch reads its input from HBM. Reported against the measured
    HBM bandwidth, with algorithmic bytes = inputs read once + outputs written once."""
    from mambaqc_b200.kernels import (cayley_discretization_fused, parallel_scan_quaternion,
                                      quaternion_layer_norm_fused, quaternion_multiply)

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peaks, peak_kind = measured_peaks()
    hbm = peaks["hbm_gbs"]
    g = torch.Generator(device=dev).manual_seed(0)
    steps = max(8, min(args.steps, 64))
    l2_bytes = 126 << 20

    def time_rotating(fns):
        # the launches are captured once in a CUDA graph and the graph is replayed,
        # so the kernels run back to back without waiting on the Python call path
        k = len(fns)
        for f in fns:
            f()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for f in fns:
                f()
        reps = max(1, steps // k)
        ms = timed(graph.replay, reps, 3, world, stream)
        del graph
        return max_over_ranks(ms / (reps * k), world, dev)

    def sets_for(bytes_per_set):
        return max(1, -(-2 * l2_bytes // bytes_per_set))  # > 2x L2 in total

    res = {}
    with torch.no_grad():
        p = torch.randn(1 << 26, 4, generator=g, device=dev)
        q = torch.randn(1 << 26, 4, generator=g, device=dev)
        ms = time_rotating([lambda: quaternion_multiply(p, q)])
        res["qmul"] = {"shape": [1 << 26, 4], "ms": ms, "bytes": 3 * p.numel() * 4, "sets": 1}
        del p, q
        zs = []
        nz = sets_for(2 * 2 * 16 * 768 * 64 * 16)
        for _ in range(nz):
            z = torch.randn(2, 16, 768, 64, 4, generator=g, device=dev)
            z[..., 0] = -z[..., 0].abs()
            zs.append(z)
        ms = time_rotating([(lambda z=z: cayley_discretization_fused(z)) for z in zs])
        res["cayley"] = {"shape": list(zs[0].shape), "ms": ms, "bytes": 2 * zs[0].numel() * 4,
                         "sets": nz}
        del zs
        u = torch.randn(2, 256, 768, 64, 4, generator=g, device=dev)
        r = torch.rand(2, 256, 768, 64, 1, generator=g, device=dev) * 0.099 + 0.9
        qs = u / torch.linalg.vector_norm(u, dim=-1, keepdim=True) * r
        del u, r
        ms = time_rotating([lambda: parallel_scan_quaternion(qs)])
        res["prefix_scan"] = {"shape": list(qs.shape), "ms": ms, "bytes": 2 * qs.numel() * 4,
                              "sets": 1}
        del qs
        gamma = torch.ones(768, device=dev)
        beta = torch.zeros(768, 4, device=dev)
        nx = sets_for(2 * 4 * 2048 * 768 * 16)
        xs = [torch.randn(4, 2048, 768, 4, generator=g, device=dev) for _ in range(nx)]
        ms = time_rotating([(lambda x=x: quaternion_layer_norm_fused(x, gamma, beta)) for x in xs])
        res["layer_norm"] = {"shape": list(xs[0].shape), "ms": ms, "sets": nx,
                             "bytes": 2 * xs[0].numel() * 4 + gamma.numel() * 4 + beta.numel() * 4}
        # the LayerNorm backward (mqc_qln_bwd): reads q and dout, writes dq, and
        # the per-CTA dgamma/dbeta partials summed in a fixed order
        import ctypes as _ct

        from mambaqc_b200 import _lib
        rows, dm = 4 * 2048, 768
        mean = torch.empty(rows, device=dev)
        rstd = torch.empty(rows, device=dev)
        douts = [torch.randn_like(x) for x in xs]
        dqs = [torch.empty_like(x) for x in xs]
        dgam = torch.empty(dm, device=dev)
        dbet = torch.empty(dm, 4, device=dev)
        lib = _lib.load()
        ws_bytes = lib.mqc_qln_bwd_workspace_size(rows, dm)
        ws = torch.empty(max(1, ws_bytes // 4), device=dev)
        for x in xs[:1]:
            _lib.call("mqc_qln_fwd", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(),
                      dqs[0].data_ptr(), mean.data_ptr(), rstd.data_ptr(), rows, dm, 1e-5, 0,
                      _lib.MQC_DTYPE_F32, stream.cuda_stream)

        def ln_bwd(i):
            _lib.call("mqc_qln_bwd", xs[i].data_ptr(), gamma.data_ptr(), douts[i].data_ptr(),
                      mean.data_ptr(), rstd.data_ptr(), dqs[i].data_ptr(), dgam.data_ptr(),
                      dbet.data_ptr(), ws.data_ptr(), _ct.c_size_t(ws_bytes), rows, dm, 1e-5,
                      _lib.MQC_DTYPE_F32, torch.cuda.current_stream(dev).cuda_stream)
        ms = time_rotating([(lambda i=i: ln_bwd(i)) for i in range(nx)])
        res["layer_norm_backward"] = {"shape": list(xs[0].shape), "ms": ms, "sets": nx,
                                      "bytes": 3 * xs[0].numel() * 4 + gamma.numel() * 4 +
                                      5 * dm * 4}
        del xs, douts, dqs
    for v in res.values():
        v["gbps"] = v["bytes"] / (v["ms"] / 1e3) / 1e9
        v["frac_of_hbm"] = v["gbps"] / hbm
    if rank == 0:
        geo = math.exp(sum(math.log(v["frac_of_hbm"]) for v in res.values()) / len(res))
        line = {
            "metric": "config2 quaternion primitives, HBM bandwidth (geometric mean fraction of "
                      "measured HBM over qmul, Cayley, prefix scan, LayerNorm forward and "
                      "backward)",
            "value": geo, "unit": "fraction of measured HBM GB/s", "n_gpus": world,
            "steps": steps, "warmup": 3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config-2 shapes)",
            "config": {"workload": "config2_primitives",
                       "l2": "Cayley and LayerNorm rotate over input/output sets totalling "
                             "more than 2x L2; qmul and prefix scan inputs exceed L2"},
            "hbm_peak_gbs": hbm, "hbm_peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
            "primitives": res, "gpu_launches": steps * len(res),
        }
        print(json.dumps(line), flush=True)
    return 0


def run_decode(args, world, rank, local):
    """Single-token decode through the block's SSM: each step advances every
    sequence of the decode batch by one token (config-3 channel and state sizes),
    updating the fp32 state cache in place (``ssm_step_cayley``). 64 steps are
    captured in a CUDA graph and replayed, as a generation loop would run them;
    the state cache (B*D*N*16 bytes) is read and written every step."""
    from mambaqc_b200.kernels import ssm_step_cayley

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    bsz, K = args.decode_batch, 64
    g = torch.Generator(device=dev).manual_seed(5 + rank)
    delta = torch.nn.functional.softplus(torch.randn(K, bsz, CHANNELS, generator=g, device=dev) - 3)
    x = torch.randn(K, bsz, CHANNELS, generator=g, device=dev)
    Bm = torch.randn(K, bsz, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)
    Cm = torch.randn(K, bsz, STATE, 4, generator=g, device=dev) / math.sqrt(STATE)
    lam = torch.empty(CHANNELS, STATE, 4, device=dev)
    lam[..., 0] = -torch.exp(torch.rand(CHANNELS, STATE, generator=g, device=dev) *
                             (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3))
    lam[..., 1:] = 0.5 * torch.randn(CHANNELS, STATE, 3, generator=g, device=dev)
    Dk = torch.ones(CHANNELS, device=dev)
    h = torch.zeros(bsz, CHANNELS, STATE, 4, device=dev)
    ys = torch.empty(K, bsz, CHANNELS, 4, device=dev)

    def steps():
        for t in range(K):
            ssm_step_cayley(delta[t], lam, Bm[t], Cm[t], x[t], Dk, h, out=ys[t])

    steps()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        steps()
    reps = max(3, min(args.steps, 50))
    ms = timed(graph.replay, reps, max(3, args.warmup), world, stream) / (reps * K)
    ms = max_over_ranks(ms, world, dev)
    # per step: state read + write, y, inputs (delta, x, B, C), Lambda
    step_bytes = (2 * h.numel() * 4 + bsz * CHANNELS * 16 + bsz * CHANNELS * 8 +
                  2 * bsz * STATE * 16 + lam.numel() * 4)
    peaks, peak_kind = measured_peaks()
    gbps = step_bytes / (ms / 1e3) / 1e9
    if rank == 0:
        line = {
            "metric": "decode tokens/s through the block SSM (one token per sequence per step, "
                      "fp32 state cache updated in place)",
            "value": bsz * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": reps * K, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded, config-3 distributions)",
            "config": {"workload": "decode", "decode_batch": bsz, "d_inner": CHANNELS,
                       "d_state": STATE, "graph_steps": K},
            "roofline": {"bound": "hbm", "achieved": gbps, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": gbps / peaks["hbm_gbs"],
                         "algorithmic_bytes_per_step": step_bytes,
                         "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})"},
            "gpu_launches": reps * K,
        }
        print(json.dumps(line), flush=True)
    return 0


def graph_replay_ms(fns, steps, world, stream, dev):
    """Mean ms per call of the callables `fns`, captured once in a CUDA graph and
    replayed (no host call overhead between kernels); max over ranks."""
    k = len(fns)
    for f in fns:
        f()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for f in fns:
            f()
    reps = max(1, steps // k)
    ms = timed(graph.replay, reps, 3, world, stream)
    del graph
    return max_over_ranks(ms / (reps * k), world, dev)


def run_block_glue(args, world, rank, local):
    """The block's fused glue kernels at the config-4 block shape (B=4, T=2048,
    d_model=768, d_inner=1536) in --dtype, forward and backward, against the torch
    ops of the reference block they replace, timed the same way (CUDA-graph
    replay, input sets rotating over more than 2x L2). Algorithmic bytes = every
    operand read once + every result written once."""
    import torch.nn.functional as F

    from mambaqc_b200.kernels import causal_conv1d_silu, gate_residual, ssm_scan_inputs
    from mambaqc_b200.kernels.block_fused import _ConvSilu, _GateResidual, _ScanInputs

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peaks, peak_kind = measured_peaks()
    hbm = peaks["hbm_gbs"]
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float32
    es = 2 if dt == torch.bfloat16 else 4
    bsz, seqlen, dmod, din, kc = 4, 2048, 768, 1536, 4
    rows = bsz * seqlen
    steps = max(8, min(args.steps, 64))
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape):
        return torch.randn(*shape, generator=g, device=dev).to(dt)

    def nsets(bytes_per_set):
        return max(2, -(-2 * (126 << 20) // bytes_per_set))

    w = torch.randn(din, 1, kc, generator=g, device=dev) * 0.5
    b = torch.randn(din, generator=g, device=dev) * 0.1
    conv = torch.nn.Conv1d(din, din, kc, groups=din, bias=True).to(dev, dt)
    with torch.no_grad():
        conv.weight.copy_(w)
        conv.bias.copy_(b)
    res = {}
    with torch.no_grad():
        # conv + SiLU: x read in place from the [B,T,2*d_inner] in_proj output
        n = nsets(rows * din * es * 4)
        xz = [rnd(bsz, seqlen, 2 * din) for _ in range(n)]
        fused = [(lambda t=t: causal_conv1d_silu(t[..., :din], w, b)) for t in xz]
        torch_ops = [(lambda t=t: F.silu(conv(F.pad(t[..., :din].transpose(1, 2), (kc - 1, 0)))
                                         .transpose(1, 2))) for t in xz]
        res["conv_silu_fwd"] = {"ms": graph_replay_ms(fused, steps, world, stream, dev),
                                "torch_ms": graph_replay_ms(torch_ops, steps, world, stream, dev),
                                "bytes": 2 * rows * din * es}
        gy = rnd(bsz, seqlen, din)

        class _Ctx:
            pass

        def conv_bwd(t):
            c = _Ctx()
            c.saved_tensors = (t[..., :din], w.reshape(din, kc).contiguous(), b)
            c.rs, c.shape, c.w_meta, c.b_dtype = 2 * din, (bsz, seqlen, din, kc), (w.shape, w.dtype), b.dtype
            return _ConvSilu.backward(c, gy)
        res["conv_silu_bwd"] = {"ms": graph_replay_ms([(lambda t=t: conv_bwd(t)) for t in xz],
                                                      steps, world, stream, dev),
                                "bytes": 3 * rows * din * es}
        del xz
        # scan inputs: delta = softplus(u), s = sigmoid(gate) * x
        n = nsets(rows * din * es * 5)
        sets = [(rnd(bsz, seqlen, din), rnd(bsz, seqlen, din), rnd(bsz, seqlen, din))
                for _ in range(n)]
        fused = [(lambda s=s: ssm_scan_inputs(*s)) for s in sets]
        torch_ops = [(lambda s=s: (F.softplus(s[0]), torch.sigmoid(s[1]) * s[2])) for s in sets]
        res["scan_inputs_fwd"] = {"ms": graph_replay_ms(fused, steps, world, stream, dev),
                                  "torch_ms": graph_replay_ms(torch_ops, steps, world, stream, dev),
                                  "bytes": 5 * rows * din * es}
        gd, gs = rnd(bsz, seqlen, din), rnd(bsz, seqlen, din)

        def si_bwd(s):
            c = _Ctx()
            c.saved_tensors = s
            c.meta = (din, din, rows, din, dt, dt)
            return _ScanInputs.backward(c, gd, gs)
        res["scan_inputs_bwd"] = {"ms": graph_replay_ms([(lambda s=s: si_bwd(s)) for s in sets],
                                                        steps, world, stream, dev),
                                  "bytes": 8 * rows * din * es}
        del sets
        # output gate + residual, z read in place from the in_proj output
        n = nsets(rows * dmod * es * 6)
        sets = [(rnd(bsz, seqlen, dmod), rnd(bsz, seqlen, 2 * din), rnd(bsz, seqlen, dmod))
                for _ in range(n)]
        fused = [(lambda s=s: gate_residual(s[0], s[1][..., din:din + dmod], s[2])) for s in sets]
        torch_ops = [(lambda s=s: s[0] + torch.sigmoid(s[1][..., din:din + dmod]) * s[2])
                     for s in sets]
        res["gate_residual_fwd"] = {"ms": graph_replay_ms(fused, steps, world, stream, dev),
                                    "torch_ms": graph_replay_ms(torch_ops, steps, world, stream,
                                                                dev),
                                    "bytes": 4 * rows * dmod * es}
        go = rnd(bsz, seqlen, dmod)

        def gr_bwd(s):
            c = _Ctx()
            c.saved_tensors = (s[1][..., din:din + dmod], s[2])
            c.meta = (2 * din, rows, dmod, dt, dt, dt)
            return _GateResidual.backward(c, go)
        res["gate_residual_bwd"] = {"ms": graph_replay_ms([(lambda s=s: gr_bwd(s)) for s in sets],
                                                          steps, world, stream, dev),
                                    "bytes": 5 * rows * dmod * es}
        del sets
    for v in res.values():
        v["gbps"] = v["bytes"] / (v["ms"] / 1e3) / 1e9
        v["frac_of_hbm"] = v["gbps"] / hbm
        if "torch_ms" in v:
            v["speedup_vs_torch_ops"] = v["torch_ms"] / v["ms"]
    if rank == 0:
        geo = math.exp(sum(math.log(v["frac_of_hbm"]) for v in res.values()) / len(res))
        line = {
            "metric": "block glue kernels (conv+SiLU, scan inputs, gate+residual; forward and "
                      "backward), geometric mean fraction of measured HBM",
            "value": geo, "unit": "fraction of measured HBM GB/s", "n_gpus": world,
            "steps": steps, "warmup": 3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32" if dt == torch.float32 else "bf16",
            "data": "synthetic (seeded N(0,1))",
            "config": {"workload": "block_glue_config4_shape", "batch": bsz, "seq_len": seqlen,
                       "d_model": dmod, "d_inner": din, "d_conv": kc,
                       "l2": "input sets rotate over more than 2x L2"},
            "hbm_peak_gbs": hbm, "hbm_peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
            "kernels": res, "gpu_launches": None,
        }
        print(json.dumps(line), flush=True)
    return 0


def time_fused_parts(bsz, seqlen, din, dmod, nst, chans, dev, world, stream, steps, seed=1):
    """The two halves of the block fused into tcgen05 kernels here, each timed
    against the unfused form it replaces (forward, bf16): the B/C projections +
    per-channel scan over ``chans`` channels (``bc_proj_scan`` against cuBLAS
    projections + ``ssm_scan_cayley``), and the LayerNorm + output projection
    (``quaternion_layer_norm_linear`` against the LayerNorm kernel + cuBLAS).
    Returns ({name: ms}, {name: TFLOP/s of the projections})."""
    from mambaqc_b200.kernels import quaternion_layer_norm_fused, ssm_scan_cayley
    from mambaqc_b200.kernels.bc_proj_scan import bc_proj_scan
    from mambaqc_b200.kernels.quaternion_norm import quaternion_layer_norm_linear

    g = torch.Generator(device=dev).manual_seed(seed)
    bf = torch.bfloat16
    xa3 = torch.randn(bsz, seqlen, din, generator=g, device=dev).to(bf)
    std = (2.0 / (din + chans * nst)) ** 0.5
    wb = (torch.randn(chans * nst * 4, din, generator=g, device=dev) * std).to(bf)
    wc = (torch.randn(chans * nst * 4, din, generator=g, device=dev) * std).to(bf)
    dl = torch.nn.functional.softplus(torch.randn(bsz, seqlen, chans, generator=g, device=dev)
                                      - 3.0).to(bf)
    sg = torch.randn(bsz, seqlen, chans, generator=g, device=dev).to(bf)
    lam = torch.empty(chans, nst, 4, device=dev)
    lam[..., 0] = -0.01
    lam[..., 1:] = 0.3
    dsk = torch.ones(chans, device=dev)
    yq = torch.randn(bsz, seqlen, din, 4, generator=g, device=dev).to(bf)
    gam = torch.ones(din, device=dev)
    bet = torch.zeros(din, 4, device=dev)
    wo = (torch.randn(dmod, 4 * din, generator=g, device=dev) * (4 * din) ** -0.5).to(bf)

    def bc_fused():
        with torch.no_grad():
            bc_proj_scan(xa3, wb, wc, dl, lam, sg, dsk)

    def bc_unfused():
        with torch.no_grad():
            Bq = (xa3 @ wb.t()).view(bsz, seqlen, chans, nst, 4)
            Cq = (xa3 @ wc.t()).view(bsz, seqlen, chans, nst, 4)
            ssm_scan_cayley(dl, lam, Bq, Cq, sg, dsk)

    def ln_fused():
        with torch.no_grad():
            quaternion_layer_norm_linear(yq, gam, bet, wo)

    def ln_unfused():
        with torch.no_grad():
            quaternion_layer_norm_fused(yq, gam, bet).flatten(-2) @ wo.t()

    parts = {}
    for name, f in (("bc_proj_scan_fused", bc_fused), ("bc_proj_scan_unfused", bc_unfused),
                    ("ln_out_proj_fused", ln_fused), ("ln_out_proj_unfused", ln_unfused)):
        parts[name] = max_over_ranks(timed(f, 4 * steps, 3, world, stream) / (4 * steps), world,
                                     dev)
    bc_flops = 2 * 2 * bsz * seqlen * din * chans * nst * 4
    ln_flops = 2 * bsz * seqlen * (4 * din) * dmod
    tflops = {k: (bc_flops if k.startswith("bc") else ln_flops) / (v / 1e3) / 1e12
              for k, v in parts.items()}
    return parts, tflops


def run_fused_parts(args, world, rank, local):
    """`--workload fused_parts`: the tcgen05 fusions against their unfused forms
    at the config-4 block shape (B=4, T=2048, d_inner 1536, d_state 64, d_model
    768), or a smaller case with --prof-batch / --prof-seq / --prof-channels
    (the number of scan channels the projections produce)."""
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    bsz = args.prof_batch or 4
    seqlen = args.prof_seq or 2048
    chans = args.prof_channels or 1536
    steps = max(1, min(args.steps, 10))
    parts, tflops = time_fused_parts(bsz, seqlen, 1536, 768, 64, chans, dev, world, stream, steps,
                                     seed=1 + rank)
    if rank == 0:
        line = {
            "metric": "tcgen05 fusions of the block against their unfused forms (forward ms)",
            "value": parts["bc_proj_scan_fused"], "unit": "ms", "n_gpus": world,
            "steps": 4 * steps, "warmup": 3, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
            "config": {"workload": "fused_parts", "batch": bsz, "seq_len": seqlen,
                       "d_inner": 1536, "d_model": 768, "d_state": 64, "scan_channels": chans},
            "parts_ms": parts, "parts_tflops": tflops,
        }
        print(json.dumps(line), flush=True)
    return 0


def run_config4_block(args, world, rank, local):
    """One block of the config-4 base preset (d_model 768, d_state 64, d_inner
    1536) at B=4 per GPU, T=2048: forward + loss + backward under bf16 autocast,
    the per-layer share of a config-4 training step (the full 14.66 B-parameter
    model does not fit one replica per GPU with an fp32 optimizer). Reports the
    time split into the per-channel B/C projections (cuBLAS) and the rest, and
    the projection GEMMs' fraction of the measured bf16 tensor peak."""
    from mambaqc_b200.models import QuaternionMamba2Block

    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    bsz, seqlen, dmod, nst = 4, 2048, 768, 64
    torch.manual_seed(0)
    blk = QuaternionMamba2Block(dmod, d_state=nst).to(dev)
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    x = torch.randn(bsz, seqlen, dmod, generator=g, device=dev).requires_grad_()
    gout = torch.randn(bsz, seqlen, dmod, generator=g, device=dev)

    def step():
        blk.zero_grad(set_to_none=True)
        x.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = blk(x)
        (out.float() * gout).sum().backward()

    xa = torch.randn(bsz * seqlen, 2 * dmod, generator=g, device=dev).to(torch.bfloat16)
    wb = blk.B_proj.weight.detach().to(torch.bfloat16) if hasattr(blk.B_proj, "weight") else None

    def proj_only():
        # the two per-channel projections' GEMMs of one step: forward and the two
        # backward GEMMs (input and weight gradients), for B and C
        for _ in range(2):
            yb = xa @ wb.t()
            _ = yb @ wb
            _ = yb.t() @ xa

    steps = max(3, min(args.steps, 10))
    step()
    torch.cuda.synchronize()
    ms = max_over_ranks(timed(step, steps, max(3, args.warmup), world, stream) / steps, world, dev)
    ms_proj = None
    if wb is not None:
        ms_proj = max_over_ranks(timed(proj_only, steps, 3, world, stream) / steps, world, dev)

    # the block's forward alone (inference, no autograd), with the B/C
    # projections fused into the scan and without (cuBLAS projections + scan)
    def fwd(fused):
        def run():
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
                blk(x, fused_bc_proj=fused)
        return run

    ms_fwd = {k: max_over_ranks(timed(fwd(k == "fused"), steps, 3, world, stream) / steps,
                                world, dev) for k in ("unfused", "fused")}

    parts, parts_tflops = time_fused_parts(bsz, seqlen, 2 * dmod, dmod, nst, 2 * dmod, dev, world,
                                           stream, steps, seed=1 + rank)

    peaks, peak_kind = measured_peaks()
    din = 2 * dmod
    proj_flops = 2 * 3 * 2 * (bsz * seqlen) * din * (din * nst * 4)
    if rank == 0:
        line = {
            "metric": "config-4 base block forward+backward tokens/s (one of 12 layers, bf16 "
                      "autocast, fp32 scan state)",
            "value": bsz * seqlen * world / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 autocast", "data": "synthetic (seeded N(0,1) block input)",
            "config": {"workload": "config4_base_block", "batch_per_gpu": bsz, "seq_len": seqlen,
                       "d_model": dmod, "d_inner": din, "d_state": nst,
                       "parallelism": f"dp{world} (independent replicas of one block)"},
            "bc_projection_gemms_ms": ms_proj,
            "bc_projection_tflops": (proj_flops / (ms_proj / 1e3) / 1e12) if ms_proj else None,
            "bc_projection_frac_of_bf16_peak": ((proj_flops / (ms_proj / 1e3) / 1e12) /
                                                peaks.get("bf16_tflops_sustained",
                                                          peaks.get("bf16_tflops", 1590.0))
                                                if ms_proj else None),
            "bf16_peak_source": f"MEASURED_PEAKS.json ({peak_kind})",
            "forward_ms": {"unfused_bc_proj": ms_fwd["unfused"], "fused_bc_proj": ms_fwd["fused"]},
            "fused_parts_ms": parts,
            "fused_parts_tflops": parts_tflops,
        }
        print(json.dumps(line), flush=True)
    return 0


def main():
    args = parse_args()
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            return run_reference(args, world, rank)
        if args.workload == "config5" and args.shard == "time":
            return run_config5_time(args, world, rank, local)
        if args.workload == "config5":
            return run_config5(args, world, rank, local)
        if args.workload == "config2":
            return run_config2(args, world, rank, local)
        if args.workload == "decode":
            return run_decode(args, world, rank, local)
        if args.workload == "fused_parts":
            return run_fused_parts(args, world, rank, local)
        if args.workload == "block_glue":
            return run_block_glue(args, world, rank, local)
        if args.workload == "config4_block":
            return run_config4_block(args, world, rank, local)
        return run_b200(args, world, rank, local)
    finally:
        if dist.is_initialized():
            from mambaqc_b200.kernels.sharded import release_peer_outputs
            release_peer_outputs()
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
