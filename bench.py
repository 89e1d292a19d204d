#!/usr/bin/env python
"""Benchmark: achieved HBM GB/s and rows/s of the row-wise kernels on 1..8 B200s; prints ONE JSON line (rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference] [--no-sweep]
  N > 1: python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

Headline workload (`--workload`, default rmsnorm_16384x4096, the BASELINE config RMSNorm bf16 [16384, 4096] with a
[4096] weight): a step is one kernel launch over one [16384, 4096] batch. Every rank runs its own batch (weak
scaling: the global batch is N x 16384 rows, row-sharded, no communication). Inputs are resident in HBM and rotate
over two buffer sets; every set moves more bytes than the 126 MB L2 holds, so no step reads the previous step's
lines. `value` = all ranks' algorithmic bytes / the max over ranks of the device time of the K timed steps.
`e2e` = the same metric through the public API (ckb200.<op>) with the step's input copied from pinned host memory
and its output copied back inside the timed region. `roofline` divides the kernel's achieved GB/s by the measured
copy bandwidth in MEASURED_PEAKS.json. At N = 1 the line also carries `kernels`: every BASELINE config measured the
same way (device time, rotated buffers) beside the reference's own kernels rebuilt for sm_100a (oracle/_ref).
`--impl reference` times the reference's CPU path on the host cores instead (the oracle's torch restatement; the
reference's own CPU code where it has one, softmax/baseline.py), on rank 0 only.
"""

import argparse
import ctypes
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "cuda-kernels-optimized-for-rtx5090_b200")
sys.path[:0] = [p for p in (ROOT, PKG_DIR) if p not in sys.path]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "achieved HBM GB/s (fraction of 8 TB/s) and rows/s per kernel at 1/2/4/8 B200"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
HEADLINE = "rmsnorm_16384x4096"


# ------------------------------------------------------------------------------------------------ environment ----
def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel):
    """DRAM bytes per launch recorded from an ncu capture in profiles/ (a `traffic_bytes_per_launch[kernel]: N`
    line), or None."""
    pat = re.compile(r"traffic_bytes_per_launch\[" + re.escape(kernel) + r"\]:\s*([0-9.eE+]+)")
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for name in sorted(os.listdir(pdir)):
        if name.endswith((".md", ".txt")):
            with open(os.path.join(pdir, name)) as f:
                m = pat.search(f.read())
            if m:
                return float(m.group(1))
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running (the timed region)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank):
        # nvidia-smi numbers GPUs physically; map the process's device through CUDA_VISIBLE_DEVICES (index or UUID)
        visible = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        self.gpu = visible[local_rank].strip() if local_rank < len(visible) else str(local_rank)
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.out = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.out, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.out is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.out.seek(0)
        rows = [[c.strip() for c in line.split(",")] for line in self.out if line.count(",") >= 8]
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s in sm if smax and s > 0.5 * max(smax)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons, "samples": len(rows)}


def setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    if args.impl == "ours":
        if not torch.cuda.is_available():
            raise SystemExit("bench: no CUDA device")
        torch.cuda.set_device(local)
        if world > 1:
            dist.init_process_group("nccl", rank=rank, world_size=world,
                                    timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
    return rank, world, local


def max_over_ranks(v, world):
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


# ---------------------------------------------------------------------------------------------- workloads -------
def _lib(op):
    from ckb200 import _native

    return _native.load(op)


def _ref_lib(op):
    path = os.path.join(ROOT, "oracle", "_ref", op, "libkernel.so")
    return ctypes.CDLL(path) if os.path.exists(path) else None


class Case:
    """One workload on the device: `launch(i)` runs step i (buffer set i % sets) through the C ABI of `impl`
    ("ours" or "ref" = the reference's kernel rebuilt for sm_100a); bytes/rows per step."""

    def __init__(self, name, bytes_per_step, rows_per_step, launch, sets, check=None, kernel=None):
        self.name, self.bytes, self.rows, self.launch, self.sets = name, bytes_per_step, rows_per_step, launch, sets
        self.check = check
        self.kernel = kernel


def make_case(name, impl="ours", seeded=True, sets=2):
    """Device buffers for workload `name`. seeded: the workloads module's CPU-seeded inputs (checkable against the
    oracle); otherwise the same distributions drawn on the device (faster to make)."""
    from ckb200 import workloads

    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream().cuda_stream
    nbytes = workloads.ALGORITHMIC_BYTES[name]
    rows = workloads.ROWS[name]
    g = torch.Generator(device=dev).manual_seed(1234)

    def dev_randn(*shape, scale=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)

    if name == "rmsnorm_16384x4096":
        if seeded:
            base = workloads.rmsnorm_16384x4096()
            x0, w = base["x"].to(dev), base["weight"].to(dev)
        else:
            x0 = dev_randn(16384, 4096, dtype=torch.bfloat16)
            w = (1 + dev_randn(4096, scale=0.1)).to(torch.bfloat16)
        xs = [x0] + [x0.clone() for _ in range(sets - 1)]
        ys = [torch.empty_like(x0) for _ in range(sets)]
        if impl == "ours":
            fn = _lib("rmsnorm").ckb_rmsnorm_weighted_launch

            def launch(i):
                return fn(xs[i % sets].data_ptr(), w.data_ptr(), ys[i % sets].data_ptr(), 16384, 4096, 1, 1, 1e-6,
                          stream)
        else:
            lib = _ref_lib("rmsnorm")
            if lib is None:
                return None
            lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
            # the reference has no weight: its unweighted kernel over the same x (the bytes differ by 8 KiB)

            def launch(i):
                return lib.launch(xs[i % sets].data_ptr(), ys[i % sets].data_ptr(), 16384, 4096, 1, 1e-6, 256, stream)

        def check():
            from oracle import rmsnorm as orc
            from oracle.numerics import to_f32, ulp_distance

            xc = xs[0][:64].cpu()
            want = orc.rmsnorm(xc, w.cpu()) if impl == "ours" else orc.rmsnorm(xc)
            return int(ulp_distance(to_f32(ys[0][:64]), to_f32(want), torch.bfloat16).max()) <= 1

        return Case(name, nbytes, rows, launch, sets, check, "rms_block_rows")

    if name.startswith("softmax_"):
        shape = {"softmax_4096x8192": (4096, 8192), "softmax_256x262144": (256, 262144),
                 "softmax_262144x128": (262144, 128)}[name]
        if seeded:
            x0 = getattr(workloads, name)()["x"].to(dev)
        else:
            scale = {"softmax_4096x8192": 2.0, "softmax_256x262144": 4.0, "softmax_262144x128": 1.0}[name]
            x0 = dev_randn(*shape, scale=scale)
        xs = [x0] + [x0.clone() for _ in range(sets - 1)]
        ys = [torch.empty_like(x0) for _ in range(sets)]
        lib = _lib("softmax") if impl == "ours" else _ref_lib("softmax")
        if lib is None:
            return None
        lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int,
                               ctypes.c_int, ctypes.c_int, ctypes.c_void_p]

        def launch(i):
            return lib.launch(xs[i % sets].data_ptr(), ys[i % sets].data_ptr(), shape[0], shape[1], 0, 256, 1024,
                              stream)

        kern = {"softmax_4096x8192": "sm_block", "softmax_256x262144": "sm_cluster",
                "softmax_262144x128": "sm_group"}[name]
        return Case(name, nbytes, rows, launch, sets, None, kern)

    if name == "rope_8x4096":
        base = workloads.rope_8x4096() if seeded else None
        if seeded:
            q0, k0 = base["q"].to(dev), base["k"].to(dev)
            cos, sin, ids = base["cos"].to(dev), base["sin"].to(dev), base["position_ids"].to(dev)
        else:
            q0 = dev_randn(8, 4096, 32, 128, dtype=torch.bfloat16)
            k0 = dev_randn(8, 4096, 8, 128, dtype=torch.bfloat16)
            c, s = workloads._rope_cache(10000.0, 128, 4096, torch.float32)
            cos, sin = c.to(dev), s.to(dev)
            ids = torch.arange(4096, device=dev).repeat(8, 1)
        qs = [q0] + [q0.clone() for _ in range(sets - 1)]
        ks = [k0] + [k0.clone() for _ in range(sets - 1)]
        lib = _lib("rope") if impl == "ours" else _ref_lib("rope")
        if lib is None:
            return None
        lib.launch.argtypes = [ctypes.c_void_p] * 7 + [ctypes.c_longlong] + [ctypes.c_int] * 7 + [ctypes.c_void_p]
        if impl == "ours":  # in place, the BASELINE config
            def launch(i):
                q, k = qs[i % sets], ks[i % sets]
                return lib.launch(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), ids.data_ptr(),
                                  q.data_ptr(), k.data_ptr(), 32768, 32, 8, 128, 1, 0, 40, 1, stream)
        else:  # the reference's wrapper is out of place (rope/candidate.py:50); same bytes moved
            qo = [torch.empty_like(q0) for _ in range(sets)]
            ko = [torch.empty_like(k0) for _ in range(sets)]

            def launch(i):
                q, k = qs[i % sets], ks[i % sets]
                return lib.launch(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), ids.data_ptr(),
                                  qo[i % sets].data_ptr(), ko[i % sets].data_ptr(), 32768, 32, 8, 128, 1, 0, 40, 1,
                                  stream)
        return Case(name, nbytes, rows, launch, sets, None, "rope_tokens")

    if name == "topk_512x151936":
        x0 = workloads.topk_512x151936()["x"].to(dev) if seeded else dev_randn(512, 151936, scale=3.0)
        xs = [x0] + [x0.clone() for _ in range(sets - 1)]
        lib = _lib("topk") if impl == "ours" else _ref_lib("topk")
        if lib is None:
            return None
        lib.plan.argtypes = [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                             ctypes.c_int]
        lib.plan.restype = ctypes.c_longlong
        lib.launch.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int,
                                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_longlong,
                                                       ctypes.c_void_p]
        chunk = lib.plan(512, 151936, 0, 256, 4, 2048)
        nch = -(-151936 // chunk)
        work = torch.empty(max(1, 512 * nch * 50), dtype=torch.int64, device=dev)
        counters = torch.zeros(4096, dtype=torch.int32, device=dev)
        vals = torch.empty(512, 50, device=dev)
        idx = torch.empty(512, 50, dtype=torch.int64, device=dev)

        def launch(i):
            return lib.launch(xs[i % sets].data_ptr(), vals.data_ptr(), idx.data_ptr(), work.data_ptr(),
                              counters.data_ptr(), 512, 151936, 50, 0, 256, 4, chunk, stream)

        return Case(name, nbytes, rows, launch, sets, None, "topk_stream")
    raise SystemExit(f"unknown workload {name}")


def time_case(case, steps, warmup, world, sampler_gpu=None):
    """Device time (ms) of `steps` launches after `warmup`, max over ranks; clocks sampled meanwhile."""
    for i in range(warmup):
        err = case.launch(i)
        if err:
            raise RuntimeError(f"{case.name}: launch returned {err}")
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(sampler_gpu) if sampler_gpu is not None else None
    if sampler:
        sampler.__enter__()
    start.record()
    for i in range(steps):
        case.launch(warmup + i)
    end.record()
    torch.cuda.synchronize()
    if sampler:
        sampler.__exit__(None, None, None)
    ms = start.elapsed_time(end)
    barrier(world)
    return max_over_ranks(ms, world), (sampler.summary() if sampler else None)


def e2e_rmsnorm(steps, warmup, world, chunks=8):
    """Public API end to end: pinned host x -> device -> ckb200.rmsnorm.rmsnorm -> pinned host y, every step moving
    the whole batch in and out, through ckb200.hostpipe.RowPipeline (row chunks on copy-in / compute / copy-out
    streams, so the two copy directions and the kernels overlap)."""
    from ckb200 import hostpipe, rmsnorm, workloads

    base = workloads.rmsnorm_16384x4096()
    hx = base["x"].pin_memory()
    hy = torch.empty_like(hx).pin_memory()
    w = base["weight"].cuda()
    rows, cols = hx.shape
    pipe = hostpipe.RowPipeline(lambda x, y: rmsnorm.rmsnorm(x, w, out=y), rows, cols, hx.dtype, chunks=chunks)

    for _ in range(warmup):
        pipe(hx, hy)
    pipe.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pipe.record_start(start)
    for _ in range(steps):
        pipe(hx, hy)
    pipe.record_end(end)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    nbytes = workloads.ALGORITHMIC_BYTES[HEADLINE]
    return {"value": round(world * nbytes * steps / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": hx.numel() * hx.element_size(),
            "d2h_bytes_per_step": hy.numel() * hy.element_size(), "ms_per_step": round(ms / steps, 4),
            "pipeline": f"{len(pipe.bounds)} row chunks, copy-in / compute / copy-out streams"}


# --------------------------------------------------------------------------------------------- CPU baselines ----
def cpu_sample_rate(name, min_seconds=10.0, max_reps=5000, reps_exact=None):
    """GB/s of the reference's CPU path (the oracle's torch restatement, all host threads) on a bounded sample of
    workload `name`: at least 3 repetitions and min_seconds (at most max_reps), or exactly reps_exact;
    returns (GB/s, sample description, threads)."""
    from ckb200 import workloads
    from oracle import rmsnorm as orms
    from oracle import rope as orope
    from oracle import softmax as osm
    from oracle import topk as otk

    torch.set_num_threads(os.cpu_count() or 1)
    if name == "rmsnorm_16384x4096":
        inp = workloads.rmsnorm_16384x4096(scale=8)
        x, w = inp["x"], inp["weight"]
        fn, nbytes, what = (lambda: orms.rmsnorm_cpu(x, w)), 2 * x.numel() * 2 + w.numel() * 2, \
            "2048 of the 16384 rows (x bf16 [2048, 4096] + weight), torch CPU restatement"
    elif name.startswith("softmax_"):
        x = getattr(workloads, name)(scale=8)["x"]
        fn, nbytes, what = (lambda: osm.softmax_cpu(x)), 2 * x.numel() * 4, \
            f"1/8 of the rows {tuple(x.shape)}, the reference's torch.softmax (softmax/baseline.py:13)"
    elif name == "rope_8x4096":
        inp = workloads.rope_8x4096(scale=8)
        fn = lambda: orope.rope_cpu(inp["q"], inp["k"], inp["cos"], inp["sin"], inp["position_ids"])  # noqa: E731
        nbytes = 2 * (inp["q"].numel() + inp["k"].numel()) * 2
        what = "1 of the 8 batches, torch CPU restatement"
    else:
        x = workloads.topk_512x151936(scale=8)["x"]
        fn, nbytes, what = (lambda: otk.topk_cpu(x, 50)), x.numel() * 4, \
            "64 of the 512 rows, torch CPU stable sort"
    fn()
    reps, t0 = 0, time.perf_counter()
    while (reps < reps_exact) if reps_exact else \
            (reps < 3 or (time.perf_counter() - t0 < min_seconds and reps < max_reps)):
        fn()
        reps += 1
    dt = time.perf_counter() - t0
    return nbytes * reps / dt / 1e9, f"{what}, {reps} reps in {dt:.1f} s", torch.get_num_threads()


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    from ckb200 import workloads

    cpu_sample_rate(args.workload, reps_exact=args.warmup)  # warm-up steps
    # timed: exactly K steps, each one bounded sample (1/8 of the workload's rows)
    gbs, sample, threads = cpu_sample_rate(args.workload, reps_exact=args.steps)
    per_step_ms = workloads.ALGORITHMIC_BYTES[args.workload] / 8 / (gbs * 1e9) * 1e3
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": _dtype(args.workload),
            "data": "synthetic (seeded, BASELINE config distributions)",
            "config": {"workload": args.workload, "sample": sample},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _dtype(name):
    return {"rmsnorm_16384x4096": "bf16", "rope_8x4096": "bf16"}.get(name, "f32")


# -------------------------------------------------------------------------------------------------- main --------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=HEADLINE)
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-kernel sweep of the other configs")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--sweep-steps", type=int, default=300)
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--vocab-exchange", choices=("peer", "nccl"), default="peer",
                    help="topk_vocab workload: the fused peer-memory exchange or an NCCL all-gather")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank, world, local = setup(args)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    from ckb200 import workloads

    if args.workload == "topk_vocab_512x151936":
        run_vocab(args, rank, world, local)
        return
    peak, peak_kind = hbm_peak()
    case = make_case(args.workload)
    ms, clocks = time_case(case, args.steps, args.warmup, world, sampler_gpu=local)
    ok = case.check() if case.check else None
    gbs = world * case.bytes * args.steps / (ms * 1e-3) / 1e9
    rows_s = world * case.rows * args.steps / (ms * 1e-3)
    achieved = case.bytes / (ms / args.steps * 1e-3) / 1e9  # one launch per step
    traffic = ncu_traffic(case.kernel)
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": _dtype(args.workload),
        "data": "synthetic (seeded, BASELINE config distributions)",
        "config": {"workload": args.workload, "rows_per_gpu": case.rows, "parallelism": f"row-sharded x{world}",
                   "l2": f"inputs larger than L2, rotated over {case.sets} buffer sets"},
        "rows_per_s": round(rows_s, 1), "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "kernel": case.kernel},
        "clocks": clocks, "gpu_launches": args.steps, "check": ok,
    }
    if args.workload == HEADLINE:
        line["e2e"] = e2e_rmsnorm(args.e2e_steps, 3, world)
    if world == 1 and rank == 0 and not args.no_cpu:
        gbs_cpu, sample, threads = cpu_sample_rate(args.workload)
        line["cpu_baseline"] = {"value": round(gbs_cpu, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                                "sample": sample}
    if world == 1 and rank == 0 and not args.no_sweep:
        line["kernels"] = sweep(args, world)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_vocab(args, rank, world, local):
    """Vocab-sharded top-k (strong scaling): the [512, 151936] fp32 logits split by columns over the ranks; a step is
    the local top-50 kernel, the exchange of the [512, 50] composite lists (by default fused into the kernels over
    peer memory; --vocab-exchange nccl: one NCCL all-gather) and the merge kernel."""
    from ckb200 import sharded, workloads

    peak, peak_kind = hbm_peak()
    dev = torch.device("cuda", local)
    full = workloads.topk_512x151936()["x"]
    lo, hi = sharded.col_range(full.shape[1], rank, world)
    shards = [full[:, lo:hi].contiguous().to(dev) for _ in range(2)]  # two copies: rotate past L2
    peer = args.vocab_exchange == "peer"
    op = (sharded.PeerVocabShardedTopK if peer else sharded.VocabShardedTopK)(full.shape[0], 50, device=dev)
    run_step = lambda i: op(shards[i % 2], lo)  # noqa: E731 (eager: one kernel per step on the peer path)
    for i in range(args.warmup):
        run_step(i)
    torch.cuda.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    sampler.__enter__()
    start.record()
    for i in range(args.steps):
        values, indices = run_step(i)
    end.record()
    torch.cuda.synchronize()
    sampler.__exit__(None, None, None)
    ms = max_over_ranks(start.elapsed_time(end), world)
    nbytes = workloads.ALGORITHMIC_BYTES["topk_512x151936"]
    ok = None
    if rank == 0:
        from oracle import topk as otk
        wv, wi = otk.topk(full, 50)
        ok = bool(torch.equal(indices.cpu(), wi) and torch.equal(values.cpu(), wv))
        line = {"metric": METRIC, "value": round(nbytes * args.steps / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (seeded, BASELINE config distributions)",
                "config": {"workload": args.workload, "cols_per_gpu": hi - lo, "parallelism": f"vocab-sharded x{world}",
                           "collective": ("fused: the shard kernel stores its [512, 50] composite lists into every "
                                          "rank's memory over NVLink (CUDA IPC) and raises per-row flags; the merge "
                                          "kernel waits on them and merges, one kernel per step" if peer else
                                          "NCCL all_gather_into_tensor of [512, 50] int64 composites")},
                "rows_per_s": round(512 * args.steps / (ms * 1e-3), 1),
                "roofline": {"bound": "hbm", "achieved": round(nbytes / world / (ms / args.steps * 1e-3) / 1e9, 1),
                             "peak": peak, "unit": "GB/s per GPU", "peak_kind": peak_kind},
                "clocks": sampler.summary(), "gpu_launches": 2 * args.steps, "check": ok}
        print(json.dumps(line), flush=True)
    if peer:
        op.close()
    if world > 1:
        dist.destroy_process_group()


def sweep(args, world):
    """Every BASELINE config: ours and the reference's kernel (rebuilt for sm_100a), device time, rotated buffers."""
    from ckb200 import workloads

    peak, _ = hbm_peak()
    out = {}
    for name in ("softmax_4096x8192", "rmsnorm_16384x4096", "rope_8x4096", "softmax_256x262144",
                 "softmax_262144x128", "topk_512x151936"):
        entry = {}
        for impl in ("ours", "ref"):
            case = make_case(name, impl=impl, seeded=False)
            if case is None:
                continue
            ms, _ = time_case(case, args.sweep_steps, 10, world)
            per = ms / args.sweep_steps
            gbs = case.bytes / (per * 1e-3) / 1e9
            entry[impl] = {"us": round(per * 1e3, 2), "GB/s": round(gbs, 1), "frac_measured": round(gbs / peak, 4),
                           "rows_per_s": round(case.rows / (per * 1e-3), 1)}
            del case
            torch.cuda.empty_cache()
        out[name] = entry
    return out


if __name__ == "__main__":
    main()
