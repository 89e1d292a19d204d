#!/usr/bin/env python
"""Benchmark: achieved HBM GB/s and rows/s of the row-wise kernels on 1..8 B200s; prints ONE JSON line (rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference] [--no-sweep]
  N > 1: python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N

Headline workload (`--workload`, default rmsnorm_16384x4096, the BASELINE config RMSNorm bf16 [16384, 4096] with a
[4096] weight): a step is one kernel launch over one [16384, 4096] batch. Every rank runs its own batch (weak
scaling: the global batch is N x 16384 rows, row-sharded, no communication). Inputs are resident in HBM and rotate
over buffer sets that together move more bytes than twice the 126 MB L2, so no step reads the previous step's lines.
`value` = all ranks' algorithmic bytes / the max over ranks of the device time of the K timed steps.
`e2e` = the same metric through the public API (ckb200.<op>) with the step's input copied from pinned host memory
and its output copied back inside the timed region. `roofline` divides the kernel's achieved GB/s by the measured
copy bandwidth in MEASURED_PEAKS.json.

Sub-records on the same line:
  strong      at every N: each row workload split N ways (rows or tokens per rank = 1/N of the
              config), per-rank device time (max over ranks), aggregate GB/s, and the speed-up over one GPU running
              the whole config (timed in the same run, on every rank's own GPU, max over ranks);
  vocab_topk  at every N: the vocab-sharded top-k over NVLink peer memory (the [512, 151936] config split by
              columns), time per step and a bit-exact check of the answer against the oracle;
  rope_tokens at every N: the RoPE config's tokens split N ways, rotated in place by each rank, every rank's shard
              checked bit for bit against the oracle on a sample of its tokens;
  host_copy   at every N: the pinned host <-> device copy rate every rank reaches at once (the e2e ceiling);
  kernels     at N = 1: every BASELINE config, ours beside the reference's own kernels rebuilt for sm_100a
              (oracle/_ref), with the reference's CPU path timed at the full config and an end-to-end number
              through the public API;
  latency     at N = 1: decode-sized calls (top-k 1 x 128256, RMSNorm 1 x 4096, RoPE decode batch 1/16/64, softmax
              1 x 128256) as eager calls and as CUDA-graph replays.
`--impl reference` times the reference's CPU path at the full config on the host cores instead (the oracle's
torch restatement; the reference's own CPU code where it has one, softmax/baseline.py), on rank 0 only.
"""

import argparse
import ctypes
import datetime
import json
import math
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
L2_BYTES = 126 * 1024 * 1024
ROW_WORKLOADS = ("softmax_4096x8192", "rmsnorm_16384x4096", "rope_8x4096", "softmax_256x262144",
                 "softmax_262144x128", "topk_512x151936")
KERNEL_OF = {"softmax_4096x8192": "sm_block", "softmax_256x262144": "sm_cluster", "softmax_262144x128": "sm_group",
             "rmsnorm_16384x4096": "rms_block_rows", "rope_8x4096": "rope_tokens", "topk_512x151936": "topk_stream"}


# ------------------------------------------------------------------------------------------------ environment ----
def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(kernel):
    """(DRAM bytes per launch, profile file) recorded from an ncu capture in profiles/ (a
    `traffic_bytes_per_launch[kernel]: N` line), or (None, None)."""
    pat = re.compile(r"traffic_bytes_per_launch\[" + re.escape(kernel) + r"\]:\s*([0-9.eE+]+)")
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None, None
    for name in sorted(os.listdir(pdir)):
        if name.endswith((".md", ".txt")):
            with open(os.path.join(pdir, name)) as f:
                m = pat.search(f.read())
            if m:
                return float(m.group(1)), "profiles/" + name
    return None, None


def cpu_info():
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"model": model, "os_cpu_count": os.cpu_count(), "torch_threads": torch.get_num_threads()}


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


def all_ranks_true(ok, world):
    if world == 1:
        return bool(ok)
    t = torch.tensor([1 if ok else 0], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


def rotation_sets(set_bytes):
    """Buffer sets to rotate so the sets together move more than twice the L2's bytes (at least 2)."""
    return max(2, math.ceil(2 * L2_BYTES / max(1, set_bytes)))


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


def workload_bytes(name, rows):
    """Algorithmic bytes of `rows` rows (tokens for RoPE) of workload `name` (the per-launch constants, weight and
    the cos/sin rows read, scale with the rows where they are per-row)."""
    if name.endswith("_bf16"):
        return workload_bytes(name[:-5], rows) // 2
    if name == "rmsnorm_16384x4096":
        return 2 * rows * 4096 * 2 + 4096 * 2
    if name == "softmax_4096x8192":
        return 2 * rows * 8192 * 4
    if name == "softmax_256x262144":
        return 2 * rows * 262144 * 4
    if name == "softmax_262144x128":
        return 2 * rows * 128 * 4
    if name == "rope_8x4096":  # q/k in place + the cos/sin rows read (at most the whole cache) + the ids
        return 2 * rows * 40 * 128 * 2 + 2 * min(rows, 4096) * 128 * 4 + rows * 8
    if name == "topk_512x151936":
        return rows * 151936 * 4 + rows * 50 * (4 + 8)
    raise SystemExit(f"unknown workload {name}")


def make_case(name, impl="ours", seeded=True, rows=None, kind="randn"):
    """Device buffers for workload `name`, `rows` rows of it (tokens for RoPE; default the full config), rotated over
    enough buffer sets to defeat the L2. seeded: the workloads module's CPU-seeded inputs (checkable against the
    oracle; full config only); otherwise the same distributions drawn on the device (faster to make)."""
    from ckb200 import workloads

    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream().cuda_stream
    half = name.endswith("_bf16")  # the softmax configs at bf16 (the reference publishes both dtypes)
    if half:
        name = name[:-5]
        seeded = False
    full_rows = workloads.ROWS[name]
    rows = full_rows if rows is None else rows
    seeded = seeded and rows == full_rows
    nbytes = workload_bytes(name, rows) // (2 if half else 1)
    sets = rotation_sets(nbytes)
    g = torch.Generator(device=dev).manual_seed(1234)

    def dev_randn(*shape, scale=1.0, dtype=torch.float32):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)

    if name == "rmsnorm_16384x4096":
        if seeded:
            base = workloads.rmsnorm_16384x4096()
            x0, w = base["x"].to(dev), base["weight"].to(dev)
        else:
            x0 = dev_randn(rows, 4096, dtype=torch.bfloat16)
            w = (1 + dev_randn(4096, scale=0.1)).to(torch.bfloat16)
        xs = [x0] + [x0.clone() for _ in range(sets - 1)]
        ys = [torch.empty_like(x0) for _ in range(sets)]
        if impl == "ours":
            fn = _lib("rmsnorm").ckb_rmsnorm_weighted_launch

            def launch(i):
                return fn(xs[i % sets].data_ptr(), w.data_ptr(), ys[i % sets].data_ptr(), rows, 4096, 1, 1, 1e-6,
                          stream)
        elif impl == "ours_noweight":
            fn = _lib("rmsnorm").launch

            def launch(i):
                return fn(xs[i % sets].data_ptr(), ys[i % sets].data_ptr(), rows, 4096, 1, 1e-6, 256, stream)
        else:
            lib = _ref_lib("rmsnorm")
            if lib is None:
                return None
            lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int, ctypes.c_int,
                                   ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
            # the reference has no weight: its unweighted kernel over the same x (the bytes differ by 8 KiB)

            def launch(i):
                return lib.launch(xs[i % sets].data_ptr(), ys[i % sets].data_ptr(), rows, 4096, 1, 1e-6, 256, stream)

        def check():
            from oracle import rmsnorm as orc
            from oracle.numerics import to_f32, ulp_distance

            xc = xs[0][:64].cpu()
            want = orc.rmsnorm(xc, w.cpu()) if impl == "ours" else orc.rmsnorm(xc)
            return int(ulp_distance(to_f32(ys[0][:64]), to_f32(want), torch.bfloat16).max()) <= 1

        return Case(name, nbytes, rows, launch, sets, check, "rms_block_rows")

    if name.startswith("softmax_"):
        cols = {"softmax_4096x8192": 8192, "softmax_256x262144": 262144, "softmax_262144x128": 128}[name]
        if seeded:
            x0 = getattr(workloads, name)()["x"].to(dev)
        else:
            scale = {"softmax_4096x8192": 2.0, "softmax_256x262144": 4.0, "softmax_262144x128": 1.0}[name]
            x0 = dev_randn(rows, cols, scale=scale, dtype=torch.bfloat16 if half else torch.float32)
        xs = [x0] + [x0.clone() for _ in range(sets - 1)]
        ys = [torch.empty_like(x0) for _ in range(sets)]
        lib = _lib("softmax") if impl == "ours" else _ref_lib("softmax")
        if lib is None:
            return None
        lib.launch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_int,
                               ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        code = 1 if half else 0

        def launch(i):
            return lib.launch(xs[i % sets].data_ptr(), ys[i % sets].data_ptr(), rows, cols, code, 256, 1024, stream)

        def check():
            from oracle import softmax as orc
            from oracle.numerics import to_f32, ulp_distance

            want = orc.softmax_f64(xs[0][:8].cpu())
            if half:  # within 1 bf16 ulp of the fp64 result rounded
                return int(ulp_distance(to_f32(ys[0][:8].cpu()), to_f32(want.to(torch.bfloat16)),
                                        torch.bfloat16).max()) <= 1
            got = ys[0][:8].cpu().double()
            return bool(((got - want).abs() <= torch.clamp(1e-6 * want.abs(), min=2.0 ** -148)).all())

        return Case(name, nbytes, rows, launch, sets, check, KERNEL_OF[name])

    if name == "rope_8x4096":
        if seeded:
            base = workloads.rope_8x4096()
            q0, k0 = base["q"].to(dev).view(1, rows, 32, 128), base["k"].to(dev).view(1, rows, 8, 128)
            cos, sin = base["cos"].to(dev), base["sin"].to(dev)
            ids = base["position_ids"].to(dev).view(1, rows)
        else:
            q0 = dev_randn(1, rows, 32, 128, dtype=torch.bfloat16)
            k0 = dev_randn(1, rows, 8, 128, dtype=torch.bfloat16)
            c, s = workloads._rope_cache(10000.0, 128, 4096, torch.float32)
            cos, sin = c.to(dev), s.to(dev)
            ids = (torch.arange(rows, device=dev) % 4096).view(1, rows)
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
                                  q.data_ptr(), k.data_ptr(), rows, 32, 8, 128, 1, 0, 40, 1, stream)
        else:  # the reference's wrapper is out of place (rope/candidate.py:50); same bytes moved
            qo = [torch.empty_like(q0) for _ in range(sets)]
            ko = [torch.empty_like(k0) for _ in range(sets)]

            def launch(i):
                q, k = qs[i % sets], ks[i % sets]
                return lib.launch(q.data_ptr(), k.data_ptr(), cos.data_ptr(), sin.data_ptr(), ids.data_ptr(),
                                  qo[i % sets].data_ptr(), ko[i % sets].data_ptr(), rows, 32, 8, 128, 1, 0, 40, 1,
                                  stream)
        return Case(name, nbytes, rows, launch, sets, None, "rope_tokens")

    if name == "topk_512x151936":
        if kind == "ascending":  # every tile beats the running top k: the overflow path on every tile
            x0 = torch.arange(151936, device=dev, dtype=torch.float32).repeat(rows, 1) + dev_randn(rows, 1)
        elif kind == "descending":  # the row's top k all in its first tile: the speculative bound fails, two passes
            x0 = -torch.arange(151936, device=dev, dtype=torch.float32).repeat(rows, 1)
        elif kind == "fewvalued":  # 8 distinct values: massive ties, resolved by index
            x0 = torch.randint(0, 8, (rows, 151936), generator=g, device=dev).float()
        else:
            x0 = workloads.topk_512x151936()["x"].to(dev) if seeded else dev_randn(rows, 151936, scale=3.0)
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
        chunk = lib.plan(rows, 151936, 0, 256, 4, 2048)
        nch = -(-151936 // chunk)
        work = torch.empty(max(1, rows * nch * 50), dtype=torch.int64, device=dev)
        counters = torch.zeros(max(4096, rows), dtype=torch.int32, device=dev)
        vals = torch.empty(rows, 50, device=dev)
        idx = torch.empty(rows, 50, dtype=torch.int64, device=dev)

        def launch(i):
            return lib.launch(xs[i % sets].data_ptr(), vals.data_ptr(), idx.data_ptr(), work.data_ptr(),
                              counters.data_ptr(), rows, 151936, 50, 0, 256, 4, chunk, stream)

        def check():
            from oracle import topk as otk

            err = launch(0)  # every set holds the same values: recompute on set 0 and compare its first rows
            torch.cuda.synchronize()
            wv, wi = otk.topk(xs[0][:16].cpu(), 50)
            return err == 0 and torch.equal(idx[:16].cpu(), wi) and torch.equal(vals[:16].cpu(), wv)

        return Case(name, nbytes, rows, launch, sets, check, "topk_stream")
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


# --------------------------------------------------------------------------------------------- end to end -------
def e2e_pipeline(name, seeded=False):
    """(pipeline, host inputs, host outputs) of workload `name` at its full config through the public API
    (ckb200.<op>): pinned host tensors, ckb200.hostpipe moving them in and out in chunks beside the kernels."""
    from ckb200 import hostpipe, rmsnorm, rope, softmax, topk, workloads

    g = torch.Generator().manual_seed(7)
    if name == "rmsnorm_16384x4096":
        base = workloads.rmsnorm_16384x4096() if seeded else None
        hx = (base["x"] if seeded else torch.randn(16384, 4096, generator=g).to(torch.bfloat16)).pin_memory()
        w = (base["weight"] if seeded else (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16)).cuda()
        pipe = hostpipe.RowPipeline(lambda x, y: rmsnorm.rmsnorm(x, w, out=y), 16384, 4096, torch.bfloat16, chunks=8)
        return pipe, [hx], [torch.empty_like(hx).pin_memory()]
    if name.startswith("softmax_"):
        shape = {"softmax_4096x8192": (4096, 8192), "softmax_256x262144": (256, 262144),
                 "softmax_262144x128": (262144, 128)}[name]
        hx = torch.randn(*shape, generator=g).pin_memory()
        pipe = hostpipe.RowPipeline(lambda x, y: softmax.softmax(x, out=y), shape[0], shape[1], torch.float32,
                                    chunks=8)
        return pipe, [hx], [torch.empty_like(hx).pin_memory()]
    if name == "rope_8x4096":
        tokens = 8 * 4096
        hq = torch.randn(tokens, 32, 128, generator=g).to(torch.bfloat16).pin_memory()
        hk = torch.randn(tokens, 8, 128, generator=g).to(torch.bfloat16).pin_memory()
        hids = (torch.arange(tokens, dtype=torch.int64) % 4096).pin_memory()
        c, s = workloads._rope_cache(10000.0, 128, 4096, torch.float32)
        cos, sin = c.cuda(), s.cuda()

        def op(ins, outs):
            q, k, ids = ins
            rope.rope(q[None], k[None], ids[None], cos, sin, out=(outs[0][None], outs[1][None]))

        pipe = hostpipe.Pipeline(op, [((tokens, 32, 128), torch.bfloat16), ((tokens, 8, 128), torch.bfloat16),
                                      ((tokens,), torch.int64)],
                                 [((tokens, 32, 128), torch.bfloat16), ((tokens, 8, 128), torch.bfloat16)], chunks=8)
        return pipe, [hq, hk, hids], [torch.empty_like(hq).pin_memory(), torch.empty_like(hk).pin_memory()]
    if name == "topk_512x151936":
        hx = (torch.randn(512, 151936, generator=g) * 3).pin_memory()

        def op(ins, outs):
            topk.topk(ins[0], 50, out=(outs[0], outs[1]))

        pipe = hostpipe.Pipeline(op, [((512, 151936), torch.float32)],
                                 [((512, 50), torch.float32), ((512, 50), torch.int64)], chunks=4)
        return pipe, [hx], [torch.empty(512, 50).pin_memory(), torch.empty(512, 50, dtype=torch.int64).pin_memory()]
    raise SystemExit(f"unknown workload {name}")


def time_e2e(name, steps, warmup, world, seeded=False):
    """End to end through the public API: every step copies the whole batch in from pinned host memory, runs the
    op and copies every output back (ckb200.hostpipe: chunks on copy-in / compute / copy-out streams). Timed by
    CUDA events from the copy-in stream's start to the copy-out stream's end, max over ranks."""
    from ckb200 import workloads

    pipe, hins, houts = e2e_pipeline(name, seeded)
    for _ in range(warmup):
        pipe(hins, houts)
    pipe.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pipe.record_start(start)
    for _ in range(steps):
        pipe(hins, houts)
    pipe.record_end(end)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    h2d, d2h = pipe.bytes_per_call()
    nbytes = workloads.ALGORITHMIC_BYTES[name]
    out = {"value": round(world * nbytes * steps / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / steps, 4),
           "pipeline": f"{len(pipe.bounds)} chunks, copy-in / compute / copy-out streams"}
    del pipe, hins, houts
    return out


def host_copy(steps, world, nbytes=128 << 20):
    """The host link's ceiling for e2e: `nbytes` pinned host -> device and `nbytes` device -> host per step on two
    streams at once (what the e2e pipeline moves), every rank at the same time; GB/s per rank (both directions'
    bytes) and aggregate, from CUDA events, max over ranks."""
    hin = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    hout = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    din = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    dout = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    for _ in range(2):
        with torch.cuda.stream(s_in):
            din.copy_(hin, non_blocking=True)
        with torch.cuda.stream(s_out):
            hout.copy_(dout, non_blocking=True)
    torch.cuda.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream()
    start.record(cur)
    s_in.wait_stream(cur)
    s_out.wait_stream(cur)
    for _ in range(steps):
        with torch.cuda.stream(s_in):
            din.copy_(hin, non_blocking=True)
        with torch.cuda.stream(s_out):
            hout.copy_(dout, non_blocking=True)
    cur.wait_stream(s_in)
    cur.wait_stream(s_out)
    end.record(cur)
    end.synchronize()
    ms = max_over_ranks(start.elapsed_time(end), world)
    per_rank = 2 * nbytes * steps / (ms * 1e-3) / 1e9
    return {"GB/s_per_rank": round(per_rank, 2), "GB/s_aggregate": round(world * per_rank, 2),
            "bytes_each_way_per_step": nbytes, "ms_per_step": round(ms / steps, 4)}


# --------------------------------------------------------------------------------------------- CPU baselines ----
def cpu_workload(name, scale=1):
    """(fn, algorithmic bytes, description) of the reference's CPU path for workload `name` at 1/scale of its rows
    (scale 1: the full config)."""
    from ckb200 import workloads
    from oracle import rmsnorm as orms
    from oracle import rope as orope
    from oracle import softmax as osm
    from oracle import topk as otk

    part = "the full config" if scale == 1 else f"1/{scale} of the rows"
    if name == "rmsnorm_16384x4096":
        inp = workloads.rmsnorm_16384x4096(scale=scale)
        x, w = inp["x"], inp["weight"]
        return (lambda: orms.rmsnorm_cpu(x, w)), 2 * x.numel() * 2 + w.numel() * 2, \
            f"{part}, x bf16 {tuple(x.shape)} + weight, torch CPU restatement (the reference has no CPU RMSNorm)"
    if name.startswith("softmax_"):
        x = getattr(workloads, name)(scale=scale)["x"]
        return (lambda: osm.softmax_cpu(x)), 2 * x.numel() * 4, \
            f"{part}, fp32 {tuple(x.shape)}, the reference's own CPU path torch.softmax (softmax/baseline.py:13)"
    if name == "rope_8x4096":
        inp = workloads.rope_8x4096(scale=scale)
        fn = lambda: orope.rope_cpu(inp["q"], inp["k"], inp["cos"], inp["sin"], inp["position_ids"])  # noqa: E731
        return fn, 2 * (inp["q"].numel() + inp["k"].numel()) * 2, \
            f"{part}, q {tuple(inp['q'].shape)} k {tuple(inp['k'].shape)} bf16, torch CPU restatement"
    x = workloads.topk_512x151936(scale=scale)["x"]
    return (lambda: otk.topk_cpu(x, 50)), x.numel() * 4, \
        f"{part}, fp32 {tuple(x.shape)}, torch CPU stable sort (the reference has no CPU top-k)"


def cpu_rate(name, reps, warmup=1, scale=1):
    """GB/s of the reference's CPU path on all host threads: `warmup` untimed then `reps` timed calls of workload
    `name` (full config by default); returns (GB/s, sample description, threads, seconds per call)."""
    torch.set_num_threads(os.cpu_count() or 1)
    fn, nbytes, what = cpu_workload(name, scale)
    for _ in range(warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    dt = time.perf_counter() - t0
    return nbytes * reps / dt / 1e9, f"{what}, {reps} calls in {dt:.2f} s", torch.get_num_threads(), dt / reps


def cpu_baseline(name, reps=2):
    gbs, sample, threads, per = cpu_rate(name, reps)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
            "ms_per_call": round(per * 1e3, 2), "cpu": cpu_info()}


def run_reference_arm(args, rank, world):
    """The reference's CPU path on the host cores at the FULL config: W warm-up and K timed steps, each step one
    call over the whole workload; rank 0 only (the other ranks exit without work)."""
    if rank != 0:
        return
    gbs, sample, threads, per = cpu_rate(args.workload, reps=args.steps, warmup=args.warmup)
    line = {"metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": _dtype(args.workload),
            "data": "synthetic (seeded, BASELINE config distributions)",
            "config": {"workload": args.workload, "sample": sample},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample, "cpu": cpu_info()},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _dtype(name):
    return {"rmsnorm_16384x4096": "bf16", "rope_8x4096": "bf16"}.get(name, "f32")


# -------------------------------------------------------------------------------------------------- main --------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", default=HEADLINE, choices=ROW_WORKLOADS)
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-kernel sweep and latency records")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baselines (profiling runs)")
    ap.add_argument("--no-multi", action="store_true", help="skip the strong / vocab / rope / host-copy records")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end record (profiling runs)")
    ap.add_argument("--sweep-steps", type=int, default=300)
    ap.add_argument("--e2e-steps", type=int, default=20)
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    rank, world, local = setup(args)
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return

    peak, peak_kind = hbm_peak()
    case = make_case(args.workload)
    ms, clocks = time_case(case, args.steps, args.warmup, world, sampler_gpu=local)
    ok = all_ranks_true(case.check() if case.check else True, world)
    gbs = world * case.bytes * args.steps / (ms * 1e-3) / 1e9
    rows_s = world * case.rows * args.steps / (ms * 1e-3)
    achieved = case.bytes / (ms / args.steps * 1e-3) / 1e9  # one launch per step
    traffic, traffic_src = ncu_traffic(case.kernel)
    del case
    torch.cuda.empty_cache()
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": _dtype(args.workload),
        "data": "synthetic (seeded, BASELINE config distributions)",
        "config": {"workload": args.workload, "rows_per_gpu": workload_rows(args.workload),
                   "parallelism": f"row-sharded x{world}",
                   "l2": "inputs larger than L2, rotated over buffer sets moving > 2x L2"},
        "rows_per_s": round(rows_s, 1), "frac_of_8tbs": round(achieved / NOMINAL_HBM_GBS, 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "traffic_source": traffic_src, "kernel": KERNEL_OF[args.workload]},
        "clocks": clocks, "gpu_launches": args.steps, "check": ok,
    }
    if not args.no_e2e:
        line["e2e"] = time_e2e(args.workload, args.e2e_steps, 3, world, seeded=True)
    if world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(args.workload)
    if world == 1 and not args.no_sweep:
        line["kernels"] = sweep(args, world)
        line["latency"] = latency()
        line["fusions"] = fusions()
    if not args.no_multi:
        line["strong"] = strong(args, rank, world)
        line["vocab_topk"] = vocab_topk(args, rank, world, local)
        line["rope_tokens"] = rope_tokens(rank, world)
        hc = host_copy(10, world)
        if "e2e" in line:
            hc["e2e_fraction"] = round(line["e2e"]["value"] / world / hc["GB/s_per_rank"] *
                                       (line["e2e"]["h2d_bytes_per_step"] + line["e2e"]["d2h_bytes_per_step"]) /
                                       workload_bytes(args.workload, workload_rows(args.workload)), 4)
        line["host_copy"] = hc
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def workload_rows(name):
    from ckb200 import workloads

    return workloads.ROWS[name]


def strong(args, rank, world):
    """Every row workload split over the ranks (rows, or tokens for RoPE, by sharded.row_range): per-rank device
    time of one launch (max over ranks), aggregate GB/s, and the speed-up over the whole config on one GPU, timed
    in the same run on every rank's GPU (max over ranks)."""
    from ckb200 import sharded, workloads

    peak, _ = hbm_peak()
    out = {}
    for name in ROW_WORKLOADS:
        full = workloads.ROWS[name]
        lo, hi = sharded.row_range(full, rank, world)
        mine = hi - lo
        rows_max = -(-full // world)
        entry = {"rows_per_gpu": rows_max}
        case = make_case(name, seeded=False, rows=mine)
        ms, _ = time_case(case, args.sweep_steps, 10, world)
        entry["sets"] = case.sets
        del case
        per = ms / args.sweep_steps
        entry["us"] = round(per * 1e3, 2)
        entry["GB/s"] = round(workload_bytes(name, full) / (per * 1e-3) / 1e9, 1)
        entry["GB/s_per_gpu_of_peak"] = round(workload_bytes(name, rows_max) / (per * 1e-3) / 1e9 / peak, 4)
        if world > 1:
            one = make_case(name, seeded=False)
            ms1, _ = time_case(one, args.sweep_steps, 10, world)
            del one
            entry["us_1gpu"] = round(ms1 / args.sweep_steps * 1e3, 2)
            entry["speedup_vs_1gpu"] = round(ms1 / ms, 3)
        torch.cuda.empty_cache()
        out[name] = entry
    return out


def vocab_topk(args, rank, world, local):
    """The vocab-sharded top-k over peer memory (PeerVocabShardedTopK): the [512, 151936] fp32 config split by
    columns over the ranks, one fused kernel per step (local top-50, lists stored into every rank's memory over
    NVLink, per-row flags, in-kernel merge). Time per step (max over ranks); the answer checked bit for bit against
    the oracle on rank 0 and the bounded waits' status checked on every rank."""
    from ckb200 import sharded, workloads

    dev = torch.device("cuda", local)
    full = workloads.topk_512x151936()["x"]
    lo, hi = sharded.col_range(full.shape[1], rank, world)
    sets = rotation_sets(512 * (hi - lo) * 4)
    shard0 = full[:, lo:hi].contiguous().to(dev)
    shards = [shard0] + [shard0.clone() for _ in range(sets - 1)]
    op = sharded.PeerVocabShardedTopK(full.shape[0], 50, device=dev)
    try:
        for i in range(args.warmup):
            op(shards[i % sets], lo)
        torch.cuda.synchronize()
        barrier(world)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for i in range(args.steps):
            values, indices = op(shards[i % sets], lo)
        end.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(start.elapsed_time(end), world)
        try:
            op.check()
            waits_ok = True
        except RuntimeError:
            waits_ok = False
        ok = True
        if rank == 0:
            from oracle import topk as otk
            wv, wi = otk.topk(full, 50)
            ok = bool(torch.equal(indices.cpu(), wi) and torch.equal(values.cpu(), wv))
        ok = all_ranks_true(ok and waits_ok, world)
    finally:
        op.close()
    per = ms / args.steps
    nbytes = workloads.ALGORITHMIC_BYTES["topk_512x151936"]
    return {"us_per_step": round(per * 1e3, 2), "GB/s": round(nbytes / (per * 1e-3) / 1e9, 1),
            "cols_per_gpu": -(-full.shape[1] // world), "check": ok, "launches_per_step": 1,
            "exchange": "fused: each rank's kernel stores its [512, 50] composite lists into every rank's memory "
                        "over NVLink (CUDA IPC), raises per-row flags and merges after bounded waits"}


def rope_tokens(rank, world, sample=512):
    """The RoPE config (q [8, 4096, 32, 128], k [8, 4096, 8, 128] bf16, in place, fp32 cos/sin cache) with its
    32768 tokens split over the ranks (sharded.token_shard): every rank rotates its shard in place and checks the
    first and last `sample` tokens of it bit for bit against the oracle; all ranks must pass."""
    from ckb200 import rope, sharded, workloads
    from oracle import rope as orope

    dev = torch.device("cuda", torch.cuda.current_device())
    base = workloads.rope_8x4096()
    q = sharded.token_shard(base["q"], rank, world)
    k = sharded.token_shard(base["k"], rank, world)
    ids = sharded.token_shard(base["position_ids"], rank, world)
    qd, kd, idd = q.to(dev), k.to(dev), ids.to(dev)
    cos, sin = base["cos"].to(dev), base["sin"].to(dev)
    rope.rope(qd, kd, idd, cos, sin, inplace=True)
    torch.cuda.synchronize()
    n = q.shape[1]
    pick = torch.cat([torch.arange(0, min(sample, n)), torch.arange(max(0, n - sample), n)]).unique()
    wq, wk = orope.rope(q[:, pick], k[:, pick], base["cos"], base["sin"], ids[:, pick])
    ok = (torch.equal(qd[:, pick].cpu().view(torch.int16), wq.view(torch.int16)) and
          torch.equal(kd[:, pick].cpu().view(torch.int16), wk.view(torch.int16)))
    lo, hi = sharded.token_range(8 * 4096, rank, world)
    return {"tokens_per_gpu": -(-8 * 4096 // world), "check": all_ranks_true(ok, world),
            "checked_tokens_per_gpu": int(pick.numel()), "first_shard": [lo, hi] if rank == 0 else None}


def sweep(args, world):
    """Every BASELINE config: ours and the reference's kernel (rebuilt for sm_100a), device time, rotated buffers;
    beside them the reference's CPU path at the full config and an end-to-end number through the public API."""
    peak, _ = hbm_peak()
    out = {}
    for name in ROW_WORKLOADS + ("softmax_4096x8192_bf16", "softmax_256x262144_bf16", "softmax_262144x128_bf16"):
        entry = {}
        impls = ("ours", "ours_noweight", "ref") if name == "rmsnorm_16384x4096" else ("ours", "ref")
        for impl in impls:
            case = make_case(name, impl=impl, seeded=False)
            if case is None:
                continue
            ms, _ = time_case(case, args.sweep_steps, 10, world)
            per = ms / args.sweep_steps
            nbytes = case.bytes - (4096 * 2 if impl != "ours" and name == "rmsnorm_16384x4096" else 0)
            gbs = nbytes / (per * 1e-3) / 1e9
            entry[impl] = {"us": round(per * 1e3, 2), "GB/s": round(gbs, 1), "frac_measured": round(gbs / peak, 4),
                           "rows_per_s": round(case.rows / (per * 1e-3), 1)}
            if impl == "ours" and case.check is not None:
                entry[impl]["check"] = bool(case.check())
            del case
            torch.cuda.empty_cache()
        if name.endswith("_bf16"):  # the fp32 entry carries the end-to-end and CPU numbers of the shape
            out[name] = entry
            continue
        if name == "topk_512x151936":
            # data-dependent paths of the streaming top-k, timed beside the reference's kernel on the same rows
            adv = {}
            for kind in ("ascending", "descending", "fewvalued"):
                adv[kind] = {}
                for impl in ("ours", "ref"):
                    case = make_case(name, impl=impl, seeded=False, kind=kind)
                    if case is None:
                        continue
                    ms, _ = time_case(case, 50, 5, world)
                    adv[kind][impl] = {"us": round(ms / 50 * 1e3, 2)}
                    if impl == "ours":
                        adv[kind][impl]["check"] = bool(case.check())
                    del case
                    torch.cuda.empty_cache()
            entry["adversarial_rows"] = adv
        entry["e2e"] = time_e2e(name, max(3, args.e2e_steps // 2), 2, world)
        torch.cuda.empty_cache()
        if not args.no_cpu:
            entry["cpu_baseline"] = cpu_baseline(name, reps=1)
        out[name] = entry
    return out


def _time_fn(fn, steps=50, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps * 1e3


def fusions():
    """The two fusions at the BASELINE shapes, each beside the unfused steps it replaces (device time per call):
    RoPE + paged KV-cache write on the RoPE config (q in place, k and v into a 2048 x 16-slot cache, k not written
    back) against this library's RoPE followed by the cache rows copied in by indexing; top-k sampling (softmax over
    the 50 largest of each [512, 151936] row, one sampled token per row) against a full-row softmax, the top-k of
    the probabilities and a renormalisation."""
    from ckb200 import rope, softmax, topk, workloads

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(9)
    out = {}
    q = torch.randn(8, 4096, 32, 128, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(8, 4096, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(8, 4096, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    c, s_ = workloads._rope_cache(10000.0, 128, 4096, torch.float32)
    cos, sin = c.to(dev), s_.to(dev)
    ids = torch.arange(4096, device=dev).repeat(8, 1)
    slots = torch.randperm(32768, generator=g, device=dev).view(8, 4096)
    kc = torch.empty(2048, 16, 8, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.empty_like(kc)
    fused = _time_fn(lambda: rope.rope_kv_cache(q, k, v, ids, cos, sin, kc, vc, slots, write_k=False))
    flat = slots.view(-1)

    def unfused():
        rope.rope(q, k, ids, cos, sin, inplace=True)
        kc.view(-1, 8, 128).index_copy_(0, flat, k.view(-1, 8, 128))
        vc.view(-1, 8, 128).index_copy_(0, flat, v.view(-1, 8, 128))

    plain = _time_fn(unfused)
    nbytes = 2 * q.numel() * 2 + 2 * (k.numel() + v.numel()) * 2 + 2 * cos.numel() * 4 + 2 * ids.numel() * 8
    out["rope_kv_cache_8x4096"] = {"fused_us": round(fused, 2), "unfused_us": round(plain, 2),
                                   "fused_GB/s": round(nbytes / (fused * 1e-6) / 1e9, 1),
                                   "unfused": "rope in place, then index_copy_ of k and v into the cache"}
    del q, k, v, kc, vc
    x = torch.randn(512, 151936, generator=g, device=dev) * 3
    u = torch.rand(512, generator=g, device=dev)
    fused = _time_fn(lambda: topk.topk_softmax(x, 50, temperature=0.8, uniforms=u))

    def unfused_tk():
        p = softmax.softmax(x / 0.8)
        vals, idx = topk.topk(p, 50)
        return vals / vals.sum(-1, keepdim=True), idx

    plain = _time_fn(unfused_tk)
    out["topk_softmax_512x151936"] = {"fused_us": round(fused, 2), "unfused_us": round(plain, 2),
                                      "fused_GB/s": round(x.numel() * 4 / (fused * 1e-6) / 1e9, 1),
                                      "unfused": "full-row softmax, top-k of the probabilities, renormalisation"}
    return out


def latency(reps=200, batch=20):
    """Decode-sized calls through the public API: `eager_us` = device time per call of `reps` back-to-back calls
    (host issue included when it is the slower side), `graph_us` = per replay of a CUDA graph holding one call,
    `graph_batched_us` = per call of a graph holding `batch` calls (the kernel plus the gap between launches)."""
    from ckb200 import rmsnorm, rope, softmax, topk, workloads

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev).manual_seed(5)
    calls = {}
    x = torch.randn(1, 128256, generator=g, device=dev) * 3
    calls["topk_1x128256_fp32_k50"] = lambda: topk.topk(x, 50)
    calls["softmax_1x128256_fp32"] = lambda: softmax.softmax(x)
    xr = torch.randn(1, 4096, generator=g, device=dev).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g, device=dev)).to(torch.bfloat16)
    calls["rmsnorm_1x4096_bf16"] = lambda: rmsnorm.rmsnorm(xr, w)
    c, s = workloads._rope_cache(10000.0, 128, 4096, torch.float32)
    cos, sin = c.to(dev), s.to(dev)
    for b in (1, 16, 64):
        q = torch.randn(b, 1, 32, 128, generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn(b, 1, 8, 128, generator=g, device=dev).to(torch.bfloat16)
        ids = torch.full((b, 1), 4095, dtype=torch.int64, device=dev)
        calls[f"rope_decode_b{b}_bf16"] = (lambda q=q, k=k, ids=ids: rope.rope(q, k, ids, cos, sin, inplace=True))
    vq = torch.randn(64, 1, 32, 128, generator=g, device=dev).to(torch.bfloat16)
    vk = torch.randn(64, 1, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    vv = torch.randn(64, 1, 8, 128, generator=g, device=dev).to(torch.bfloat16)
    vids = torch.full((64, 1), 4095, dtype=torch.int64, device=dev)
    vslots = torch.arange(64, device=dev).view(64, 1) * 16
    kcache = torch.zeros(256, 16, 8, 128, dtype=torch.bfloat16, device=dev)
    vcache = torch.zeros_like(kcache)
    calls["rope_kv_cache_decode_b64_bf16"] = lambda: rope.rope_kv_cache(vq, vk, vv, vids, cos, sin, kcache, vcache,
                                                                         vslots, write_k=False)
    us = torch.rand(1, generator=g, device=dev)
    calls["topk_softmax_sample_1x128256_fp32"] = lambda: topk.topk_softmax(x, 50, uniforms=us)
    out = {}
    for name, fn in calls.items():
        try:
            out[name] = _latency_one(fn, reps, batch)
        except RuntimeError as e:  # a call that cannot be captured is reported, not fatal to the bench
            torch.cuda.synchronize()
            out[name] = {"error": str(e).splitlines()[0][:200]}
    return out


def _latency_one(fn, reps, batch):
    if True:
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(reps):
            fn()
        end.record()
        torch.cuda.synchronize()
        eager = start.elapsed_time(end) / reps * 1e3
        res = {"eager_us": round(eager, 2)}
        for n_calls, key in ((1, "graph_us"), (batch, "graph_batched_us")):
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream().wait_stream(side)
            with torch.cuda.graph(graph):
                for _ in range(n_calls):
                    fn()
            for _ in range(5):
                graph.replay()
            torch.cuda.synchronize()
            replays = max(1, reps // n_calls)
            start.record()
            for _ in range(replays):
                graph.replay()
            end.record()
            torch.cuda.synchronize()
            res[key] = round(start.elapsed_time(end) / (replays * n_calls) * 1e3, 2)
            del graph
        return res


if __name__ == "__main__":
    main()
