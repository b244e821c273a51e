"""Benchmark: ResNet-18 bf16 inference images/s on 1..8 B200s (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

Workload ("resnet18_bf16_b256"): the config-0 ResNet-18 architecture (random
Kaiming weights, random BN statistics, BN folded by the pass pipeline), bf16
activations and weights with fp32 accumulation, B = 256 images per GPU of
3x224x224 N(0,1) synthetic input. One step = one forward of the whole batch.
Weak scaling: every rank runs its own B-image shard (batch-sharded inference,
weights replicated, no collective on the hot path).

Reported line (rank 0):
* ``value``   images/s of the whole job with inputs resident in HBM (CUDA events
  on each rank's stream, max over ranks);
* ``e2e``     the same through the public host API: every step copies its
  fp32 NCHW input from pinned host memory and reads the logits back, with the
  double-buffered ``Executable.submit`` (one slot's upload overlapping the
  other slot's forward); ``serial_value`` is the same with ``run_pinned``
  (upload, forward, read-back in sequence);
* ``roofline`` of the dominant kernel (the tcgen05 implicit-GEMM conv):
  algorithmic conv FLOPs per launch / average launch time, from CUDA events
  recorded around every conv launch in a second timed pass of the same
  forwards (the pass ``value`` is timed on carries no per-kernel events),
  against the measured bf16 tensor peak in MEASURED_PEAKS.json;
* ``cpu_baseline`` the NumPy oracle (same algorithm as the reference executor,
  single-threaded einsum) on a bounded sample of b=1 forwards.

``--impl reference`` times the reference's CPU implementation of the path (the
NumPy oracle restatement, one process per host core) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ResNet-18 images/s (b=256, 1/2/4/8 B200)"
WORKLOAD = "resnet18_bf16_b256"
# other configurations measured with the same harness (``--workload``); the
# default line is the headline metric above
WORKLOADS = {
    "resnet18_bf16_b256": ("resnet18", "bf16", 256),
    "resnet18_int8_b1024": ("resnet18", "int8", 1024),
    "resnet18_fp32_b256": ("resnet18", "fp32", 256),
    "mobilenetv2_bf16_b256": ("mobilenetv2", "bf16", 256),
    "repvit_bf16_b256": ("repvit", "bf16", 256),
}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        smax = max(float(r[2]) for r in rows)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": reasons, "samples": len(rows)}


def conv_flops(exe):
    """Algorithmic FLOPs of each conv step (2*N*OH*OW*K*C/g*R*S of the graph node,
    before any backend rewrite such as the space-to-depth stem) for one shard."""
    lo = exe.devices[0].lo
    return [lo.weights[st.params["weight"]][0]["flops"] for st in lo.steps if st.kind == "conv"]


def conv_traffic(workload):
    """DRAM bytes (read + write) per conv_tc_kernel launch of one forward of
    ``workload``, from the committed single-kernel ncu captures
    (profiles/conv_tc_<workload>_dram.json: every conv launch of one forward,
    captured three launches per ncu run), averaged over the launches; or None."""
    try:
        with open(os.path.join(ROOT, "profiles", f"conv_tc_{workload}_dram.json")) as f:
            per = json.load(f)["dram_bytes_per_launch"]
        return round(sum(per) / len(per)) if per else None
    except Exception:
        return None


def timed_steps(exe, steps):
    """`steps` forwards issued back to back between two CUDA events on the
    device stream (inputs resident); returns the elapsed ms."""
    dev = exe.devices[0]
    ctx = dev.ctx
    ctx.event_record(0)
    for _ in range(steps):
        dev.issue_forward()
    ctx.event_record(1)
    ctx.sync()
    return ctx.event_elapsed(0, 1)


def _esz(t):
    from mdlc_b200 import _lib as L
    return L.ELEM_BYTES[t]


def call_work(dev, call):
    """(kernel class, roofline bound, algorithmic bytes, algorithmic FLOPs) of one
    prepared call: bytes = every tensor the kernel must read or write, once, in
    its stored layout (weights as packed); FLOPs = 2 x MACs of the graph node."""
    from mdlc_b200 import _lib as L
    kind = call[0]
    if kind == "conv":
        _, d, x, w, b, r, y, epi, cfg = call
        ein, eout = _esz(d.in_type), _esz(d.out_type)
        xb = d.n * d.h * d.w * d.c_stride * ein
        yb = d.n * d.oh * d.ow * d.k_stride * eout
        rb = d.n * d.oh * d.ow * (d.res_stride or d.k_stride) * eout if r else 0
        wb = L.weight_bytes(d)
        flops = 2.0 * d.n * d.oh * d.ow * d.k * (d.c // d.groups) * d.r * d.s
        if d.groups == 1 and d.in_type != L.F32:
            # tensor- or HBM-bound by arithmetic intensity against the measured peaks
            peak_tf, peak_gbs, _ = _peaks()
            if flops / (xb + wb + yb + rb) >= peak_tf * 1e3 / peak_gbs:
                cls, bound = "conv_tc", "tensor"
            else:
                cls, bound = "conv_tc(hbm-bound)", "hbm"
            if d.r == 1 and d.s == 1 and d.h * d.w == 1:
                cls = "conv_tc(fc)"
        elif d.groups == 1:
            cls, bound = "conv_tc(3xtf32)", "tensor"
        elif d.groups == d.c == d.k:
            cls, bound = "conv_dw", "hbm"
        else:
            cls, bound = "conv_grouped", "hbm"
        return cls, bound, xb + wb + yb + rb, flops
    if kind == "pool":
        d = call[1]
        e = _esz(d.dtype)
        cls = {0: "maxpool", 1: "avgpool", 2: "gap"}[d.kind]
        return cls, "hbm", d.n * d.h * d.w * d.c_stride * e + d.n * d.oh * d.ow * d.c_stride * e, 0.0
    if kind == "se":
        d = call[1]
        e = _esz(d.dtype)
        # input (the pooled map, or with the squeeze fused the activations it
        # averages), gate output (n x c_stride) and both fp32 weight matrices
        nbytes = (max(d.hw, 1) + 1) * d.n * d.c_stride * e + 2 * d.rd * d.c * 4
        return "se_fc", "hbm", nbytes, 4.0 * d.n * d.rd * d.c
    if kind in ("copy", "softmax"):
        d = call[1]
        e = _esz(d.dtype)
        dims = list(d.out_dims) + [d.out_cs] if kind == "copy" else list(d.dims) + [d.cs]
        n = dims[0] * dims[2] * dims[3] * dims[4]
        return kind, "hbm", 2 * n * e, 0.0
    prog = call[1]
    e = _esz(prog.dtype)
    full = prog.n * prog.hw * prog.c_stride * e
    ins = sum({L.BC_FULL: full, L.BC_NC: prog.n * prog.c_stride * e, L.BC_C: prog.c_stride * 4,
               L.BC_SCALAR: e}[prog.bcast[i]] for i in range(prog.n_inputs))
    return "eltwise", "hbm", ins + prog.n_outputs * full, 0.0


def io_work(dev):
    """Work of the graph-boundary conversions of one forward: [(class, bytes)]."""
    lo = dev.lo
    out = []
    for name in lo.inputs:
        t = lo.tensors[name]
        n = int(np.prod(lo.shapes[name]))
        out.append(("to_s2d" if t.layout == "s2d2" else "to_nhwc", n * 4 + t.n * t.h * t.w * t.cs * _esz(t.dtype)))
    for name in lo.outputs:
        if dev.out_dev[name] is not None:
            t = lo.tensors[name]
            out.append(("to_nchw", int(np.prod(lo.shapes[name])) * 4 + t.n * t.h * t.w * t.cs * _esz(t.dtype)))
    return out


def launch_times(exe, steps):
    """A second timed pass of the same forwards with CUDA events recorded
    around every kernel launch (kept out of the region `value` is measured
    on, since the extra event records cost the stream a little). Event slots
    are finite, so at most ~2000 launches are instrumented. Returns
    (pass_ms, {class: {launches, ms, bytes, flops, bound}}, forwards)."""
    dev = exe.devices[0]
    ctx = dev.ctx
    io = io_work(dev)
    per_fwd = len(dev.calls) + len(io)
    steps = max(1, min(steps, (4000 // 2) // max(per_fwd, 1)))
    slot = 3
    marks = []   # (class, bound, bytes, flops, start slot)

    def timed(cls, bound, nbytes, flops, fn):
        nonlocal slot
        ctx.event_record(slot)
        fn()
        ctx.event_record(slot + 1)
        marks.append((cls, bound, nbytes, flops, slot))
        slot += 2

    n_in = len(dev.lo.inputs)
    ctx.event_record(0)
    for _ in range(steps):
        if n_in:   # one call converts every graph input
            timed(io[0][0], "hbm", sum(b for _, b in io[:n_in]), 0.0, dev.issue_inputs)
        for c in dev.calls:
            cls, bound, nbytes, flops = call_work(dev, c)
            if c[0] == "conv":
                _, d, x, w, b, r, y, epi, cfg = c
                timed(cls, bound, nbytes, flops, lambda: ctx.conv2d(d, x, w, b, r, y, epi, cfg))
            elif c[0] == "pool":
                timed(cls, bound, nbytes, flops, lambda: ctx.pool2d(c[1], c[2], c[3]))
            elif c[0] == "copy":
                timed(cls, bound, nbytes, flops, lambda: ctx.copy4d(c[1], c[2], c[3]))
            elif c[0] == "softmax":
                timed(cls, bound, nbytes, flops, lambda: ctx.softmax(c[1], c[2], c[3]))
            elif c[0] == "se":
                timed(cls, bound, nbytes, flops, lambda: ctx.se_fc(*c[1:]))
            else:
                timed(cls, bound, nbytes, flops, lambda: ctx.eltwise(c[1], c[2], c[3]))
        if len(io) > n_in:
            timed("to_nchw", "hbm", sum(b for _, b in io[n_in:]), 0.0, dev.issue_outputs)
        else:
            dev.issue_outputs()   # logits written by the FC epilogue: no conversion kernel
    ctx.event_record(1)
    ctx.sync()
    table = {}
    for cls, bound, nbytes, flops, a in marks:
        e = table.setdefault(cls, {"launches": 0, "ms": 0.0, "bytes": 0, "flops": 0.0, "bound": bound})
        e["launches"] += 1
        e["ms"] += ctx.event_elapsed(a, a + 1)
        e["bytes"] += nbytes
        e["flops"] += flops
    return ctx.event_elapsed(0, 1), table, steps


def kernel_table(table, pass_ms, peak_tf, peak_gbs):
    """Per kernel class: share of the instrumented pass, mean launch time, and
    the achieved rate against its roofline (TFLOP/s against the measured bf16
    tensor peak for tensor-bound classes, GB/s against the measured HBM copy
    bandwidth for memory-bound ones; both figures are given for every class)."""
    out = {}
    for cls, e in sorted(table.items(), key=lambda kv: -kv[1]["ms"]):
        s = e["ms"] / 1e3
        tf = e["flops"] / s / 1e12 if e["flops"] else 0.0
        gbs = e["bytes"] / s / 1e9
        frac = tf / peak_tf if e["bound"] == "tensor" else gbs / peak_gbs
        out[cls] = {"launches": e["launches"], "share": round(e["ms"] / pass_ms, 4),
                    "avg_launch_us": round(1e3 * e["ms"] / e["launches"], 2), "bound": e["bound"],
                    "achieved_tflops": round(tf, 1), "achieved_gbs": round(gbs, 1),
                    "frac": round(frac, 4)}
    return out


def int8_peak_tops(device):
    """Dense int8 tensor throughput measured on this GPU: torch._int_mm (a
    cuBLASLt int8 x int8 -> int32 GEMM) at 8192^3, best of 10 launches timed
    with CUDA events; the denominator for the int8 convs (the bf16 figure in
    MEASURED_PEAKS.json is measured the same way with a bf16 GEMM)."""
    import torch
    dev = torch.device("cuda", device)
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device=dev)
    for _ in range(3):
        torch._int_mm(a, b)
    best = None
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    del a, b
    torch.cuda.empty_cache()
    return round(2.0 * n ** 3 / (best / 1e3) / 1e12, 1)


def g1_graph(model):
    from mdlc_b200 import builders, passes
    return passes.default_pipeline(builders.BUILDERS[model](batch=1, seed=0))


def b1_latency(g, dtype, device, iters, calib=None):
    """b=1 forward latency (CUDA graph): p50/p99 of per-forward CUDA-event times
    with the input resident, and p50 of the host wall time of the public
    ``run_pinned`` call (pinned H2D of the image, forward, D2H of the logits)."""
    from mdlc_b200.compiler import compile as mdlc_compile
    exe = mdlc_compile(g, dtype=dtype, batch=1, devices=[device], calib=calib)
    try:
        dev = exe.devices[0]
        ctx = dev.ctx
        exe.pinned_inputs()["input"][...] = np.random.default_rng(7).standard_normal(
            (1, 3, 224, 224), dtype=np.float32)
        for _ in range(20):
            exe.run_pinned(use_graph=True)
        dev_ms, wall_ms = [], []
        for i in range(iters):
            ctx.event_record(3000)
            dev.forward(True)
            ctx.event_record(3001)
            ctx.sync()
            dev_ms.append(ctx.event_elapsed(3000, 3001))
        for i in range(iters):
            t0 = time.perf_counter()
            exe.run_pinned(use_graph=True)
            wall_ms.append(1e3 * (time.perf_counter() - t0))
        dev_ms.sort()
        return {"p50_ms": round(statistics.median(dev_ms), 4),
                "p99_ms": round(dev_ms[min(len(dev_ms) - 1, int(0.99 * len(dev_ms)))], 4),
                "p50_e2e_ms": round(statistics.median(wall_ms), 4), "iters": iters,
                "how": "CUDA graph of the whole forward; device p50/p99 from CUDA events around each "
                       "replay (input resident); e2e = host wall time of run_pinned (H2D 602112 B, "
                       "forward, D2H of the logits, sync)"}
    finally:
        exe.close()


def cpu_baseline_sample(images=8, seed=0):
    """Oracle (reference algorithm) b=1 forwards on the host; returns (img/s, seconds)."""
    from mdlc_b200 import builders, passes
    from oracle import reference as oref
    g = passes.default_pipeline(builders.resnet18(batch=1, seed=seed))
    x = np.random.default_rng(1).standard_normal((1, 3, 224, 224)).astype(np.float32)
    oref.run(g, {"input": x})   # warm-up
    t0 = time.perf_counter()
    for _ in range(images):
        oref.run(g, {"input": x})
    dt = time.perf_counter() - t0
    return images / dt, dt


_REF = {}


def _ref_worker(images):
    """One host process of the reference arm: b=1 oracle forwards (graph built once)."""
    from oracle import reference as oref
    if "g" not in _REF:
        from mdlc_b200 import builders, passes
        _REF["g"] = passes.default_pipeline(builders.resnet18(batch=1, seed=0))
        _REF["x"] = np.random.default_rng(1).standard_normal((1, 3, 224, 224)).astype(np.float32)
        oref.run(_REF["g"], {"input": _REF["x"]})
    t0 = time.perf_counter()
    for _ in range(images):
        oref.run(_REF["g"], {"input": _REF["x"]})
    return images, time.perf_counter() - t0


def run_reference_arm(args, rank, world):
    """Reference's CPU implementation of the path on all host cores."""
    if rank != 0:
        return 0
    import multiprocessing as mp
    cores = args.ref_procs or os.cpu_count() or 1
    per_proc = 2
    total_imgs, wall = 0, []
    ctx = mp.get_context("spawn")
    with ctx.Pool(cores) as pool:
        for _ in range(args.warmup):                       # imports, graph build, warm forwards
            pool.map(_ref_worker, [1] * cores, chunksize=1)
        for _ in range(args.steps):
            t0 = time.perf_counter()
            res = pool.map(_ref_worker, [per_proc] * cores, chunksize=1)
            wall.append(time.perf_counter() - t0)
            total_imgs += sum(r[0] for r in res)
    value = total_imgs / sum(wall)
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(1e3 * sum(wall) / args.steps, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "model": "resnet18", "per_step_sample": f"{cores * per_proc} images",
                       "parallelism": f"{cores} host processes"},
            "cpu_baseline": {"value": round(value, 3), "unit": "images/s", "cores": cores, "kind": "port",
                             "sample": f"{cores} processes x {per_proc} b=1 forwards per step, "
                                       f"{args.steps} steps (NumPy oracle, reference algorithm)"},
            "e2e": {"value": round(value, 3), "unit": "images/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=None, help="images per GPU (default: the workload's)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=12, help="b=1 oracle forwards for cpu_baseline")
    ap.add_argument("--workload", default=WORKLOAD, choices=sorted(WORKLOADS))
    ap.add_argument("--latency-iters", type=int, default=200, help="b=1 forwards for the p50 latency")
    ap.add_argument("--ref-procs", type=int, default=0, help="reference arm: host processes (0 = every core)")
    ap.add_argument("--requant", default="fixed", choices=["fixed", "fp32"],
                    help="int8 workloads: requantisation form of the 8-bit conv epilogues")
    ap.add_argument("--tune", default=None, metavar="CACHE",
                    help="time every tile configuration of each conv shape the cache lacks on this GPU "
                         "(mdlc_b200.tuner) and write the cache to CACHE")
    ap.add_argument("--forwards-only", action="store_true",
                    help="compile, stage the input and run --warmup forwards, then exit (no timing, no "
                         "JSON line): the program profiled by the committed ncu captures")
    args = ap.parse_args()
    if not args.forwards_only:
        args.warmup = max(args.warmup, 3)

    from mdlc_b200 import dist as mdist
    dist = mdist.from_env()
    rank, world, local = dist.rank, dist.world, dist.local_rank

    if args.impl == "reference":
        rc = run_reference_arm(args, rank, world)
        dist.close()
        return rc

    from mdlc_b200 import builders, passes
    from mdlc_b200.compiler import compile as mdlc_compile

    model, dtype, default_batch = WORKLOADS[args.workload]
    if args.batch is None:
        args.batch = default_batch
    g = passes.default_pipeline(builders.BUILDERS[model](batch=args.batch, seed=0))
    kw = {"requant": args.requant} if dtype == "int8" else {}
    if args.tune:
        from mdlc_b200 import _lib as L
        from mdlc_b200 import tuner as T
        tctx = L.Context(local)
        cache = T.TuneCache(args.tune)
        kw["tuner"] = T.Tuner(cache, ctx=tctx)
    exe = mdlc_compile(g, dtype=dtype, devices=[local], **kw)
    if args.tune:
        cache.save()
        tctx.close()
    dev = exe.devices[0]
    ins, outs = exe.pinned_inputs(), exe.pinned_outputs()
    rng = np.random.default_rng(1234 + rank)
    ins["input"][...] = rng.standard_normal(ins["input"].shape, dtype=np.float32)
    exe.run_pinned()                       # stage the input once (resident for `value`)
    flops = conv_flops(exe)

    barrier, max_over_ranks = dist.barrier, dist.max

    # ---- warm-up
    for _ in range(args.warmup):
        dev.issue_forward()
    exe.sync()
    if args.forwards_only:
        if rank == 0:
            print(f"forwards-only: {args.workload} b={args.batch}, {1 + args.warmup} forwards of "
                  f"{exe.launches_per_forward()} launches each", flush=True)
        exe.close()
        dist.close()
        return 0

    # ---- timed: device-resident inputs
    barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    launches0 = dev.ctx.launch_count()
    total_ms = timed_steps(exe, args.steps)
    launches = dev.ctx.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    barrier()
    total_ms = max_over_ranks(total_ms)
    ms_per_step = total_ms / args.steps
    value = world * args.batch / (ms_per_step / 1e3)

    # ---- per-kernel CUDA events for the roofline (a second timed pass)
    barrier()
    inst_ms, ktable, inst_steps = launch_times(exe, args.steps)
    barrier()

    # ---- e2e through the public host API: every step uploads its fp32 input
    # from pinned host memory and reads its logits back. Serial form: one
    # run_pinned per step. Serving form: double-buffered submit(slot), the
    # upload of one slot (copy stream) overlapping the other slot's forward.
    from mdlc_b200 import _lib as L
    for _ in range(2):
        exe.run_pinned()
    barrier()
    dev.ctx.event_record(2)
    for _ in range(args.steps):
        exe.run_pinned(sync=False)
    dev.ctx.event_record(3)
    exe.sync()
    serial_ms = max_over_ranks(dev.ctx.event_elapsed(2, 3)) / args.steps
    exe.pinned_inputs(slot=1)["input"][...] = ins["input"]
    for _ in range(2):
        exe.submit(0)
        exe.submit(1)
    exe.sync()
    barrier()
    dev.ctx.event_record(2, L.STREAM_COPY)
    t0 = time.perf_counter()
    for i in range(args.steps):
        exe.submit(i % 2)
    dev.ctx.event_record(3)
    exe.sync()
    e2e_wall = time.perf_counter() - t0
    e2e_ms = max_over_ranks(dev.ctx.event_elapsed(2, 3)) / args.steps
    barrier()
    e2e_value = world * args.batch / (e2e_ms / 1e3)
    logits = exe.wait(0)["logits"]
    assert np.isfinite(logits).all() and np.isfinite(exe.wait(1)["logits"]).all()

    # ---- the whole job on the wall clock: from a common start (barrier) to
    # every rank's logits gathered, per step: pinned H2D of the shard's
    # images, forward, D2H of its logits, all-gather of all ranks' logits
    exe.run_pinned()
    dist.gather(outs["logits"])
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        exe.run_pinned()
        gathered = dist.gather(outs["logits"])
    job_s = max_over_ranks(time.perf_counter() - t0)
    assert gathered.shape[0] == world * args.batch
    barrier()

    latency = None
    if rank == 0 and args.latency_iters > 0:
        latency = b1_latency(g1_graph(model), dtype, local, args.latency_iters,
                             calib=getattr(exe, "ranges", None))

    if rank == 0:
        peak_tf, _, peak_kind = _peaks()
        if dtype == "int8":
            peak_tf, peak_kind = int8_peak_tops(local), "measured in this run (torch._int_mm) int8"
        elif dtype == "fp32":
            # 3xTF32: three tf32 MMAs per fp32 product, each at half the bf16 rate
            peak_tf, peak_kind = round(peak_tf / 6, 1), f"{peak_kind} bf16 / 6 (3xTF32 ceiling)"
        conv_flops_step = sum(flops)
        tc = [e for k, e in ktable.items() if k.startswith("conv_tc")]
        conv_ms = sum(e["ms"] for e in tc)
        nconv = sum(e["launches"] for e in tc)
        avg_launch_ms = conv_ms / nconv
        achieved_tf = (sum(e["flops"] for e in tc) / nconv) / (avg_launch_ms / 1e3) / 1e12
        _, peak_gbs, _ = _peaks()
        kernels = kernel_table(ktable, inst_ms, peak_tf, peak_gbs)
        cpu = None
        if world == 1 and args.cpu_sample > 0 and model == "resnet18":
            ips, dt = cpu_baseline_sample(args.cpu_sample)
            cpu = {"value": round(ips, 4), "unit": "images/s", "cores": 1, "kind": "port",
                   "sample": f"{args.cpu_sample} ResNet-18 b=1 forwards ({dt:.1f} s), NumPy oracle "
                             "(reference algorithm: im2col + single-threaded einsum)"}
        in_bytes = int(np.prod(g.value_info["input"].shape)) * 4
        line = {
            "metric": METRIC if args.workload == WORKLOAD else f"{model} {dtype} images/s",
            "value": round(value, 1), "unit": "images/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": {"bf16": "bf16", "fp32": "f32", "int8": "u8 x s8 -> s32"}[dtype],
            "data": "synthetic (N(0,1) 3x224x224 images, random Kaiming weights)",
            "config": {"workload": args.workload, "model": model, "per_gpu_batch": args.batch,
                       **({"requant": args.requant} if dtype == "int8" else {}),
                       "global_batch": args.batch * world, "image": 224, "parallelism": f"dp{world}",
                       "l2": "working set > 126 MB L2 (input 154 MB fp32 + activations), no flush needed"},
            "e2e": {"value": round(e2e_value, 1), "unit": "images/s", "h2d_bytes_per_step": in_bytes,
                    "d2h_bytes_per_step": int(np.prod(logits.shape)) * 4,
                    "wall_s": round(e2e_wall, 4),
                    "api": "Executable.submit(slot) double-buffered: pinned H2D on the copy stream "
                           "overlapping the other slot's forward, D2H of the logits every step",
                    "serial_value": round(world * args.batch / (serial_ms / 1e3), 1),
                    "serial_api": "Executable.run_pinned per step (H2D, forward, D2H in sequence)"},
            "latency_b1": latency,
            "roofline": {"kernel": "conv_tc_kernel (tcgen05 implicit GEMM)", "bound": "tensor",
                         "achieved": round(achieved_tf, 1),
                         "peak": peak_tf, "unit": "TFLOP/s", "frac": round(achieved_tf / peak_tf, 4),
                         "peak_kind": peak_kind if dtype != "bf16" else f"{peak_kind} bf16 (burst)", "traffic": conv_traffic(args.workload),
                         "traffic_unit": "bytes per launch (ncu dram read+write)",
                         "conv_share_of_step": round(conv_ms / inst_ms, 4) if inst_ms else None,
                         "flops_per_launch": round(conv_flops_step / len(flops)),
                         "algorithmic_bytes_per_launch": round(sum(e["bytes"] for e in tc) / nconv),
                         "avg_launch_ms": round(avg_launch_ms, 5),
                         "how": f"CUDA events around each of the {nconv} conv launches of {inst_steps} "
                                "forwards, in a timed pass after the one `value` is measured on"},
            "kernels": kernels,
            "kernels_how": f"per kernel class over {inst_steps} forwards of the instrumented pass: share of "
                           "that pass, mean launch time, achieved TFLOP/s (algorithmic FLOPs of the graph "
                           "nodes) and GB/s (algorithmic bytes: each tensor read or written once in its "
                           "stored layout); frac against the measured bf16 tensor peak for tensor-bound "
                           f"classes, the measured HBM copy bandwidth ({peak_gbs} GB/s) for the others",
            "job": {"value": round(world * args.batch * args.steps / job_s, 1), "unit": "images/s",
                    "ms_per_step": round(1e3 * job_s / args.steps, 4),
                    "how": "host wall clock, max over ranks, from a common start (barrier) over "
                           f"{args.steps} steps of: pinned H2D of each rank's {args.batch} images, forward, "
                           "D2H of its logits, all-gather of every rank's logits (the final output "
                           "gather); no overlap between steps"},
            "gpu_launches": launches,
            "network_tflops": round(world * conv_flops_step / (ms_per_step / 1e3) / 1e12, 1),
        }
        if clocks:
            line["clocks"] = clocks
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    exe.close()
    dist.barrier()
    dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
