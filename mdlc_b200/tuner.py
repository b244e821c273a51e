"""Per-shape autotuning of the tensor-core conv kernel's tile configuration.

Restates the reference autotuner's contract (``mdlc/autotuner/tuner.py:60-174``:
a schedule search per GEMM shape with a JSON cache, measured on a GPU when
one is available, an analytical cost model otherwise) for the B200 kernels:
the search space is the conv kernel's tile width ``bn`` (64/128/256 output
channels per CTA) and shared-memory pipeline depth ``stages`` — the only
knobs of the prebuilt kernel; the shallow (64, 3) and (128, 2) pipelines fit
two CTAs on one SM — and the cache key is
``(kind, n, h, w, c, k, r, s, stride, pad, dtype, arch)``.

``Tuner`` is passed to :func:`mdlc_b200.compile` as ``tuner=`` (the
reference's ``schedule_fn`` hook, ``mdlc/codegen/cuda/emit.py:27,100``).

As a module it is also the single-layer microbenchmark used for profiling:

    python -m mdlc_b200.tuner --layer N,C,H,W,K,R,S,STRIDE,PAD [--cfg BN,STAGES] [--iters 20]
"""

from __future__ import annotations

import argparse
import json
import os
from dataclasses import dataclass

import numpy as np

from mdlc_b200 import _lib as L

CONFIGS = ((64, 3), (128, 2), (256, 3), (192, 3), (64, 8), (128, 4))
# fp32 (3xTF32) keeps hi and lo stages: its own tile set
CONFIGS_F32 = ((64, 3), (64, 4), (128, 2), (128, 3), (256, 2))
KERNEL_TAG = "conv_tc_v3"
# resident CTAs per SM of each bf16 / 8-bit configuration (shared memory <= 113 KB:
# two); every fp32 (3xTF32) configuration runs one (hi, lo and weight stages)
CTAS_PER_SM = {(64, 3): 2, (128, 2): 2, (256, 3): 1, (192, 3): 1, (64, 8): 1, (128, 4): 1, (256, 2): 1, (64, 4): 1,
               (128, 3): 1}
# Cost-model constants, fitted to B200 measurements of this kernel (b=256
# ResNet-18 layers, CUDA events): tensor-pipe cycles of one 128 x bn x 16 bf16
# MMA with operands fresh from the stage ring; the cycles one CTA's issuing
# thread adds per k-block for narrow tiles (barrier waits, commits, operand
# hand-offs: 64-wide 819 and 128-wide 867 cycles per k-block against 252 / 256
# of MMAs), which a second resident CTA overlaps; and the operand load latency
# that bounds an SM's L2 -> shared-memory bandwidth to the bytes its stage
# rings hold in flight (Little's law), up to a sustained maximum.
MMA_CYCLES = {64: 63.0, 128: 64.0, 192: 96.0, 256: 128.0}


def configs_for(dtype) -> tuple:
    return CONFIGS_F32 if dtype == L.F32 else CONFIGS
ISSUE_GAP = 560.0
LOAD_LATENCY = 2700.0
L2_MAX_BYTES_PER_CYCLE = 64.0


def round_up(v, m):
    return (v + m - 1) // m * m


@dataclass(frozen=True)
class ConvShape:
    n: int
    c: int
    h: int
    w: int
    k: int
    r: int
    s: int
    stride: int
    pad: int
    dtype: int = L.BF16

    @property
    def oh(self):
        return (self.h + 2 * self.pad - self.r) // self.stride + 1

    @property
    def ow(self):
        return (self.w + 2 * self.pad - self.s) // self.stride + 1

    def key(self) -> str:
        return (f"conv:{self.n}x{self.c}x{self.h}x{self.w}->{self.k}:{self.r}x{self.s}"
                f"/s{self.stride}p{self.pad}:dt{self.dtype}:{KERNEL_TAG}")

    def desc(self) -> L.ConvDesc:
        esz8 = self.dtype in (L.U8, L.S8)
        a = 16 if esz8 else 8
        return L.ConvDesc(n=self.n, h=self.h, w=self.w, c=self.c, c_stride=round_up(self.c, a), k=self.k,
                          k_stride=round_up(self.k, a), r=self.r, s=self.s, stride_h=self.stride,
                          stride_w=self.stride, pad_t=self.pad, pad_l=self.pad, dil_h=1, dil_w=1,
                          oh=self.oh, ow=self.ow, groups=1, in_type=self.dtype,
                          out_type=self.dtype if not esz8 else L.F32)

    def flops(self) -> float:
        return 2.0 * self.n * self.oh * self.ow * self.k * self.c * self.r * self.s

    def bytes(self) -> float:
        esz = L.ELEM_BYTES[self.dtype]
        d = self.desc()
        return (self.n * self.h * self.w * d.c_stride + self.n * self.oh * self.ow * d.k_stride
                + self.k * self.r * self.s * d.c_stride) * esz


def analytical_cost(shape: ConvShape, bn: int, stages: int, num_sms: int = 148) -> float:
    """Estimated SM cycles without a device. Per k-block an SM is bound by its
    MMA issue (4 MMAs plus the issuer's gap for narrow tiles, overlapped by as
    many issuers as CTAs share the SM), by the tensor pipe, or by the L2 -> SM
    operand bytes (A and B tiles) at the bandwidth its in-flight stages
    sustain; the busiest SM gets ``ceil(tiles /
    num_sms)`` tiles, and with one tile per SM the pipeline's fill latency
    shows."""
    d = shape.desc()
    m = shape.n * shape.oh * shape.ow
    tiles = -(-m // 128) * -(-d.k_stride // bn)
    kb = -(-shape.r * shape.s * d.c_stride // (128 // L.ELEM_BYTES[shape.dtype]))
    occ = 1 if shape.dtype == L.F32 else CTAS_PER_SM.get((bn, stages), 1)
    per_sm = -(-tiles // num_sms)
    conc = min(occ, per_sm)               # CTAs of this configuration busy on one SM
    issue = 4 * MMA_CYCLES[bn] + (ISSUE_GAP if bn <= 128 else 0.0)
    pipe = max(issue / conc, 4 * MMA_CYCLES[bn])
    stage_bytes = 128 * 128 + bn * 128
    bw = min(L2_MAX_BYTES_PER_CYCLE, conc * stages * stage_bytes / LOAD_LATENCY)
    per_kb = max(pipe, stage_bytes / bw)
    latency = 1.0 + 1.0 / stages if per_sm == 1 else 1.0   # one tile per SM: nothing overlaps its fill
    return per_sm * kb * per_kb * latency


class _Bench:
    """Device buffers for timing one conv shape."""

    def __init__(self, ctx: L.Context, shape: ConvShape, seed=0):
        self.ctx, self.shape = ctx, shape
        d = shape.desc()
        self.d = d
        rng = np.random.default_rng(seed)
        w = (rng.standard_normal((shape.k, shape.c, shape.r, shape.s)) * 0.05).astype(np.float32)
        if shape.dtype in (L.U8, L.S8):
            w = np.clip(np.rint(w * 2000), -127, 127).astype(np.float32)
        self.w = ctx.to_device(L.pack_weights(d, w))
        esz = L.ELEM_BYTES[shape.dtype]
        xb = shape.n * shape.h * shape.w * d.c_stride * esz
        self.x = ctx.alloc(xb)
        ctx.memset(self.x, 0x11, xb)
        ob = 4 if d.out_type == L.F32 else L.ELEM_BYTES[d.out_type]
        self.y = ctx.alloc(shape.n * shape.oh * shape.ow * d.k_stride * ob)
        if shape.dtype in (L.U8, L.S8):
            self.b = ctx.to_device(np.zeros(d.k_stride, np.int32))
            self.scale = ctx.to_device(np.full(d.k_stride, 1e-3, np.float32))
            self.epi = L.Epilogue(act=L.ACT_NONE, deq_scale=self.scale)
        else:
            self.b = ctx.to_device(np.zeros(d.k_stride, np.float32))
            self.epi = L.Epilogue(act=L.ACT_RELU)

    def run(self, cfg):
        self.ctx.conv2d(self.d, self.x, self.w, self.b, 0, self.y, self.epi, cfg)

    def time_ms(self, bn=0, stages=0, iters=20, warmup=3) -> float:
        cfg = L.TileCfg(bn=bn, stages=stages, flags=0) if bn else None
        for _ in range(warmup):
            self.run(cfg)
        self.ctx.sync()
        self.ctx.event_record(0)
        for _ in range(iters):
            self.run(cfg)
        self.ctx.event_record(1)
        self.ctx.sync()
        return self.ctx.event_elapsed(0, 1) / iters

    def close(self):
        for p in (self.w, self.x, self.y, self.b):
            self.ctx.free(p)
        if hasattr(self, "scale"):
            self.ctx.free(self.scale)


class TuneCache:
    """JSON cache of the best configuration per shape key (``tuner.py:60-90``)."""

    def __init__(self, path: str | None = None):
        self.path = path or os.path.join(os.path.dirname(os.path.abspath(__file__)), "tune_cache.json")
        self.entries = {}
        if os.path.exists(self.path):
            with open(self.path) as f:
                self.entries = json.load(f)

    def get(self, key):
        e = self.entries.get(key)
        return tuple(e["cfg"]) if e else None

    def put(self, key, cfg, metric, measured):
        self.entries[key] = {"cfg": list(cfg), "metric": metric, "measured": measured}

    def save(self):
        with open(self.path, "w") as f:
            json.dump(self.entries, f, indent=1, sort_keys=True)


def tune(shape: ConvShape, ctx: L.Context | None = None, iters: int = 10):
    """Best (bn, stages) for ``shape``: measured on ``ctx`` if given, else modeled."""
    ranking = []
    if ctx is None:
        for bn, st in configs_for(shape.dtype):
            ranking.append(((bn, st), analytical_cost(shape, bn, st)))
    else:
        bench = _Bench(ctx, shape)
        try:
            for bn, st in configs_for(shape.dtype):
                try:
                    ranking.append(((bn, st), bench.time_ms(bn, st, iters=iters)))
                except L.MdlcError as e:
                    if e.status in (L.ERR_DEVICE, L.ERR_CUDA):
                        raise          # a kernel fault or timeout is a bug, not a slow config
                    continue
        finally:
            bench.close()
    ranking.sort(key=lambda t: t[1])
    return ranking[0][0], ranking[0][1], ranking


class Tuner:
    """Cache-backed tile-config oracle, callable as ``tuner(kind, geom)``.

    A shape in the cache gets its cached configuration. Otherwise: with a
    context, every configuration is timed on the device and the best cached;
    without one, the cost model ranks them (``model=True``) or the library's
    own heuristic decides (``None`` is returned)."""

    def __init__(self, cache: TuneCache | None = None, ctx: L.Context | None = None, iters: int = 10,
                 model: bool = True):
        self.cache = cache or TuneCache()
        self.ctx = ctx
        self.iters = iters
        self.model = model

    def __call__(self, kind, geom):
        if kind != "conv" or geom.get("groups", 1) != 1:
            return None
        if geom["dh"] != 1 or geom["sh"] != geom["sw"] or geom["pt"] != geom["pl"]:
            return None
        shape = ConvShape(geom["n"], geom["c"], geom["h"], geom["w"], geom["k"], geom["r"], geom["s"],
                          geom["sh"], geom["pt"], geom.get("dtype", L.BF16))
        cached = self.cache.get(shape.key())
        if cached:
            return cached
        if self.ctx is None and not self.model:
            return None
        cfg, metric, _ = tune(shape, self.ctx, self.iters)
        self.cache.put(shape.key(), cfg, metric, self.ctx is not None)
        return cfg


TILE_WIDTHS = (64, 128, 192, 256)


def from_reference_schedule(schedule_fn, node, geom):
    """Tile choice for one conv from the reference's schedule hook.

    The reference codegen calls ``schedule_fn(node, (M, N, K))``
    (``mdlc/codegen/cuda/emit.py:27,100``; ``autotuner/tuner.py:164-174``'s
    ``Tuner`` is such a callable) and tiles its GEMM with the returned
    ``GemmSchedule`` (``mdlc/codegen/schedule.py:16-31``: ``BM x BN`` block
    tile). Here the hook is called with the same (M, N, K) for the same node
    (conv: (OC, OH*OW, C/g*KH*KW); Gemm / MatMul: (rows, out features, in
    features)), and the schedule's tile along the output-channel axis (``BM``
    for a conv, where the reference puts output channels on M; ``BN`` for a
    GEMM) picks this kernel's tile width ``bn``: the smallest of 64 / 128 / 192
    / 256 that covers it. The pipeline depth stays the library's choice for
    that width. A hook returning a ``(bn, stages)`` tuple sets both directly;
    ``None`` keeps the defaults. Returns ``(bn, stages)`` or None."""
    sched = schedule_fn(node, tuple(geom["ref_mnk"]))
    if sched is None:
        return None
    if isinstance(sched, tuple):
        return int(sched[0]), int(sched[1])
    width = int(getattr(sched, "BM" if geom["ref_channel_axis"] == "M" else "BN"))
    bn = next((w for w in TILE_WIDTHS if w >= width), TILE_WIDTHS[-1])
    return bn, 0


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--layer", required=True, help="N,C,H,W,K,R,S,STRIDE,PAD")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "u8", "s8"])
    ap.add_argument("--cfg", default=None, help="BN,STAGES (default: library heuristic)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--tune", action="store_true", help="time every configuration")
    args = ap.parse_args()
    n, c, h, w, k, r, s, st, pad = (int(v) for v in args.layer.split(","))
    dt = {"bf16": L.BF16, "u8": L.U8, "s8": L.S8}[args.dtype]
    shape = ConvShape(n, c, h, w, k, r, s, st, pad, dt)
    ctx = L.Context(0)
    if args.tune:
        best, ms, ranking = tune(shape, ctx, args.iters)
        for cfg, t in ranking:
            print(f"{cfg}: {t * 1e3:.1f} us  {shape.flops() / t / 1e9:.1f} TFLOP/s")
        print(f"best {best}")
        return 0
    b = _Bench(ctx, shape)
    bn, stg = (int(v) for v in args.cfg.split(",")) if args.cfg else (0, 0)
    ms = b.time_ms(bn, stg, iters=args.iters)
    print(json.dumps({"layer": shape.key(), "cfg": [bn, stg], "us": round(ms * 1e3, 2),
                      "tflops": round(shape.flops() / ms / 1e9, 1),
                      "gbs": round(shape.bytes() / ms / 1e6, 1)}))
    b.close()
    ctx.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())

