"""INT8 quantisation for the backend's int8 executables.

The reference has no quantised operators (``DType.INT8`` exists only as a type,
``mdlc/ir/tensor.py:29``; "INT8/DP4A path not started", ``docs/GAPS.md:128``), so
this module defines the scheme: gemmlowp / TFLite-style asymmetric uint8
activations and symmetric per-channel int8 weights, with fbgemm-style fp32
requantisation (published methods):

* activations: per-tensor asymmetric uint8, ``q = clamp(rint(x / s) + zp, 0, 255)``
  with ``s = (max(hi, 0) - min(lo, 0)) / 255`` and ``zp = rint(-min(lo, 0) / s)``,
  ranges calibrated on seeded N(0, 1) batches run through the backend's own fp32
  executable; the network input is symmetric int8 instead
  (``s = max(|lo|, |hi|) / 127``, zero point 0, ``q = clamp(rint(x / s), -128, 127)``)
  so that the first conv's padded taps are real zeros;
* weights: per-output-channel symmetric int8, ``s_w[k] = max|w[k]| / 127``,
  ``w_q = clamp(rint(w / s_w), -127, 127)``;
* conv / GEMM: int32 accumulation ``acc = sum(x_q * w_q)`` with padded taps reading
  the input zero point, ``bias32 = rint(b / (s_x s_w)) - zp_x * sum(w_q)``, then
  ``f = float32(acc + bias32) * r[k] [+ float32(res_q - zp_r) * r_res]`` with
  ``r[k] = float32(s_x s_w[k] / s_y)``, ``r_res = float32(s_r / s_y)``, each product
  and sum rounded once in IEEE float32 (no fused multiply-add), and
  ``y_q = zp_y + clamp(rint(f), qmin - zp_y, qmax - zp_y)`` (round half to even);
  the activation (ReLU / ReLU6) is the clamp. A layer with fp32 output (the
  logits) computes ``y = act(float32(acc + bias32) * float32(s_x s_w[k]) + float32(b[k])
  [+ float32(res_q - zp_r) * s_r])`` in the same float32 arithmetic;
* max pooling works on the codes (output keeps the input's scale and zero point);
  global average pooling requantises ``sum(q - zp_in)`` by ``s_in / (H W s_out)`` in
  gemmlowp fixed point (SaturatingRoundingDoublingHighMul + RoundingDivideByPOT).

Bit-exactness is defined against the integer NumPy restatement in the test
oracle, which consumes the same :class:`QuantPlan`.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

from mdlc_b200 import _lib as L
from mdlc_b200 import lowering


def act_qparams(lo: float, hi: float):
    """(scale, zero_point) of a per-tensor asymmetric uint8 quantiser for [lo, hi]."""
    lo, hi = min(float(lo), 0.0), max(float(hi), 0.0)
    scale = np.float32((hi - lo) / 255.0) if hi > lo else np.float32(1.0)
    zp = int(np.clip(np.rint(-lo / float(scale)), 0, 255))
    return scale, zp


def sym_qparams(lo: float, hi: float):
    """(scale, 0) of a per-tensor symmetric int8 quantiser for [lo, hi]."""
    amax = max(abs(float(lo)), abs(float(hi)))
    return (np.float32(amax / 127.0) if amax > 0 else np.float32(1.0)), 0


def quantize_multiplier(real: float):
    """gemmlowp / TFLite QuantizeMultiplier: real = M * 2^-(31 + shift) with M in
    [2^30, 2^31). ``shift > 0`` is a right shift after the high multiply,
    ``shift < 0`` a left shift of the input before it (saturated to int32)."""
    if real <= 0.0:
        return 0, 0
    m, e = math.frexp(real)          # real = m * 2^e, m in [0.5, 1)
    q = int(round(m * (1 << 31)))
    if q == (1 << 31):
        q //= 2
        e += 1
    shift = -e
    if shift > 31:                   # below int32 resolution: the term is zero
        return 0, 0
    if shift < -30:
        raise ValueError(f"requantisation multiplier {real} out of range")
    return q, shift


def shared_shift_multipliers(real_acc, real_res=None):
    """Per-channel fixed-point multipliers for ``t = (acc * M1 + r * M2 + 2^(S-1)) >> S``
    (the single-rounding form of TFLite's MultiplyByQuantizedMultiplier, with
    the residual term sharing the channel's shift so the sum is rounded once).

    For channel k, S[k] = 31 - e with m = max(real_acc[k], real_res) = f * 2^e,
    f in [0.5, 1): the larger multiplier gets 31 significant bits
    (M in [2^30, 2^31)), the other as many as its ratio to the larger allows.
    Returns int32 arrays (M1, M2, S); S is clamped to 62 (a multiplier below
    2^-31 then rounds to 0)."""
    real_acc = np.asarray(real_acc, np.float64)
    rr = 0.0 if real_res is None else float(real_res)
    k = real_acc.shape[0]
    m1, m2, sh = np.zeros(k, np.int64), np.zeros(k, np.int64), np.zeros(k, np.int64)
    for i in range(k):
        big = max(float(real_acc[i]), rr)
        if big <= 0.0:
            sh[i] = 31
            continue
        _, e = math.frexp(big)
        S = 31 - e
        if S < 1:
            raise ValueError(f"requantisation multiplier {big} too large for the fixed-point form")
        S = min(S, 62)
        a = int(round(float(real_acc[i]) * 2.0 ** S))
        b = int(round(rr * 2.0 ** S))
        if max(a, b) >= (1 << 31):      # rounded up to 2^31: one bit less
            S -= 1
            a = int(round(float(real_acc[i]) * 2.0 ** S))
            b = int(round(rr * 2.0 ** S))
        m1[i], m2[i], sh[i] = a, b, S
    return m1.astype(np.int32), m2.astype(np.int32), sh.astype(np.int32)


@dataclass
class ConvQ:
    """Quantisation of one conv step (keyed by its weight name)."""

    x: str
    y: str
    residual: str | None
    w_q: np.ndarray          # int8 codes as float32 OIHW (backend geometry, e.g. space-to-depth)
    w_q_orig: np.ndarray     # int8 codes, OIHW of the graph node (for the oracle)
    s_w: np.ndarray          # float32 [k]
    bias32: np.ndarray       # int32 [k]
    rq_scale: np.ndarray     # float32 [k] s_x s_w[k] / s_y (8-bit output)
    qmin: int = 0
    qmax: int = 255
    res_scale: float = 0.0   # float32 residual scale: s_r / s_y (8-bit output), s_r (fp32 output)
    deq_scale: np.ndarray | None = None   # float32 [k] (fp32 output)
    deq_bias: np.ndarray | None = None    # float32 [k] (fp32 output)
    rq_mult: np.ndarray | None = None     # int32 [k] fixed-point accumulator multipliers (8-bit output)
    rq_res_mult: np.ndarray | None = None # int32 [k] residual multipliers (same shift)
    rq_shift: np.ndarray | None = None    # int32 [k] right shifts
    act: str | None = None
    nodes: list = field(default_factory=list)


@dataclass
class QuantPlan:
    tensors: dict            # activation name -> (scale float32, zero point int)
    convs: dict              # weight name -> ConvQ
    gap: dict                # output name -> (mult, shift, in_zp, out_zp)
    steps: list              # lowered steps (names, grouping), shared with the oracle
    signed: set = field(default_factory=set)   # tensors holding signed int8 codes
    requant: str = "fixed"   # 8-bit conv outputs: "fixed" (integer multiplier + shift) or "fp32"


def _act_range(act, attrs, s_y, zp_y):
    if act in (None, "Identity"):
        return 0, 255
    if act == "Relu":
        return zp_y, 255
    if act in ("Clip", "Relu6"):
        lo = attrs.get("clip_min", 0.0 if act == "Relu6" else None)
        hi = attrs.get("clip_max", 6.0 if act == "Relu6" else None)
        qlo = 0 if lo is None else int(np.clip(zp_y + np.rint(lo / float(s_y)), 0, 255))
        qhi = 255 if hi is None else int(np.clip(zp_y + np.rint(hi / float(s_y)), 0, 255))
        return qlo, qhi
    raise lowering.LoweringError(f"int8: activation {act!r} has no integer epilogue")


def build_plan(lo_f32, lo_i8, ranges: dict, graph, requant: str = "fixed") -> QuantPlan:
    """Quantisation plan for the int8 lowering ``lo_i8`` of ``graph``.

    ``ranges`` maps activation tensor names to (min, max) observed in fp32;
    ``lo_f32`` supplies the unrewritten fp32 weights of each step.
    """
    tensors, signed = {}, set()
    for name in lo_i8.inputs:
        if lo_i8.tensors[name].dtype == L.S8:
            tensors[name] = sym_qparams(*ranges[name])
            signed.add(name)
        else:
            tensors[name] = act_qparams(*ranges[name])
    convs, gap = {}, {}
    for st in lo_i8.steps:
        y = st.outputs[0]
        if st.kind == "pool":
            src = lo_i8.tensors[st.inputs[0]]
            src_name = src.alias_of or src.name
            s_in, zp_in = tensors[src_name] if src_name in tensors else tensors[st.inputs[0]]
            if st.params["kind"] == 0:
                tensors[y] = (s_in, zp_in)          # max commutes with the monotone code map
            elif st.params["kind"] == 2:
                s_out, zp_out = act_qparams(*ranges[y])
                tensors[y] = (s_out, zp_out)
                hw = src.h * src.w
                m, sh = quantize_multiplier(float(s_in) / (hw * float(s_out)))
                gap[y] = (m, sh, zp_in, zp_out)
            else:
                raise lowering.LoweringError("int8: average pooling is not supported")
            continue
        if st.kind != "conv":
            raise lowering.LoweringError(f"int8: {st.label()} has no integer kernel")
        geom, w_bk, bias = lo_i8.weights[st.params["weight"]]
        if geom["groups"] != 1:
            raise lowering.LoweringError("int8: depthwise / grouped conv is not supported")
        _, w_orig, _ = lo_f32.weights[st.params["weight"]]
        x = st.inputs[0]
        xs = lo_i8.tensors[x]
        s_x, zp_x = tensors[xs.alias_of or x] if (xs.alias_of or x) in tensors else tensors[x]
        k = w_orig.shape[0]
        amax = np.abs(w_orig.reshape(k, -1)).max(axis=1)
        s_w = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
        w_q_orig = np.clip(np.rint(w_orig / s_w.reshape(k, 1, 1, 1)), -127, 127).astype(np.float32)
        if st.params.get("s2d"):
            w_q, _, _ = lowering.s2d_weights(w_q_orig, geom["pt_orig"], geom["pl_orig"])
            if geom.get("paired"):   # two output columns per row: the same codes, re-indexed
                w_q, _, _ = lowering.pair_weights(w_q, geom["cs_unpaired"], geom["pl_unpaired"])
        else:
            w_q = w_q_orig
        acc_scale = (np.float64(s_x) * s_w.astype(np.float64))
        b = np.zeros(k, np.float64) if bias is None else bias[:k].astype(np.float64)
        wsum = w_q_orig.reshape(k, -1).sum(axis=1).astype(np.int64)
        out_t = lo_i8.tensors[y]
        q = ConvQ(x=x, y=y, residual=st.params.get("residual"), w_q=w_q, w_q_orig=w_q_orig, s_w=s_w,
                  bias32=None, rq_scale=np.zeros(k, np.float32), act=st.params.get("act"),
                  nodes=list(st.nodes))
        if out_t.dtype == L.F32:
            q.bias32 = (-zp_x * wsum).astype(np.int32)
            q.deq_scale = (np.float32(s_x) * s_w).astype(np.float32)
            q.deq_bias = b.astype(np.float32)
            if q.residual:
                q.res_scale = float(np.float32(tensors[q.residual][0]))
        else:
            s_y, zp_y = act_qparams(*ranges[y])
            tensors[y] = (s_y, zp_y)
            q.bias32 = (np.rint(b / acc_scale).astype(np.int64) - zp_x * wsum).astype(np.int32)
            q.rq_scale = (acc_scale / np.float64(s_y)).astype(np.float32)
            q.qmin, q.qmax = _act_range(q.act, st.params["attrs"], s_y, zp_y)
            real_res = None
            if q.residual:
                s_r, _ = tensors[q.residual]
                q.res_scale = float(np.float32(np.float64(s_r) / np.float64(s_y)))
                real_res = np.float64(s_r) / np.float64(s_y)
            if requant == "fixed":
                q.rq_mult, q.rq_res_mult, q.rq_shift = shared_shift_multipliers(
                    acc_scale / np.float64(s_y), real_res)
                # the kernel keeps p >> S in 32 bits: bound it for every possible
                # 8-bit input (|x| <= 255, |w| <= 127 over the whole reduction)
                red = int(np.prod(w_q_orig.shape[1:]))
                acc_max = red * 255 * 127 + np.abs(q.bias32.astype(np.int64))
                top = (acc_max * q.rq_mult.astype(np.int64) + 255 * np.abs(q.rq_res_mult.astype(np.int64))
                       ) >> q.rq_shift.astype(np.int64)
                if top.max() >= (1 << 30):
                    raise lowering.LoweringError(f"int8: fixed-point requantisation of {st.label()} "
                                                 "could exceed 32 bits; use requant='fp32'")
        convs[st.params["weight"]] = q
    if requant not in ("fixed", "fp32"):
        raise ValueError(f"requant must be 'fixed' or 'fp32', not {requant!r}")
    return QuantPlan(tensors, convs, gap, lo_i8.steps, signed, requant)


def calibrate(graph, batches, *, device: int = 0) -> dict:
    """Per-tensor (min, max) of every activation the int8 executable stores,
    observed by running ``batches`` (a list of feed dicts) through an fp32
    executable of the same graph on the GPU."""
    from mdlc_b200.compiler import Executable
    n = int(np.asarray(next(iter(batches[0].values()))).shape[0])
    exe = Executable(graph, dtype="fp32", batch=n, devices=[device], keep_all=True)
    ranges = {}
    try:
        for feeds in batches:
            exe.run(feeds)
            for name, arr in exe.read_tensors().items():
                lo, hi = float(arr.min()), float(arr.max())
                if name in ranges:
                    lo, hi = min(lo, ranges[name][0]), max(hi, ranges[name][1])
                ranges[name] = (lo, hi)
            for name, arr in feeds.items():
                a = np.asarray(arr, np.float32)
                lo, hi = float(a.min()), float(a.max())
                if name in ranges:
                    lo, hi = min(lo, ranges[name][0]), max(hi, ranges[name][1])
                ranges[name] = (lo, hi)
    finally:
        exe.close()
    return ranges


def calibration_batches(graph, count: int = 32, batch: int = 4, seed: int = 0):
    """``count`` seeded N(0, 1) batches shaped like the graph input."""
    out = []
    for i in range(count):
        rng = np.random.default_rng(seed + i)
        feeds = {}
        for name in graph.runtime_inputs:
            shp = (batch,) + tuple(graph.value_info[name].shape[1:])
            feeds[name] = rng.standard_normal(shp).astype(np.float32)
        out.append(feeds)
    return out
