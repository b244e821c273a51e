"""Integer NumPy restatement of the INT8 path — TEST INFRASTRUCTURE ONLY.

The reference has no quantised operators (``mdlc/ir/tensor.py:29``,
``docs/GAPS.md:128``), so this module *defines* INT8 parity: given the same
quantisation plan as the device (scales, zero points, int8 weight codes, int32
biases, requantisation scales), it evaluates the network with exact integer
accumulation and IEEE float32 requantisation:

* conv / GEMM: im2col of the uint8 codes padded with the input zero point, then
  an int64 ``einsum("ok,nkp->nop")`` — the reference's conv algorithm
  (``mdlc/runtime/ops.py:35-81``) on integers — plus the int32 bias;
* conv requantisation (8-bit outputs), as the plan says:
  fixed point (the default), one rounding: ``zp + clip((acc*M1[k] [+ (res - zp_r)*M2[k]]
  + 2^(S[k]-1)) >> S[k], qmin - zp, qmax - zp)`` in int64 -- the single-rounding
  form of TFLite's MultiplyByQuantizedMultiplier (``TFLITE_SINGLE_ROUNDING``),
  the residual product sharing the channel's shift; or IEEE float32, one
  rounding per product and sum:
  ``zp + clip(rint(f32(acc + bias32) * r[k] [+ f32(res - zp_r) * r_res]), qmin - zp, qmax - zp)``;
* global-average-pool requantisation in gemmlowp fixed point:
  SaturatingRoundingDoublingHighMul (truncating division by 2^31) followed by
  RoundingDivideByPOT (round half away from zero);
* max pool on codes over in-bounds taps; global average pool as an int32 sum of
  ``q - zp`` requantised;
* fp32 logits ``act(float32(acc + bias32) * float32(scale) + float32(bias)
  [+ float32(res - zp_r) * float32(s_r)])``.

Device results must match this bit for bit (int32 accumulators are covered
through the requantised codes and the fp32 logits derived from them).
"""

from __future__ import annotations

import numpy as np

from oracle import reference as oref

ALIASES = {"Flatten", "Reshape", "Squeeze", "Unsqueeze", "Identity"}
INT32_MIN = -(1 << 31)
INT32_MAX = (1 << 31) - 1


def srdhm(a, b):
    """SaturatingRoundingDoublingHighMul on int32 values held in int64 arrays."""
    a = np.asarray(a, np.int64)
    b = np.asarray(b, np.int64)
    ab = a * b
    t = ab + np.where(ab >= 0, 1 << 30, 1 - (1 << 30))
    q = np.where(t >= 0, t >> 31, -((-t) >> 31))            # truncation toward zero
    return np.where((a == INT32_MIN) & (b == INT32_MIN), INT32_MAX, q)


def rdbpot(x, shift):
    """RoundingDivideByPOT: x / 2^shift rounded half away from zero."""
    x = np.asarray(x, np.int64)
    shift = np.asarray(shift, np.int64)
    mask = (np.int64(1) << shift) - 1
    rem = x & mask
    thr = (mask >> 1) + (x < 0)
    return (x >> shift) + (rem > thr)


def requant(v, mult, shift):
    """gemmlowp MultiplyByQuantizedMultiplier: a negative shift is a left shift of
    the input (saturated to int32) before the high multiply."""
    shift = np.asarray(shift, np.int64)
    lsh = np.maximum(-shift, 0)
    v = np.clip(np.asarray(v, np.int64) << lsh, INT32_MIN, INT32_MAX)
    return rdbpot(srdhm(v, mult), np.maximum(shift, 0))


def quantize_input(x, scale, zp, signed=False):
    inv = np.float32(1.0) / np.float32(scale)
    q = np.rint(np.asarray(x, np.float32) * inv).astype(np.int64) + zp
    return np.clip(q, -128, 127) if signed else np.clip(q, 0, 255)


def conv_int(xq, wq, zp, attrs):
    """int64 conv of 8-bit codes (N,C,H,W) with zero-point padding (ops.py:56-81)."""
    n, c, ih, iw = xq.shape
    k, _, kh, kw = wq.shape
    sh, sw = attrs.get("strides", [1, 1])
    dh, dw = attrs.get("dilations", [1, 1])
    (pt, pb), (pl, pr) = oref.resolve_pads(attrs.get("auto_pad", "NOTSET"), attrs.get("pads"), (ih, iw),
                                           (kh, kw), (sh, sw), (dh, dw))
    xp = np.pad(xq, ((0, 0), (0, 0), (pt, pb), (pl, pr)), constant_values=zp)
    oh = (ih + pt + pb - (dh * (kh - 1) + 1)) // sh + 1
    ow = (iw + pl + pr - (dw * (kw - 1) + 1)) // sw + 1
    taps = [xp[:, :, ky * dh: ky * dh + sh * oh: sh, kx * dw: kx * dw + sw * ow: sw][:, :, :oh, :ow]
            for ky in range(kh) for kx in range(kw)]
    cols = np.stack(taps, axis=2).reshape(n, c * kh * kw, oh * ow)
    out = np.einsum("ok,nkp->nop", wq.reshape(k, -1).astype(np.int64), cols)
    return out.reshape(n, k, oh, ow)


def run_int8(graph, plan, feeds):
    """Evaluate ``graph`` under ``plan`` (a mdlc_b200.quant.QuantPlan) on fp32 feeds.
    Returns {output name: array} — uint8 codes for quantised outputs, fp32 for
    dequantised ones — plus every intermediate under ``"__codes__"``."""
    nodes = {n.name: n for n in graph.nodes}
    alias = {}
    for n in graph.nodes:
        if n.op_type in ALIASES:
            alias[n.outputs[0]] = n.inputs[0]

    def src(name):
        while name in alias:
            name = alias[name]
        return name

    env = {}
    for name in graph.runtime_inputs:
        s, zp = plan.tensors[name]
        env[name] = quantize_input(feeds[name], s, zp, name in plan.signed)
    for st in plan.steps:
        if st.kind == "pool":
            x = env[src(st.inputs[0])]
            p = st.params
            if p["kind"] == 0:
                oh, ow = p["oh"], p["ow"]
                pb = max(0, (oh - 1) * p["sh"] + p["kh"] - x.shape[2] - p["pt"])
                pr = max(0, (ow - 1) * p["sw"] + p["kw"] - x.shape[3] - p["pl"])
                xp = np.pad(x, ((0, 0), (0, 0), (p["pt"], pb), (p["pl"], pr)),
                            constant_values=-1)          # -1: below every code, i.e. not a tap
                out = np.full(x.shape[:2] + (oh, ow), -1, np.int64)
                for ky in range(p["kh"]):
                    for kx in range(p["kw"]):
                        win = xp[:, :, ky: ky + p["sh"] * oh: p["sh"], kx: kx + p["sw"] * ow: p["sw"]]
                        out = np.maximum(out, win[:, :, :oh, :ow])
                env[st.outputs[0]] = out
            else:
                m, sh, zp_in, zp_out = plan.gap[st.outputs[0]]
                s = (x - zp_in).reshape(x.shape[0], x.shape[1], -1).sum(axis=2)
                q = np.clip(zp_out + requant(s, m, sh), 0, 255)
                env[st.outputs[0]] = q.reshape(x.shape[0], x.shape[1], 1, 1)
            continue
        cq = plan.convs[st.params["weight"]]
        node = nodes[st.nodes[0]]
        x = env[src(cq.x)]
        if x.ndim == 2:
            x = x.reshape(x.shape[0], x.shape[1], 1, 1)
        attrs = node.attrs if node.op_type not in ("Gemm", "FusedGemmAct", "MatMul") else {}
        zp_x = plan.tensors[src(cq.x)][1]
        acc = conv_int(x, cq.w_q_orig, zp_x, attrs)
        k = acc.shape[1]
        acc = acc + cq.bias32.astype(np.int64).reshape(1, k, 1, 1)
        if cq.deq_scale is not None:
            y = (acc.astype(np.float32) * cq.deq_scale.reshape(1, k, 1, 1)).astype(np.float32)
            y = (y + cq.deq_bias.reshape(1, k, 1, 1)).astype(np.float32)
            if cq.residual:
                r = env[src(cq.residual)]
                zp_r = plan.tensors[src(cq.residual)][1]
                y = (y + (r - zp_r).astype(np.float32) * np.float32(cq.res_scale)).astype(np.float32)
            y = oref.activation(cq.act, y, node.attrs).astype(np.float32)
            env[st.outputs[0]] = y.reshape(y.shape[0], k) if node.op_type in ("Gemm", "FusedGemmAct", "MatMul") else y
        elif getattr(cq, "rq_mult", None) is not None:
            # single-rounding fixed point (TFLite MultiplyByQuantizedMultiplier,
            # TFLITE_SINGLE_ROUNDING form): t = (acc*M1 + (r - zp_r)*M2 + 2^(S-1)) >> S
            # in int64 (|acc*M1| < 2^62), arithmetic shift = floor, so ties round up
            zp_y = plan.tensors[st.outputs[0]][1]
            m1 = cq.rq_mult.astype(np.int64).reshape(1, k, 1, 1)
            sh = cq.rq_shift.astype(np.int64).reshape(1, k, 1, 1)
            v = acc.astype(np.int64) * m1 + (np.int64(1) << (sh - 1))
            if cq.residual:
                r = env[src(cq.residual)]
                zp_r = plan.tensors[src(cq.residual)][1]
                v = v + (np.asarray(r, np.int64) - zp_r) * cq.rq_res_mult.astype(np.int64).reshape(1, k, 1, 1)
            t = np.clip(v >> sh, cq.qmin - zp_y, cq.qmax - zp_y) + zp_y
            env[st.outputs[0]] = t.reshape(t.shape[0], k) if node.op_type in ("Gemm", "FusedGemmAct", "MatMul") else t
        else:
            zp_y = plan.tensors[st.outputs[0]][1]
            f = acc.astype(np.float32) * cq.rq_scale.astype(np.float32).reshape(1, k, 1, 1)
            if cq.residual:
                r = env[src(cq.residual)]
                zp_r = plan.tensors[src(cq.residual)][1]
                f = f + (r - zp_r).astype(np.float32) * np.float32(cq.res_scale)
            assert f.dtype == np.float32
            t = np.clip(np.rint(f), cq.qmin - zp_y, cq.qmax - zp_y).astype(np.int64) + zp_y
            env[st.outputs[0]] = t.reshape(t.shape[0], k) if node.op_type in ("Gemm", "FusedGemmAct", "MatMul") else t
    outs = {o: env[src(o)] for o in graph.outputs}
    outs["__codes__"] = env
    return outs
