"""NumPy restatement of the reference executor — TEST INFRASTRUCTURE ONLY.

Semantics follow ``mdlc/runtime/reference.py`` (node dispatch, lines 80-195)
and ``mdlc/runtime/ops.py`` (op definitions, lines 12-255). Convolution keeps
the reference's algorithm — im2col then ``np.einsum("ok,nkp->nop")``
(``ops.py:56-81``) — so fp32 results are bit-identical to the reference on the
same inputs (checked against ``tests/golden`` fixtures). Grouped convolution is
evaluated for all groups in one einsum instead of a Python loop per group
(``ops.py:68-78``); each output is still the same k-ordered sum.

Extensions beyond the reference (parity for these is defined here, not pinned
by the reference, which raises ``NotImplementedError`` for them):
``Erf`` (scipy.special.erf), ``ReduceMean`` (``np.mean``), and ``Gelu``.

``bf16_emulation=True`` rounds every weight and every node output to bfloat16
(round-to-nearest-even) to model a backend that stores tensors in bf16 and
accumulates in fp32; it is a diagnosis aid, not the parity target.
"""

from __future__ import annotations

import numpy as np


# ----------------------------------------------------------------- helpers

def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 -> fp32 with round-to-nearest-even (NaN kept quiet)."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(np.float32)
    return np.where(np.isnan(a), a, out).reshape(a.shape)


def resolve_pads(auto_pad, pads, in_hw, k_hw, s_hw, d_hw):
    """((top, bottom), (left, right)) per ONNX, as ``ops.py:15-32``."""
    (ih, iw), (kh, kw), (sh, sw), (dh, dw) = in_hw, k_hw, s_hw, d_hw
    if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
        oh, ow = -(-ih // sh), -(-iw // sw)
        ph = max(0, (oh - 1) * sh + (kh - 1) * dh + 1 - ih)
        pw = max(0, (ow - 1) * sw + (kw - 1) * dw + 1 - iw)
        if auto_pad == "SAME_UPPER":
            return (ph // 2, ph - ph // 2), (pw // 2, pw - pw // 2)
        return (ph - ph // 2, ph // 2), (pw - pw // 2, pw // 2)
    if pads is None:
        return (0, 0), (0, 0)
    return (pads[0], pads[2]), (pads[1], pads[3])


def im2col(x, kh, kw, sh, sw, dh, dw, pads):
    """(N,C,H,W) -> (N, C*kh*kw, OH*OW); column order c-major then ky, kx
    (``ops.py:35-51``)."""
    n, c, h, w = x.shape
    (pt, pb), (pl, pr) = pads
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    oh = (h + pt + pb - (dh * (kh - 1) + 1)) // sh + 1
    ow = (w + pl + pr - (dw * (kw - 1) + 1)) // sw + 1
    taps = [xp[:, :, ky * dh: ky * dh + sh * oh: sh, kx * dw: kx * dw + sw * ow: sw][:, :, :oh, :ow]
            for ky in range(kh) for kx in range(kw)]
    cols = np.stack(taps, axis=2)                      # (n, c, kh*kw, oh, ow)
    return cols.reshape(n, c * kh * kw, oh * ow), oh, ow


# --------------------------------------------------------------------- ops

def conv(x, w, b, *, strides=(1, 1), pads=None, dilations=(1, 1), group=1, auto_pad="NOTSET"):
    n, c, ih, iw = x.shape
    oc, icg, kh, kw = w.shape
    p = resolve_pads(auto_pad, pads, (ih, iw), (kh, kw), tuple(strides), tuple(dilations))
    if group == 1:
        cols, oh, ow = im2col(x, kh, kw, strides[0], strides[1], dilations[0], dilations[1], p)
        out = np.einsum("ok,nkp->nop", w.reshape(oc, -1), cols).reshape(n, oc, oh, ow)
    else:
        ocg = oc // group
        cols, oh, ow = im2col(x, kh, kw, strides[0], strides[1], dilations[0], dilations[1], p)
        cols = cols.reshape(n, group, icg * kh * kw, oh * ow)
        wm = w.reshape(group, ocg, icg * kh * kw)
        out = np.einsum("gok,ngkp->ngop", wm, cols).reshape(n, oc, oh, ow)
    if b is not None:
        out = out + b.reshape(1, -1, 1, 1)
    return out


def gemm(a, b, c, *, alpha=1.0, beta=1.0, transA=0, transB=0):
    a = a.T if transA else a
    b = b.T if transB else b
    y = alpha * (a @ b)
    return y if c is None else y + beta * c


def batchnorm(x, scale, bias, mean, var, *, epsilon=1e-5):
    shp = [1] * x.ndim
    shp[1] = x.shape[1]
    return ((x - mean.reshape(shp)) / np.sqrt(var.reshape(shp) + epsilon)
            * scale.reshape(shp) + bias.reshape(shp))


def maxpool(x, *, kernel, strides=(1, 1), pads=None, dilations=(1, 1), auto_pad="NOTSET", ceil_mode=0):
    n, c, ih, iw = x.shape
    kh, kw = kernel
    sh, sw = strides
    dh, dw = dilations
    (pt, pb), (pl, pr) = resolve_pads(auto_pad, pads, (ih, iw), (kh, kw), (sh, sw), (dh, dw))
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr)), constant_values=-np.inf)
    div = (lambda a, q: -(-a // q)) if ceil_mode else (lambda a, q: a // q)
    oh = div(ih + pt + pb - (dh * (kh - 1) + 1), sh) + 1
    ow = div(iw + pl + pr - (dw * (kw - 1) + 1), sw) + 1
    out = np.full((n, c, oh, ow), -np.inf, dtype=x.dtype)
    for ky in range(kh):
        for kx in range(kw):
            win = xp[:, :, ky * dh: ky * dh + sh * oh: sh, kx * dw: kx * dw + sw * ow: sw]
            out = np.maximum(out, win[:, :, :oh, :ow])
    return out


def averagepool(x, *, kernel, strides=(1, 1), pads=None, auto_pad="NOTSET", count_include_pad=0, ceil_mode=0):
    n, c, ih, iw = x.shape
    kh, kw = kernel
    sh, sw = strides
    (pt, pb), (pl, pr) = resolve_pads(auto_pad, pads, (ih, iw), (kh, kw), (sh, sw), (1, 1))
    xp = np.pad(x, ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    div = (lambda a, q: -(-a // q)) if ceil_mode else (lambda a, q: a // q)
    oh = div(ih + pt + pb - kh, sh) + 1
    ow = div(iw + pl + pr - kw, sw) + 1
    acc = np.zeros((n, c, oh, ow), dtype=np.float64)
    cnt = np.zeros((n, c, oh, ow), dtype=np.float64)
    ones = np.pad(np.ones((n, c, ih, iw)), ((0, 0), (0, 0), (pt, pb), (pl, pr)))
    for ky in range(kh):
        for kx in range(kw):
            acc += xp[:, :, ky: ky + sh * oh: sh, kx: kx + sw * ow: sw][:, :, :oh, :ow]
            cnt += ones[:, :, ky: ky + sh * oh: sh, kx: kx + sw * ow: sw][:, :, :oh, :ow]
    denom = (kh * kw) if count_include_pad else np.maximum(cnt, 1)
    return (acc / denom).astype(x.dtype)


def global_average_pool(x):
    return x.mean(axis=tuple(range(2, x.ndim)), keepdims=True).astype(x.dtype)


def clip(x, lo=None, hi=None):
    return np.clip(x, -np.inf if lo is None else lo, np.inf if hi is None else hi)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def erf(x):
    from scipy.special import erf as _erf
    return _erf(x).astype(x.dtype)


def activation(name, x, attrs):
    """Epilogue activation table (``reference.py:19-38``)."""
    if not name or name == "Identity":
        return x
    if name == "Relu":
        return np.maximum(x, 0)
    if name == "Clip":
        return clip(x, attrs.get("clip_min"), attrs.get("clip_max"))
    if name == "Relu6":
        return clip(x, 0.0, 6.0)
    if name == "Sigmoid":
        return sigmoid(x)
    if name == "Tanh":
        return np.tanh(x)
    if name == "LeakyRelu":
        a = attrs.get("alpha", 0.01)
        return np.where(x >= 0, x, a * x)
    if name == "HardSigmoid":
        return np.clip(attrs.get("alpha", 0.2) * x + attrs.get("beta", 0.5), 0.0, 1.0)
    if name == "HardSwish":
        return x * np.clip(x / 6.0 + 0.5, 0.0, 1.0)
    if name == "Gelu":
        return (0.5 * x * (1.0 + erf(x / np.float32(np.sqrt(2.0))))).astype(x.dtype)
    raise NotImplementedError(f"activation {name!r}")


def _reshape(x, shape):
    out = []
    for i, s in enumerate(int(v) for v in np.asarray(shape).ravel()):
        out.append(x.shape[i] if s == 0 else s)
    return x.reshape(out)


def _flatten(x, axis=1):
    axis = axis + x.ndim if axis < 0 else axis
    outer = int(np.prod(x.shape[:axis])) if axis > 0 else 1
    return x.reshape(outer, -1)


# ---------------------------------------------------------------- executor

def exec_node(node, env, bf16_emulation=False):
    """Evaluate one node; returns the list of output arrays."""
    op, a = node.op_type, node.attrs
    ins = [env[i] if i else None for i in node.inputs]

    if op in ("FusedConvAct", "FusedConvBNAct", "Conv"):
        y = conv(ins[0], ins[1], ins[2] if len(ins) > 2 else None,
                 strides=a.get("strides", [1, 1]), pads=a.get("pads"),
                 dilations=a.get("dilations", [1, 1]), group=a.get("group", 1),
                 auto_pad=a.get("auto_pad", "NOTSET"))
        return [activation(a.get("activation"), y, a) if op != "Conv" else y]
    if op in ("FusedGemmAct", "Gemm"):
        y = gemm(ins[0], ins[1], ins[2] if len(ins) > 2 else None,
                 alpha=a.get("alpha", 1.0) if op == "Gemm" else a.get("alpha", 1.0),
                 beta=a.get("beta", 1.0), transA=a.get("transA", 0), transB=a.get("transB", 0))
        return [activation(a.get("activation"), y, a) if op != "Gemm" else y]
    if op == "FusedElementwise":
        local = dict(env)
        for sn in a["subgraph"]:
            for oname, oval in zip(sn.outputs, exec_node(sn, local, bf16_emulation=False)):
                if oname:
                    local[oname] = oval
        return [local[o] for o in node.outputs]
    if op == "MatMul":
        return [ins[0] @ ins[1]]
    if op == "BatchNormalization":
        return [batchnorm(*ins[:5], epsilon=a.get("epsilon", 1e-5))]
    if op == "MaxPool":
        return [maxpool(ins[0], kernel=a["kernel_shape"], strides=a.get("strides", [1, 1]),
                        pads=a.get("pads"), dilations=a.get("dilations", [1, 1]),
                        auto_pad=a.get("auto_pad", "NOTSET"), ceil_mode=a.get("ceil_mode", 0))]
    if op == "AveragePool":
        return [averagepool(ins[0], kernel=a["kernel_shape"], strides=a.get("strides", [1, 1]),
                            pads=a.get("pads"), auto_pad=a.get("auto_pad", "NOTSET"),
                            count_include_pad=a.get("count_include_pad", 0),
                            ceil_mode=a.get("ceil_mode", 0))]
    if op == "GlobalAveragePool":
        return [global_average_pool(ins[0])]
    if op == "ReduceMean":
        axes = ins[1] if len(ins) > 1 and ins[1] is not None else a.get("axes")
        axes = None if axes is None else tuple(int(v) for v in np.asarray(axes).ravel())
        return [np.mean(ins[0], axis=axes, keepdims=bool(a.get("keepdims", 1))).astype(ins[0].dtype)]
    if op in ("Relu", "Sigmoid", "Tanh", "HardSwish", "Gelu"):
        return [activation(op, ins[0], a)]
    if op == "Clip":
        lo = ins[1] if len(ins) > 1 and ins[1] is not None else a.get("min")
        hi = ins[2] if len(ins) > 2 and ins[2] is not None else a.get("max")
        lo = None if lo is None else float(np.asarray(lo).item())
        hi = None if hi is None else float(np.asarray(hi).item())
        return [clip(ins[0], lo, hi)]
    if op == "LeakyRelu":
        return [activation(op, ins[0], {"alpha": a.get("alpha", 0.01)})]
    if op == "HardSigmoid":
        return [activation(op, ins[0], {"alpha": a.get("alpha", 0.2), "beta": a.get("beta", 0.5)})]
    if op == "Erf":
        return [erf(ins[0])]
    if op == "Softmax":
        z = ins[0] - np.max(ins[0], axis=a.get("axis", -1), keepdims=True)
        e = np.exp(z)
        return [e / np.sum(e, axis=a.get("axis", -1), keepdims=True)]
    if op == "Add":
        return [ins[0] + ins[1]]
    if op == "Sub":
        return [ins[0] - ins[1]]
    if op == "Mul":
        return [ins[0] * ins[1]]
    if op == "Div":
        return [ins[0] / ins[1]]
    if op == "Flatten":
        return [_flatten(ins[0], a.get("axis", 1))]
    if op == "Reshape":
        return [_reshape(ins[0], ins[1])]
    if op == "Transpose":
        return [np.transpose(ins[0], a.get("perm"))]
    if op == "Concat":
        return [np.concatenate([x for x in ins if x is not None], axis=a.get("axis", 0))]
    if op == "Pad":   # ops.py:249-255: pads = [begin..., end...], constant / reflect / edge
        pads = ins[1] if len(ins) > 1 and ins[1] is not None else a.get("pads")
        pads = [int(p) for p in np.asarray(pads).ravel()]
        val = ins[2] if len(ins) > 2 and ins[2] is not None else a.get("value", 0.0)
        half = len(pads) // 2
        width = [(pads[i], pads[i + half]) for i in range(half)]
        mode = a.get("mode", "constant")
        mode = mode.decode() if isinstance(mode, bytes) else mode
        if mode == "constant":
            return [np.pad(ins[0], width, mode="constant", constant_values=float(np.asarray(val).item()))]
        return [np.pad(ins[0], width, mode={"reflect": "reflect", "edge": "edge"}.get(mode, "constant"))]
    if op == "Squeeze":
        axes = ins[1] if len(ins) > 1 and ins[1] is not None else a.get("axes")
        return [np.squeeze(ins[0]) if axes is None
                else np.squeeze(ins[0], axis=tuple(int(v) for v in np.asarray(axes).ravel()))]
    if op == "Unsqueeze":
        axes = ins[1] if len(ins) > 1 and ins[1] is not None else a.get("axes")
        x = ins[0]
        for ax in sorted(int(v) for v in np.asarray(axes).ravel()):
            x = np.expand_dims(x, ax)
        return [x]
    if op == "Constant":
        return [a["value"]]
    if op == "Identity":
        return [ins[0]]
    if op == "Shape":
        return [np.array(ins[0].shape, dtype=np.int64)]
    raise NotImplementedError(f"oracle: op {op!r}")


def run(graph, feeds, *, return_all=False, bf16_emulation=False):
    """Run ``graph`` over numpy feeds in topological order (``reference.py:47-70``)."""
    env = {}
    for name, arr in graph.initializers.items():
        arr = np.asarray(arr)
        if bf16_emulation and arr.dtype == np.float32 and arr.ndim >= 2:
            arr = round_bf16(arr)
        env[name] = arr
    for name, arr in feeds.items():
        arr = np.asarray(arr)
        env[name] = round_bf16(arr) if bf16_emulation else arr
    for node in graph.topo_sort():
        for oname, oval in zip(node.outputs, exec_node(node, env, bf16_emulation)):
            if oname:
                oval = np.asarray(oval)
                if bf16_emulation and oval.dtype == np.float32 and oname not in graph.outputs:
                    oval = round_bf16(oval)
                env[oname] = oval
    if return_all:
        return env
    return {o: env[o] for o in graph.outputs}
