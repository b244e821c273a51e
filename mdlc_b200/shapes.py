"""Static shape propagation for the op set the backend lowers.

The reference infers shapes by executing its NumPy executor once
(``mdlc/passes/shape_inference.py:36-50``). The backend cannot execute the
graph on the host, so it applies per-op shape rules instead; when the caller
already ran the reference's shape inference, the recorded static shapes are
used as they are and only checked against these rules.
"""

from __future__ import annotations

import numpy as np


def _pads(attrs, in_hw, k_hw, s_hw, d_hw):
    auto = attrs.get("auto_pad", "NOTSET")
    (ih, iw), (kh, kw), (sh, sw), (dh, dw) = in_hw, k_hw, s_hw, d_hw
    if auto in ("SAME_UPPER", "SAME_LOWER"):
        oh, ow = -(-ih // sh), -(-iw // sw)
        ph = max(0, (oh - 1) * sh + (kh - 1) * dh + 1 - ih)
        pw = max(0, (ow - 1) * sw + (kw - 1) * dw + 1 - iw)
        if auto == "SAME_UPPER":
            return (ph // 2, ph - ph // 2), (pw // 2, pw - pw // 2)
        return (ph - ph // 2, ph // 2), (pw - pw // 2, pw // 2)
    p = attrs.get("pads") or [0, 0, 0, 0]
    return (p[0], p[2]), (p[1], p[3])


def conv_geometry(attrs, x_shape, w_shape):
    """Returns (oh, ow, (pt, pb), (pl, pr)) for a Conv node (``ops.py:15-32,56-60``)."""
    n, c, h, w = x_shape
    k, _, kh, kw = w_shape
    sh, sw = attrs.get("strides", [1, 1])
    dh, dw = attrs.get("dilations", [1, 1])
    (pt, pb), (pl, pr) = _pads(attrs, (h, w), (kh, kw), (sh, sw), (dh, dw))
    oh = (h + pt + pb - (dh * (kh - 1) + 1)) // sh + 1
    ow = (w + pl + pr - (dw * (kw - 1) + 1)) // sw + 1
    return oh, ow, (pt, pb), (pl, pr)


def pool_geometry(attrs, x_shape, is_max):
    n, c, h, w = x_shape
    kh, kw = attrs["kernel_shape"]
    sh, sw = attrs.get("strides", [1, 1])
    dh, dw = attrs.get("dilations", [1, 1]) if is_max else (1, 1)
    (pt, pb), (pl, pr) = _pads(attrs, (h, w), (kh, kw), (sh, sw), (dh, dw))
    div = (lambda a, q: -(-a // q)) if attrs.get("ceil_mode", 0) else (lambda a, q: a // q)
    oh = div(h + pt + pb - (dh * (kh - 1) + 1), sh) + 1
    ow = div(w + pl + pr - (dw * (kw - 1) + 1), sw) + 1
    return oh, ow, (pt, pb), (pl, pr)


def broadcast(*shapes):
    return tuple(int(d) for d in np.broadcast_shapes(*[tuple(s) for s in shapes]))


def node_shapes(node, shape_of, const_of):
    """Output shapes of ``node``; ``shape_of(name)`` gives known shapes and
    ``const_of(name)`` constant arrays (or None)."""
    op, a = node.op_type, node.attrs
    ins = node.inputs
    if op in ("Conv", "FusedConvAct", "FusedConvBNAct"):
        xs, ws = shape_of(ins[0]), shape_of(ins[1])
        oh, ow, _, _ = conv_geometry(a, xs, ws)
        return [(xs[0], ws[0], oh, ow)]
    if op in ("Gemm", "FusedGemmAct"):
        A, B = shape_of(ins[0]), shape_of(ins[1])
        M = A[1] if a.get("transA", 0) else A[0]
        N = B[0] if a.get("transB", 0) else B[1]
        return [(M, N)]
    if op == "MatMul":
        A, B = shape_of(ins[0]), shape_of(ins[1])
        return [tuple(A[:-1]) + (B[-1],)]
    if op in ("MaxPool", "AveragePool"):
        xs = shape_of(ins[0])
        oh, ow, _, _ = pool_geometry(a, xs, op == "MaxPool")
        return [(xs[0], xs[1], oh, ow)]
    if op == "GlobalAveragePool":
        xs = shape_of(ins[0])
        return [tuple(xs[:2]) + (1,) * (len(xs) - 2)]
    if op == "ReduceMean":
        xs = list(shape_of(ins[0]))
        axes = a.get("axes")
        if axes is None and len(ins) > 1 and ins[1]:
            axes = [int(v) for v in np.asarray(const_of(ins[1])).ravel()]
        axes = range(len(xs)) if axes is None else [x % len(xs) for x in axes]
        if a.get("keepdims", 1):
            return [tuple(1 if i in axes else d for i, d in enumerate(xs))]
        return [tuple(d for i, d in enumerate(xs) if i not in axes)]
    if op == "Flatten":
        xs = shape_of(ins[0])
        ax = a.get("axis", 1)
        ax = ax + len(xs) if ax < 0 else ax
        return [(int(np.prod(xs[:ax])) if ax else 1, int(np.prod(xs[ax:])))]
    if op == "Reshape":
        xs = shape_of(ins[0])
        tgt = [int(v) for v in np.asarray(const_of(ins[1])).ravel()]
        tgt = [xs[i] if t == 0 else t for i, t in enumerate(tgt)]
        if -1 in tgt:
            known = int(np.prod([t for t in tgt if t != -1]))
            tgt[tgt.index(-1)] = int(np.prod(xs)) // known
        return [tuple(tgt)]
    if op in ("Squeeze", "Unsqueeze"):
        xs = list(shape_of(ins[0]))
        axes = a.get("axes")
        if axes is None and len(ins) > 1 and ins[1]:
            axes = [int(v) for v in np.asarray(const_of(ins[1])).ravel()]
        if op == "Squeeze":
            axes = [i for i, d in enumerate(xs) if d == 1] if axes is None else [x % len(xs) for x in axes]
            return [tuple(d for i, d in enumerate(xs) if i not in axes)]
        for ax in sorted(axes):
            xs.insert(ax if ax >= 0 else ax + len(xs) + 1, 1)
        return [tuple(xs)]
    if op == "Identity":
        return [shape_of(ins[0])]
    if op == "FusedElementwise":
        local = {}

        def sh(nm):
            return local[nm] if nm in local else shape_of(nm)

        for sn in a["subgraph"]:
            for o, s in zip(sn.outputs, node_shapes(sn, sh, const_of)):
                local[o] = s
        return [local[o] for o in node.outputs]
    if op in ("Add", "Sub", "Mul", "Div"):
        return [broadcast(shape_of(ins[0]), shape_of(ins[1]))]
    if op == "BatchNormalization":
        return [shape_of(ins[0])]
    if op == "Transpose":
        xs = shape_of(ins[0])
        perm = a.get("perm", list(range(len(xs)))[::-1])
        return [tuple(xs[int(p)] for p in perm)]
    if op == "Pad":
        xs = shape_of(ins[0])
        pads = const_of(ins[1]) if len(ins) > 1 and ins[1] else a.get("pads")
        pads = [int(v) for v in np.asarray(pads).ravel()]
        r = len(xs)
        return [tuple(xs[i] + pads[i] + pads[i + r] for i in range(r))]
    if op == "Concat":
        parts = [shape_of(i) for i in ins if i]
        axis = int(a.get("axis", 0)) % len(parts[0])
        out = list(parts[0])
        out[axis] = sum(p[axis] for p in parts)
        return [tuple(out)]
    if op in ("Relu", "Clip", "Sigmoid", "Tanh", "HardSwish", "HardSigmoid", "LeakyRelu", "Erf",
              "Gelu", "Softmax"):
        return [shape_of(ins[0])]
    raise NotImplementedError(f"shape rule for {op!r}")


def infer(graph, batch=None) -> dict:
    """Static shape of every value. Graph inputs with symbolic dims take ``batch``."""
    shapes = {}
    for k, v in graph.initializers.items():
        shapes[k] = tuple(int(d) for d in np.asarray(v).shape)
    for name in graph.inputs:
        if name in shapes:
            continue
        info = graph.value_info.get(name)
        if info is None:
            raise ValueError(f"graph input {name!r} has no TensorInfo")
        dims = []
        for d in info.shape:
            if isinstance(d, (int, np.integer)) and d >= 0:
                dims.append(int(d))
            elif batch is not None:
                dims.append(int(batch))
            else:
                raise ValueError(f"input {name!r} has symbolic dim {d!r}; pass batch=")
        shapes[name] = tuple(dims)
    if batch is not None:
        for name in graph.runtime_inputs:
            shapes[name] = (int(batch),) + shapes[name][1:]

    def const_of(nm):
        return graph.initializers.get(nm)

    for node in graph.topo_sort():
        outs = node_shapes(node, lambda nm: shapes[nm], const_of)
        for o, s in zip(node.outputs, outs):
            if o:
                shapes[o] = tuple(int(d) for d in s)
    return shapes
