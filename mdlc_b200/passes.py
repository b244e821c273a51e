"""The reference's default graph pipeline, restated so graphs can be prepared
for the backend on machines without the reference package.

``compile()`` consumes a *post-pass* graph. When the reference package is
installed its ``default_pipeline()`` produces that graph; this module produces
the same graph (same node order, op types, node names, attrs and folded
initializer bytes) for the model builders in :mod:`mdlc_b200.builders`.
Parity with the reference pipeline is checked by the CPU test suite against
committed fixtures.

Passes restated (run to a fixed point in this order, ``mdlc/passes/base.py:76-102``):
  * constant folding of ``Constant``/``Identity`` nodes only — the builders emit
    no other all-constant subgraphs (``mdlc/passes/constant_folding.py``);
  * Conv+BatchNormalization folding (``mdlc/passes/fuse_conv_bn.py:23-81``);
  * dead-code elimination (``mdlc/passes/dce.py:9-49``);
  * activation fusion onto Conv/Gemm (``mdlc/passes/fuse_activation.py:17-94``);
  * elementwise-chain fusion by union-find over single-use edges
    (``mdlc/passes/fuse_elementwise.py:46-137``).
"""

from __future__ import annotations

from collections import defaultdict

import numpy as np

from mdlc_b200.ir import Graph, Node

ACTIVATIONS = {"Relu", "Clip", "Sigmoid", "Tanh", "HardSwish", "HardSigmoid", "LeakyRelu"}
ELEMENTWISE = {"Add", "Sub", "Mul", "Div"} | ACTIVATIONS
_FUSED_NAME = {"Conv": "FusedConvAct", "Gemm": "FusedGemmAct"}


def _fold_constants(g: Graph) -> bool:
    changed = False
    for node in list(g.nodes):
        if node.op_type == "Constant" and not node.real_inputs():
            g.set_initializer(node.outputs[0], np.asarray(node.attrs["value"]))
        elif node.op_type == "Identity" and node.real_inputs() and g.is_constant(node.inputs[0]):
            g.set_initializer(node.outputs[0], g.initializers[node.inputs[0]])
        else:
            continue
        g.remove_nodes([node])
        changed = True
    return changed


def _fuse_conv_bn(g: Graph) -> bool:
    changed = False
    producer = g.producers()
    uses = g.use_count()
    for bn in list(g.nodes):
        if bn.op_type != "BatchNormalization":
            continue
        conv = producer.get(bn.inputs[0])
        if conv is None or conv.op_type != "Conv":
            continue
        if uses.get(conv.outputs[0], 0) != 1 or conv.outputs[0] in g.outputs:
            continue
        w_name = conv.inputs[1]
        params = bn.inputs[1:5]
        if not g.is_constant(w_name) or not all(g.is_constant(p) for p in params):
            continue
        eps = bn.attr("epsilon", 1e-5)
        w = g.initializers[w_name].astype(np.float32)
        gamma, beta, mean, var = (g.initializers[p].astype(np.float32) for p in params)
        scale = gamma / np.sqrt(var + eps)
        oc = w.shape[0]
        w_new = w * scale.reshape(oc, *([1] * (w.ndim - 1)))
        if len(conv.inputs) > 2 and conv.inputs[2]:
            b_conv = g.initializers[conv.inputs[2]].astype(np.float32)
        else:
            b_conv = np.zeros(oc, dtype=np.float32)
        b_new = b_conv * scale + (beta - mean * scale)
        new_w, new_b = w_name + "_bnfold", (conv.name or "conv") + "_bias_bnfold"
        g.set_initializer(new_w, w_new)
        g.set_initializer(new_b, b_new)
        conv.inputs = [conv.inputs[0], new_w, new_b]
        conv.outputs = [bn.outputs[0]]
        g.remove_nodes([bn])
        changed = True
    return changed


def _dce(g: Graph) -> bool:
    producer = g.producers()
    needed = set(g.outputs)
    stack = list(g.outputs)
    live = set()
    while stack:
        node = producer.get(stack.pop())
        if node is None or id(node) in live:
            continue
        live.add(id(node))
        for i in node.real_inputs():
            if i not in needed:
                needed.add(i)
                stack.append(i)
    before = len(g.nodes)
    g.nodes = [n for n in g.nodes if id(n) in live]
    changed = len(g.nodes) != before
    used = set(g.outputs) | set(g.inputs)
    for n in g.nodes:
        used.update(n.real_inputs())
        used.update(o for o in n.outputs if o)
    for k in list(g.initializers):
        if k not in used:
            del g.initializers[k]
            changed = True
    for k in list(g.value_info):
        if k not in used:
            del g.value_info[k]
    return changed


def _const_scalar(g: Graph, node: Node, idx: int, fallback):
    if len(node.inputs) > idx and node.inputs[idx]:
        arr = g.initializers.get(node.inputs[idx])
        if arr is None:
            return False, None
        return True, float(np.asarray(arr).item())
    return True, (None if fallback is None else float(fallback))


def _fuse_activation(g: Graph) -> bool:
    changed = False
    producer = g.producers()
    uses = g.use_count()
    for act in list(g.nodes):
        if act.op_type not in ACTIVATIONS:
            continue
        src = producer.get(act.inputs[0])
        if src is None or src.op_type not in _FUSED_NAME:
            continue
        feed = src.outputs[0]
        if uses.get(feed, 0) != 1 or feed in g.outputs:
            continue
        fused = Node(_FUSED_NAME[src.op_type], list(src.inputs), list(act.outputs),
                     dict(src.attrs), (src.name or src.op_type) + "+" + act.op_type,
                     [src.op_type, act.op_type])
        fused.attrs["activation"] = act.op_type
        if act.op_type == "Clip":
            ok_lo, lo = _const_scalar(g, act, 1, act.attr("min"))
            ok_hi, hi = _const_scalar(g, act, 2, act.attr("max"))
            if not (ok_lo and ok_hi):
                continue
            fused.attrs["clip_min"], fused.attrs["clip_max"] = lo, hi
        elif act.op_type == "LeakyRelu":
            fused.attrs["alpha"] = act.attr("alpha", 0.01)
        elif act.op_type == "HardSigmoid":
            fused.attrs["alpha"] = act.attr("alpha", 0.2)
            fused.attrs["beta"] = act.attr("beta", 0.5)
        g.nodes[g.nodes.index(src)] = fused
        g.remove_nodes([act])
        changed = True
    return changed


def _fuse_elementwise(g: Graph) -> bool:
    nodes = g.nodes
    idx = {id(n): k for k, n in enumerate(nodes)}
    ew = [k for k, n in enumerate(nodes) if n.op_type in ELEMENTWISE]
    if not ew:
        return False
    producer, uses, consumers = g.producers(), g.use_count(), g.consumers()
    out_set = set(g.outputs)
    parent = list(range(len(nodes)))

    def find(x):
        while parent[x] != x:
            parent[x] = parent[parent[x]]
            x = parent[x]
        return x

    for k in ew:
        for e in nodes[k].real_inputs():
            p = producer.get(e)
            if p is None or p.op_type not in ELEMENTWISE:
                continue
            if uses.get(e, 0) == 1 and e not in out_set:
                ra, rb = find(idx[id(p)]), find(k)
                if ra != rb:
                    parent[ra] = rb
    groups = defaultdict(list)
    for k in ew:
        groups[find(k)].append(k)

    replacement, drop = {}, set()
    for members in groups.values():
        if len(members) < 2:
            continue
        members = sorted(members)
        member_ids = {id(nodes[m]) for m in members}
        inner = [nodes[k] for k in members]
        internal = {o for n in inner for o in n.outputs if o}
        g_in, seen = [], set()
        for n in inner:
            for e in n.real_inputs():
                if e not in internal and e not in seen:
                    seen.add(e)
                    g_in.append(e)
        g_out = []
        for n in inner:
            for o in n.outputs:
                if o and (o in out_set or any(id(c) not in member_ids
                                              for c in consumers.get(o, []))):
                    g_out.append(o)
        fused = Node("FusedElementwise", g_in, g_out, {"subgraph": inner},
                     "fused_ew_" + "_".join(str(k) for k in members),
                     [nodes[k].op_type for k in members])
        replacement[members[-1]] = fused
        drop.update(members)
    if not replacement:
        return False
    g.nodes = [replacement[k] if k in replacement else n
               for k, n in enumerate(nodes) if k in replacement or k not in drop]
    return True


PIPELINE = (("constant_folding", _fold_constants), ("fuse_conv_bn", _fuse_conv_bn),
            ("dce", _dce), ("fuse_activation", _fuse_activation),
            ("fuse_elementwise", _fuse_elementwise), ("dce", _dce))


def default_pipeline(graph: Graph, max_iters: int = 8) -> Graph:
    """Run the pipeline to a fixed point, then reorder topologically
    (``mdlc/passes/base.py:50-66``). Mutates and returns ``graph``."""
    for _ in range(max_iters):
        any_changed = False
        for _, fn in PIPELINE:
            any_changed |= bool(fn(graph))
        if not any_changed:
            break
    graph.reorder_topologically()
    return graph
