"""Generate the golden fixtures that pin the oracle and the pass pipeline to
the reference implementation.

Run in a container where the reference package is importable (its source tree
is passed with ``--reference``; nothing else in the repository reads it):

    python tests/golden/make_golden.py --reference /path/to/mdlc-reference

For every case the graph comes from :mod:`mdlc_b200.builders` (seeded), is
converted to the reference's own ``Graph``/``Node`` classes, and:
  * the reference ``default_pipeline()`` is run on it; the resulting node list
    (op types, names, edges, attrs, fused groups) and a SHA-256 of every
    initializer is written to ``passes.json``;
  * the reference ``run_reference`` output on the seeded feeds is written to
    ``<case>.npz`` (raw graph and post-pass graph), along with the reference
    ``plan_memory`` summary to ``memplan.json``.
The CPU test suite compares :mod:`oracle.reference`, :mod:`mdlc_b200.passes`
and the backend's planner against these files.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from mdlc_b200 import builders  # noqa: E402

# (case name, builder, kwargs, run reference on raw graph too)
CASES = [
    ("conv_bn_relu", "conv_bn_relu", dict(n=2, cin=3, cout=8, h=10, w=10)),
    ("conv_bn_relu6_s2", "conv_bn_relu", dict(n=2, cin=16, cout=24, h=9, w=11, stride=2, act="Relu6")),
    ("conv_bn_k1", "conv_bn_relu", dict(n=3, cin=32, cout=16, h=7, w=7, k=1, act=None)),
    ("residual_block", "residual_block", dict(n=2, c=8, h=8, w=8)),
    ("mlp", "mlp", dict()),
    ("resnet18_s64_b2", "resnet18", dict(batch=2, image=64)),
    ("resnet18_b1", "resnet18", dict(batch=1, image=224)),
    ("mobilenetv2_s64_b2", "mobilenetv2", dict(batch=2, image=64)),
    ("mobilenetv2_b1", "mobilenetv2", dict(batch=1, image=224)),
]
# graphs the reference pipeline is checked on structurally (RepViT needs
# Erf/ReduceMean, which the reference executor lacks, so only its passes are pinned)
PASS_CASES = CASES + [("repvit_s64_b1", "repvit", dict(batch=1, image=64))]


def to_reference_graph(g, ref_ir):
    rg = ref_ir.Graph(g.name)
    rg.inputs, rg.outputs = list(g.inputs), list(g.outputs)
    rg.initializers = {k: np.asarray(v) for k, v in g.initializers.items()}
    for k, v in g.value_info.items():
        rg.value_info[k] = ref_ir.TensorInfo(v.name, v.dtype, tuple(v.shape))
    for n in g.nodes:
        rg.nodes.append(ref_ir.Node(n.op_type, list(n.inputs), list(n.outputs), dict(n.attrs),
                                    n.name, None if n.fused_from is None else list(n.fused_from)))
    return rg


def describe(graph):
    """JSON-able structural summary of a post-pass graph."""
    nodes = []
    for n in graph.nodes:
        attrs = {k: v for k, v in n.attrs.items() if k != "subgraph"}
        d = {"op": n.op_type, "name": n.name, "inputs": list(n.inputs), "outputs": list(n.outputs),
             "attrs": json.loads(json.dumps(attrs, default=float)),
             "fused_from": n.fused_from}
        if "subgraph" in n.attrs:
            d["subgraph"] = [{"op": s.op_type, "name": s.name, "inputs": list(s.inputs),
                              "outputs": list(s.outputs)} for s in n.attrs["subgraph"]]
        nodes.append(d)
    inits = {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest()
             for k, v in sorted(graph.initializers.items())}
    return {"nodes": nodes, "initializers": inits, "inputs": list(graph.inputs),
            "outputs": list(graph.outputs)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="reference source tree (contains mdlc/)")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import mdlc.ir as ref_ir
    from mdlc.passes import default_pipeline
    from mdlc.runtime.memory_planner import plan_memory
    from mdlc.runtime.reference import run_reference
    from mdlc.passes.shape_inference import infer_shapes_by_execution

    passes_out = {}
    for case, bname, kw in PASS_CASES:
        g = builders.BUILDERS[bname](**kw)
        rg = default_pipeline().run(to_reference_graph(g, ref_ir))
        passes_out[case] = describe(rg)
    with open(os.path.join(HERE, "passes.json"), "w") as f:
        json.dump(passes_out, f, indent=0, sort_keys=True)

    memplans = {}
    for case, bname, kw in CASES:
        g = builders.BUILDERS[bname](**kw)
        feeds = builders.make_input(g, seed=0)
        raw = run_reference(to_reference_graph(g, ref_ir), feeds)
        rg = default_pipeline().run(to_reference_graph(g, ref_ir))
        post = run_reference(rg, feeds)
        np.savez_compressed(os.path.join(HERE, f"{case}.npz"),
                            **{f"raw.{k}": v for k, v in raw.items()},
                            **{f"post.{k}": v for k, v in post.items()})
        infer_shapes_by_execution(rg, feeds)
        plan = plan_memory(rg)
        memplans[case] = {"assignment": plan.assignment,
                          "buffers": [b.size for b in plan.buffers],
                          "naive": plan.naive_activation_bytes,
                          "planned": plan.planned_activation_bytes}
        print(f"{case}: outputs {[(k, v.shape) for k, v in post.items()]}, "
              f"{len(plan.buffers)} buffers, {plan.planned_activation_bytes} B planned")
    with open(os.path.join(HERE, "memplan.json"), "w") as f:
        json.dump(memplans, f, indent=0, sort_keys=True)


if __name__ == "__main__":
    main()
