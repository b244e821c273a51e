"""The oracle and the restated pass pipeline reproduce the reference.

Fixtures come from the reference's own ``run_reference`` and
``default_pipeline`` (``tests/golden/make_golden.py``); nothing here imports
the reference.
"""

import hashlib
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden
from mdlc_b200 import builders, passes
from oracle import reference as oref

with open(os.path.join(GOLDEN, "passes.json")) as f:
    PASSES = json.load(f)

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
PASS_CASES = CASES + [("repvit_s64_b1", "repvit", dict(batch=1, image=64))]


def _describe(g):
    out = []
    for n in g.nodes:
        d = {"op": n.op_type, "name": n.name, "inputs": list(n.inputs), "outputs": list(n.outputs),
             "fused_from": n.fused_from,
             "attrs": json.loads(json.dumps({k: v for k, v in n.attrs.items() if k != "subgraph"},
                                            default=float))}
        if "subgraph" in n.attrs:
            d["subgraph"] = [{"op": s.op_type, "name": s.name, "inputs": list(s.inputs),
                              "outputs": list(s.outputs)} for s in n.attrs["subgraph"]]
        out.append(d)
    return out


@pytest.mark.parametrize("case,bname,kw", PASS_CASES, ids=[c[0] for c in PASS_CASES])
def test_pass_pipeline_matches_reference(case, bname, kw):
    want = PASSES[case]
    g = passes.default_pipeline(builders.BUILDERS[bname](**kw))
    assert _describe(g) == want["nodes"]
    got_init = {k: hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest()
                for k, v in sorted(g.initializers.items())}
    assert got_init == want["initializers"]   # folded weights are bit-identical


@pytest.mark.parametrize("case,bname,kw", CASES, ids=[c[0] for c in CASES])
def test_oracle_matches_reference_executor(case, bname, kw):
    ref = golden(case)
    g = builders.BUILDERS[bname](**kw)
    feeds = builders.make_input(g, seed=0)
    raw = oref.run(g, feeds)
    post = oref.run(passes.default_pipeline(g.clone()), feeds)
    for o in g.outputs:
        want_raw, want_post = ref[f"raw.{o}"], ref[f"post.{o}"]
        if "mobilenetv2" in case:
            # grouped conv: one einsum over all groups vs the reference's loop per group
            np.testing.assert_allclose(raw[o], want_raw, rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(post[o], want_post, rtol=1e-5, atol=1e-5)
        else:
            np.testing.assert_array_equal(raw[o], want_raw)
            np.testing.assert_array_equal(post[o], want_post)
        assert np.abs(want_post).max() > 100 * 1e-4, "golden magnitude too small (vacuous)"


def test_round_bf16_is_rne():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-3, 3.4e38, np.inf], dtype=np.float32)
    r = oref.round_bf16(x)
    # 1 + 2^-8 is a tie between 1 and 1+2^-7: rounds to even (1.0)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.015625)
    assert np.isinf(r[5])
    import torch
    t = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(r[:5], t[:5])
