"""Lowering of the data-movement / normalisation ops the reference GPU
executor bounced to the host (Softmax, Transpose, Concat, Pad,
BatchNormalization, Gemm transA=1; mdlc/codegen/cuda/emit.py:32-35): the
steps they become, with no GPU."""

import numpy as np
import pytest

from mdlc_b200 import _lib as L
from mdlc_b200 import lowering, passes
from mdlc_b200 import shapes as S
from mdlc_b200.builders import _Builder


def ops_graph(kind, seed=0):
    """Small graphs exercising one op each (inputs ~N(0,1))."""
    b = _Builder(f"ops_{kind}", seed)
    if kind == "bn":
        x = b.input("x", (2, 20, 9, 11))
        c = 20
        prm = [b.const(f"bn.{n}", v) for n, v in (("scale", b.rng.uniform(0.5, 1.5, c)), ("bias", b.rng.normal(0, 0.1, c)),
                                                  ("mean", b.rng.normal(0, 0.1, c)), ("var", b.rng.uniform(0.5, 1.5, c)))]
        y = b.node("BatchNormalization", [x] + prm, {"epsilon": 1e-5}, "bn")
        return b.finish(b.conv(y, c, 16, 3, name="conv"), "y")
    if kind == "softmax":
        x = b.input("x", (4, 37))
        return b.finish(b.node("Softmax", [b.fc(x, 37, 100)], {"axis": -1}, "softmax"), "y")
    if kind == "softmax4d":
        x = b.input("x", (2, 12, 5, 6))
        y = b.conv(x, 12, 20, 3, name="conv")
        return b.finish(b.node("Softmax", [y], {"axis": 1}, "softmax"), "y")
    if kind == "transpose":
        x = b.input("x", (2, 8, 5, 7))
        t = b.node("Transpose", [x], {"perm": [0, 1, 3, 2]}, "tr")
        return b.finish(b.conv(t, 8, 16, 3, name="conv"), "y")
    if kind in ("pad_constant", "pad_edge", "pad_reflect"):
        x = b.input("x", (2, 8, 6, 7))
        p = b.const("pads", np.array([0, 0, 1, 2, 0, 0, 2, 1], np.float32))
        t = b.node("Pad", [x, p], {"mode": kind.split("_")[1], "value": 0.5}, "pad")
        return b.finish(b.conv(t, 8, 16, 3, name="conv"), "y")
    if kind == "concat":
        x = b.input("x", (2, 8, 10, 10))
        u = b.relu(b.conv(x, 8, 12, 3, name="ca"))
        v = b.relu(b.conv(x, 8, 20, 1, name="cb"))
        t = b.node("Concat", [u, v], {"axis": 1}, "cat")
        return b.finish(b.conv(t, 32, 16, 3, name="conv"), "y")
    if kind == "gemm_transA":
        x = b.input("x", (24, 6))          # A is [K, M]: 24 x 6 -> y [6, 40]
        w = b.const("w", b.rng.standard_normal((40, 24)).astype(np.float32) * 0.2)
        return b.finish(b.node("Gemm", [x, w], {"transA": 1, "transB": 1}, "gemm"), "y")
    raise ValueError(kind)


KINDS = ["bn", "softmax", "softmax4d", "transpose", "pad_constant", "pad_edge", "pad_reflect", "concat",
         "gemm_transA"]


@pytest.mark.parametrize("kind", KINDS)
def test_ops_lower_without_host_fallback(kind):
    g = passes.default_pipeline(ops_graph(kind))
    lo = lowering.lower(g, S.infer(g, None), L.BF16)
    kinds = [st.kind for st in lo.steps]
    want = {"bn": "eltwise", "softmax": "softmax", "softmax4d": "softmax", "transpose": "copy",
            "pad_constant": "copy", "pad_edge": "copy", "pad_reflect": "copy", "concat": "copy",
            "gemm_transA": "copy"}[kind]
    assert want in kinds, kinds
    if kind == "concat":
        st = next(s for s in lo.steps if s.kind == "copy")
        assert [p["mode"] for p in st.params["parts"]] == [0, 1]
        assert [p["offset"][1] for p in st.params["parts"]] == [0, 12]
    if kind == "gemm_transA":
        assert kinds == ["copy", "conv"] and lo.steps[0].params["batch_mixing"]


def test_batch_mixing_ops_refuse_sharding():
    """A transpose of the batch axis cannot run on batch shards."""
    g = passes.default_pipeline(ops_graph("gemm_transA"))
    lo = lowering.lower(g, S.infer(g, None), L.BF16)
    assert any(st.params.get("batch_mixing") for st in lo.steps)
    g2 = passes.default_pipeline(ops_graph("transpose"))
    lo2 = lowering.lower(g2, S.infer(g2, None), L.BF16)
    assert not any(st.params.get("batch_mixing") for st in lo2.steps)


def test_bf16_constant_bits_round_to_nearest_even():
    """Elementwise constants of bf16 graphs are uploaded as bf16 bit patterns (RNE)."""
    import torch
    from mdlc_b200.compiler import _bf16_bits
    rng = np.random.default_rng(3)
    a = np.concatenate([rng.standard_normal(4096).astype(np.float32) * 100,
                        np.array([0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, np.inf, -np.inf], np.float32)])
    want = torch.from_numpy(a).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(_bf16_bits(a), want)
    assert _bf16_bits(np.array([np.nan], np.float32))[0] & 0x7FC0 == 0x7FC0


def test_squeeze_excite_fused_into_one_step():
    """RepViT's squeeze-excite gates (ReduceMean -> 1x1 conv + ReLU -> 1x1 conv
    + Sigmoid -> Mul) lower to one "se" step (the pool absorbed: it reads the
    activations themselves) and the multiply; the FC weights leave the conv
    weight table; keep_all lowering keeps the pool and the two convs."""
    from mdlc_b200 import builders
    g = passes.default_pipeline(builders.BUILDERS["repvit"](batch=2, seed=0))
    shp = S.infer(g, 2)
    lo = lowering.lower(g, shp, L.BF16)
    se = [st for st in lo.steps if st.kind == "se"]
    assert len(se) == 10
    for st in se:
        p = st.params
        rd, c = p["w1"].shape
        assert p["w2t"].shape == (rd, c) and p["b1"].shape == (rd,) and p["b2"].shape == (c,)
        assert (p["act1"], p["act2"]) == ("Relu", "Sigmoid")
        assert not any(n in w for n in st.nodes for w in lo.weights)
        # the activations and the gate keep the same channel stride
        x, y = lo.tensors[st.inputs[0]], lo.tensors[st.outputs[0]]
        assert x.cs == y.cs and x.h * x.w > 1 and y.h * y.w == 1
        assert len(st.nodes) == 3
    # only the head's global average pool is left as a pool step
    assert sum(st.kind == "pool" and st.params["kind"] == 2 for st in lo.steps) == 1
    # the second FC's weight, transposed, is the step's w2t
    node = {n.name: n for n in g.nodes}[se[0].nodes[-1]]
    rd, c = se[0].params["w1"].shape
    w2 = np.asarray(g.initializers[node.inputs[1]], np.float32).reshape(c, rd)
    np.testing.assert_array_equal(se[0].params["w2t"], w2.T)
    lo_all = lowering.lower(g, shp, L.BF16, fuse_se=False)
    assert not any(st.kind == "se" for st in lo_all.steps)
    assert sum(st.kind == "conv" for st in lo_all.steps) == sum(st.kind == "conv" for st in lo.steps) + 20
    assert sum(st.kind == "pool" and st.params["kind"] == 2 for st in lo_all.steps) == 11


def test_squeeze_excite_keeps_a_pool_with_other_readers():
    """A global average pool whose output another step also reads stays a pool
    step; the gate then reads the pooled map (mdlc_se_desc.hw == 1)."""
    from mdlc_b200 import builders
    g = passes.default_pipeline(builders.BUILDERS["repvit"](batch=2, seed=0))
    lo = lowering.lower(g, S.infer(g, 2), L.BF16, fuse_se=False)
    i = next(k for k, st in enumerate(lo.steps) if st.kind == "pool" and st.params["kind"] == 2)
    pooled = lo.steps[i].outputs[0]
    extra = lowering.Step("eltwise", [pooled], [pooled + "_copy"], ["extra_reader"], {})
    lo.steps.insert(i + 3, extra)
    lowering.fuse_squeeze_excite(lo)
    first = next(st for st in lo.steps if st.kind == "se")
    assert first.inputs == [pooled]
    assert lo.steps[i].kind == "pool" and lo.steps[i].outputs == [pooled]
    # every other gate still absorbed its pool
    se = [st for st in lo.steps if st.kind == "se"]
    assert len(se) == 10 and all(lo.tensors[st.inputs[0]].h > 1 for st in se[1:])
