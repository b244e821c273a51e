"""The reference-facing boundary of ``compile()``, checked on CPU.

* ``mem_plan=``: the reference ``MemoryPlan`` (its tensor -> buffer assignment,
  committed in ``tests/golden/memplan.json`` from the reference's own
  ``plan_memory``) laid out as the backend arena, with no two live tensors
  sharing memory under the backend's fused steps.
* ``schedule_fn=``: the reference hook ``schedule_fn(node, (M, N, K))`` called
  with the reference codegen's (M, N, K) per node and its tile mapped to the
  kernel's tile width.
* The reference's own ``Graph`` (from its ``default_pipeline()``) accepted by
  the lowering and shape path (skipped where the reference is not mounted).
"""

import json
import os
import sys
from dataclasses import dataclass

import numpy as np
import pytest

from conftest import GOLDEN
from mdlc_b200 import _lib as L
from mdlc_b200 import builders, lowering, memory, passes
from mdlc_b200 import shapes as S
from mdlc_b200 import tuner as T

with open(os.path.join(GOLDEN, "memplan.json")) as f:
    MEMPLAN = json.load(f)

CASES = {
    "conv_bn_relu": ("conv_bn_relu", dict(n=2, cin=3, cout=8, h=10, w=10)),
    "residual_block": ("residual_block", dict(n=2, c=8, h=8, w=8)),
    "mlp": ("mlp", dict()),
    "resnet18_b1": ("resnet18", dict(batch=1, image=224)),
    "resnet18_s64_b2": ("resnet18", dict(batch=2, image=64)),
    "mobilenetv2_b1": ("mobilenetv2", dict(batch=1, image=224)),
}


def _lowered(bname, kw, dtype=L.BF16):
    g = passes.default_pipeline(builders.BUILDERS[bname](**kw))
    return g, lowering.lower(g, S.infer(g, None), dtype)


@pytest.mark.parametrize("case", sorted(CASES))
def test_reference_memory_plan_honoured_and_safe(case):
    bname, kw = CASES[case]
    _, lo = _lowered(bname, kw)
    ref = MEMPLAN[case]["assignment"]
    plan = memory.plan_from_reference(lo.steps, lo.tensors, lo.inputs, lo.outputs, ref)
    assert memory.conflicts(plan, lo.steps, lo.tensors, lo.inputs, lo.outputs) == []
    # tenants of one reference buffer share one region unless a note says why not
    moved = {n.split("'")[1] for n in plan.notes if "moved out of" in n}
    by_buf = {}
    for name, bid in ref.items():
        if name in plan.offsets and name not in moved:
            by_buf.setdefault(bid, set()).add(plan.offsets[name])
    assert by_buf and all(len(offs) == 1 for offs in by_buf.values()), by_buf
    # distinct reference buffers never share a region
    region = {bid: next(iter(offs)) for bid, offs in by_buf.items()}
    assert len(set(region.values())) == len(region)
    # every activation the backend stores has a place; graph inputs their own
    live = memory.liveness(lo.steps, lo.tensors, lo.inputs, lo.outputs)
    assert set(live) == set(plan.offsets)
    for i in lo.inputs:
        assert plan.offsets[i] not in region.values()
    assert "reference buffers honoured" in plan.report()


def test_reference_plan_moves_only_what_fusion_needs():
    """ResNet-18: the reference plans over IR nodes, where a block's residual
    Add runs after its conv; fused here, the conv reads its input while writing
    the Add's output, so the reference sharing of those two (if any) is split.
    Every move is such a case: the moved tensor is live together with an
    earlier tenant of its reference buffer under the backend steps."""
    _, lo = _lowered("resnet18", dict(batch=1, image=224))
    ref = MEMPLAN["resnet18_b1"]["assignment"]
    plan = memory.plan_from_reference(lo.steps, lo.tensors, lo.inputs, lo.outputs, ref)
    live = memory.liveness(lo.steps, lo.tensors, lo.inputs, lo.outputs)
    for note in plan.notes[1:]:
        moved, other = note.split("'")[1], note.split("'")[3]
        assert ref[moved] == ref[other]
        (f0, l0), (f1, l1) = live[moved], live[other]
        assert f0 <= l1 and f1 <= l0
    # the backend's own planner is safe too, and no larger than the naive layout
    own = memory.plan_arena(lo.steps, lo.tensors, lo.inputs, lo.outputs)
    assert memory.conflicts(own, lo.steps, lo.tensors, lo.inputs, lo.outputs) == []
    assert own.total_bytes <= own.naive_bytes


def test_conflict_checker_finds_a_planted_overlap():
    """The checker is not vacuous: putting a step's output on its own input's
    memory is reported."""
    _, lo = _lowered("conv_bn_relu", dict(n=2, cin=3, cout=8, h=10, w=10))
    plan = memory.plan_arena(lo.steps, lo.tensors, lo.inputs, lo.outputs)
    x, y = lo.steps[0].inputs[0], lo.steps[0].outputs[0]
    assert memory.conflicts(plan, lo.steps, lo.tensors, lo.inputs, lo.outputs) == []
    plan.offsets[y] = plan.offsets[x]
    bad = memory.conflicts(plan, lo.steps, lo.tensors, lo.inputs, lo.outputs)
    assert {frozenset(p) for p in bad} == {frozenset((x, y))}


@dataclass(frozen=True)
class _GemmSchedule:
    """Duck type of the reference's GemmSchedule (mdlc/codegen/schedule.py:16-31)."""
    BM: int = 64
    BN: int = 64
    BK: int = 16
    TM: int = 4
    TN: int = 4


def test_schedule_fn_gets_reference_mnk_and_maps_the_channel_tile():
    g, lo = _lowered("resnet18", dict(batch=1, image=224))
    calls = []

    def fn(node, mnk):
        calls.append((node, mnk))
        return _GemmSchedule(BM=128, BN=32)

    geoms = [lo.weights[st.params["weight"]][0] for st in lo.steps if st.kind == "conv"]
    stem, fc = geoms[0], geoms[-1]
    # reference codegen: conv (OC, OH*OW, C*KH*KW) (emit.py:202), Gemm (M, N, K) (emit.py:225)
    assert stem["ref_mnk"] == (64, 112 * 112, 3 * 7 * 7)
    assert fc["ref_mnk"] == (1, 1000, 512)
    assert T.from_reference_schedule(fn, "stem", stem) == (128, 0)      # conv: BM tiles output channels
    assert T.from_reference_schedule(fn, "fc", fc) == (64, 0)           # GEMM: BN (32 -> 64)
    assert calls == [("stem", (64, 12544, 147)), ("fc", (1, 1000, 512))]
    assert T.from_reference_schedule(lambda n, m: _GemmSchedule(BM=512), None, stem) == (256, 0)
    assert T.from_reference_schedule(lambda n, m: (192, 3), None, stem) == (192, 3)
    assert T.from_reference_schedule(lambda n, m: None, None, stem) is None


REF_ROOT = os.environ.get("MDLC_REFERENCE", "/root/reference")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_ROOT, "mdlc")), reason="reference source not mounted")
def test_reference_graph_through_lowering_and_hooks():
    """The reference's own Graph, after its own default_pipeline(), passes the
    backend's shape inference and lowering, and the reference's own Tuner works
    as schedule_fn; the resulting steps match the backend's restated pipeline."""
    sys.path.insert(0, REF_ROOT)
    sys.path.insert(0, GOLDEN)
    import mdlc.ir as ref_ir
    from make_golden import to_reference_graph
    from mdlc.autotuner.tuner import Tuner
    from mdlc.passes import default_pipeline
    from mdlc.runtime.memory_planner import plan_memory
    from mdlc.passes.shape_inference import infer_shapes_by_execution

    g = builders.resnet18(batch=1, image=64)
    rg = default_pipeline().run(to_reference_graph(g, ref_ir))
    lo = lowering.lower(rg, S.infer(rg, None), L.BF16)
    _, mine = _lowered("resnet18", dict(batch=1, image=64))
    assert [st.label() for st in lo.steps] == [st.label() for st in mine.steps]
    for name, (geom, wt, bias) in lo.weights.items():
        np.testing.assert_array_equal(wt, mine.weights[name][1])
    tuner = Tuner()
    geom = [lo.weights[st.params["weight"]][0] for st in lo.steps if st.kind == "conv"][1]
    bn, stages = T.from_reference_schedule(tuner, None, geom)
    assert bn in T.TILE_WIDTHS and stages == 0
    infer_shapes_by_execution(rg, builders.make_input(g, seed=0))
    rplan = plan_memory(rg)
    plan = memory.plan_from_reference(lo.steps, lo.tensors, lo.inputs, lo.outputs, rplan)
    assert memory.conflicts(plan, lo.steps, lo.tensors, lo.inputs, lo.outputs) == []
