"""INT8 scheme pieces on CPU: fixed-point helpers against exact integer
arithmetic, multiplier quantisation, plan construction, and the integer oracle
against the fp32 oracle (quantisation error only)."""

import math

import numpy as np
import pytest

from mdlc_b200 import _lib as L
from mdlc_b200 import builders, lowering, passes, quant
from mdlc_b200 import shapes as S
from oracle import quant as oq
from oracle import reference as oref


def _srdhm_exact(a, b):
    if a == b == -(1 << 31):
        return (1 << 31) - 1
    ab = a * b
    nudge = (1 << 30) if ab >= 0 else 1 - (1 << 30)
    t = ab + nudge
    return int(t / (1 << 31)) if abs(t) < (1 << 52) else (t // (1 << 31) if t >= 0 else -((-t) // (1 << 31)))


def _rdbpot_exact(x, e):
    mask = (1 << e) - 1
    rem = x & mask
    thr = (mask >> 1) + (1 if x < 0 else 0)
    return (x >> e) + (1 if rem > thr else 0)


def test_fixed_point_helpers_match_exact_integers():
    rng = np.random.default_rng(0)
    a = rng.integers(-(1 << 31), 1 << 31, 2000, dtype=np.int64)
    b = rng.integers(1 << 30, 1 << 31, 2000, dtype=np.int64)
    got = oq.srdhm(a, b)
    want = [(ai * bi + ((1 << 30) if ai * bi >= 0 else 1 - (1 << 30))) for ai, bi in zip(a.tolist(), b.tolist())]
    want = [w // (1 << 31) if w >= 0 else -((-w) // (1 << 31)) for w in want]
    np.testing.assert_array_equal(got, want)
    x = rng.integers(-(1 << 31), 1 << 31, 2000, dtype=np.int64)
    for e in (0, 1, 5, 13, 31):
        np.testing.assert_array_equal(oq.rdbpot(x, e), [_rdbpot_exact(v, e) for v in x.tolist()])
    # rounding half away from zero
    assert oq.rdbpot(np.int64(3), 1) == 2 and oq.rdbpot(np.int64(-3), 1) == -2
    assert oq.rdbpot(np.int64(5), 2) == 1 and oq.rdbpot(np.int64(-5), 2) == -1


@pytest.mark.parametrize("real", [0.5, 0.999999, 0.1234567, 3.1e-5, 1e-9, 1.0, 1.4274, 37.5])
def test_quantize_multiplier(real):
    m, sh = quant.quantize_multiplier(real)
    if real < 2.0 ** -32:
        assert (m, sh) == (0, 0) or m * 2.0 ** (-31 - sh) < 2 ** -31
        return
    assert (1 << 30) <= m < (1 << 31)
    assert abs(m * 2.0 ** (-31 - sh) - real) <= real * 2.0 ** -30
    # the integer requantisation approximates multiplication by `real`
    v = np.array([-20000, -7, 0, 5, 1234, 99999], np.int64)
    got = oq.requant(v, m, sh)
    assert np.all(np.abs(got - np.clip(v * real, -2**31, 2**31 - 1)) <= 1)


def test_act_qparams():
    s, zp = quant.act_qparams(0.0, 6.0)
    assert zp == 0 and math.isclose(float(s), 6.0 / 255, rel_tol=1e-6)
    s, zp = quant.act_qparams(-1.0, 3.0)
    assert zp == 64 and math.isclose(float(s), 4.0 / 255, rel_tol=1e-6)


def _plan(name, kw):
    g = passes.default_pipeline(builders.BUILDERS[name](**kw))
    shp = S.infer(g)
    lo_i8 = lowering.lower(g, shp, L.U8, s2d=True)
    for o in lo_i8.outputs:
        prod = [st for st in lo_i8.steps if o in st.outputs]
        if prod and prod[0].kind == "conv":
            lo_i8.tensors[o].dtype = L.F32
    lo_orig = lowering.lower(g, shp, L.U8, s2d=False)
    ranges = {}
    for i in range(4):
        feeds = builders.make_input(g, seed=100 + i)
        env = oref.run(g, feeds, return_all=True)
        for k, v in env.items():
            if k in g.initializers:
                continue
            v = np.asarray(v, np.float32)
            lo, hi = float(v.min()), float(v.max())
            if k in ranges:
                lo, hi = min(lo, ranges[k][0]), max(hi, ranges[k][1])
            ranges[k] = (lo, hi)
    return g, quant.build_plan(lo_orig, lo_i8, ranges, g)


def test_plan_structure_resnet18():
    g, plan = _plan("resnet18", dict(batch=1, image=64))
    assert len(plan.convs) == 21 and len(plan.gap) == 1
    for cq in plan.convs.values():
        assert np.all(np.abs(cq.w_q_orig) <= 127) and np.all(cq.w_q_orig == np.rint(cq.w_q_orig))
        assert cq.bias32.dtype == np.int32 and cq.rq_scale.dtype == np.float32
        if cq.deq_scale is None:
            assert np.all(cq.rq_scale > 0) and np.all(np.isfinite(cq.rq_scale))
    # the stem's space-to-depth, column-paired weights hold the same codes, once
    # for each of the two output columns of a row
    stem = next(c for w, c in plan.convs.items() if w.startswith("conv1"))
    assert stem.w_q.shape[:2] == (128, 64) and np.abs(stem.w_q).sum() == 2 * np.abs(stem.w_q_orig).sum()
    assert stem.bias32.shape == (64,)     # per-channel parameters keep the graph's K


@pytest.mark.parametrize("name,kw", [("conv_bn_relu", dict(n=2, cin=3, cout=16, h=12, w=12)),
                                     ("residual_block", dict(n=2, c=16, h=16, w=16)),
                                     ("mlp", dict(n=4, din=16, dh=32, dout=8)),
                                     ("resnet18", dict(batch=1, image=64))])
def test_int8_oracle_tracks_fp32(name, kw):
    g, plan = _plan(name, kw)
    feeds = builders.make_input(g, seed=7)
    ref = oref.run(g, feeds)
    got = oq.run_int8(g, plan, feeds)
    for o in g.outputs:
        y = got[o]
        if y.dtype != np.float32:     # uint8 codes: dequantise
            s, zp = plan.tensors[o]
            y = (y - zp) * np.float32(s)
        want = ref[o]
        rel = np.linalg.norm(y - want) / np.linalg.norm(want)
        assert rel < 0.1, f"int8 vs fp32 relative error {rel:.3f}"


def test_shared_shift_multipliers():
    """M1, M2 represent the real multipliers to 31 significant bits of the
    larger one, with one shift per channel."""
    rng = np.random.default_rng(3)
    real = np.exp(rng.uniform(np.log(1e-6), np.log(0.9), 64))
    for rres in (None, 0.013, 1.7):
        m1, m2, sh = quant.shared_shift_multipliers(real, rres)
        assert m1.dtype == np.int32 and sh.min() >= 1 and sh.max() <= 62
        for k in range(64):
            big = max(real[k], rres or 0.0)
            assert (1 << 30) <= max(int(m1[k]), int(m2[k])) < (1 << 31)
            assert abs(int(m1[k]) / 2.0 ** int(sh[k]) - real[k]) <= 0.5 / 2.0 ** int(sh[k])
            if rres:
                assert abs(int(m2[k]) / 2.0 ** int(sh[k]) - rres) <= 0.5 / 2.0 ** int(sh[k])
            assert abs(max(int(m1[k]), int(m2[k])) / 2.0 ** int(sh[k]) - big) <= big * 2.0 ** -30


def test_fixed_point_requant_is_one_rounding_of_the_exact_value():
    """The oracle's fixed-point step equals floor(exact + 1/2) of the rational
    (acc*M1 + r*M2) / 2^S computed with Python integers."""
    from fractions import Fraction
    g, plan = _plan("resnet18", dict(batch=1, image=64))
    assert plan.requant == "fixed"
    cq = next(c for c in plan.convs.values() if c.residual and c.rq_mult is not None)
    rng = np.random.default_rng(5)
    k = cq.rq_mult.shape[0]
    acc = rng.integers(-(1 << 24), 1 << 24, (3, k), dtype=np.int64)
    res = rng.integers(-128, 128, (3, k), dtype=np.int64)
    m1, m2, sh = (cq.rq_mult.astype(np.int64), cq.rq_res_mult.astype(np.int64), cq.rq_shift.astype(np.int64))
    got = (acc * m1 + res * m2 + (np.int64(1) << (sh - 1))) >> sh
    for i in range(3):
        for j in range(k):
            exact = Fraction(int(acc[i, j]) * int(m1[j]) + int(res[i, j]) * int(m2[j]), 1 << int(sh[j]))
            assert got[i, j] == math.floor(exact + Fraction(1, 2))


@pytest.mark.parametrize("name,kw", [("residual_block", dict(n=2, c=16, h=16, w=16)),
                                     ("resnet18", dict(batch=1, image=64))])
def test_fixed_and_fp32_requant_agree_within_one_code(name, kw):
    g = passes.default_pipeline(builders.BUILDERS[name](**kw))
    _, plan_fx = _plan(name, kw)
    shp = S.infer(g)
    lo_i8 = lowering.lower(g, shp, L.U8, s2d=True)
    for o in lo_i8.outputs:
        prod = [st for st in lo_i8.steps if o in st.outputs]
        if prod and prod[0].kind == "conv":
            lo_i8.tensors[o].dtype = L.F32
    lo_orig = lowering.lower(g, shp, L.U8, s2d=False)
    ranges = {t: plan_fx.tensors[t] for t in plan_fx.tensors}
    feeds = builders.make_input(g, seed=9)
    # the same ranges -> same scales; only the requantisation arithmetic differs
    env = oref.run(g, feeds, return_all=True)
    rng_ = {kk: (float(np.asarray(v).min()), float(np.asarray(v).max())) for kk, v in env.items()
            if kk not in g.initializers}
    p_fx = quant.build_plan(lo_orig, lo_i8, rng_, g, requant="fixed")
    p_fp = quant.build_plan(lo_orig, lo_i8, rng_, g, requant="fp32")
    a = oq.run_int8(g, p_fx, feeds)["__codes__"]
    b = oq.run_int8(g, p_fp, feeds)["__codes__"]
    # the first requantised layer sees identical inputs: its codes differ by <= 1
    first = next(st.outputs[0] for st in p_fx.steps if st.kind == "conv")
    d = np.abs(np.asarray(a[first], np.int64) - np.asarray(b[first], np.int64))
    assert d.max() <= 1 and d.mean() < 0.01
    del ranges
