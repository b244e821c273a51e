"""INT8 executables on the B200 against the integer restatement (bit-exact).

The device quantises the fp32 feeds, runs the tcgen05 ``kind::i8`` convs with
the fixed-point (default) or fp32 requantisation epilogue, max-pools codes, requantises the global
average pool in fixed point and dequantises the logits. Every stored code and the fp32
logits must equal ``oracle.quant.run_int8`` evaluated under the executable's
own quantisation plan (calibrated on the GPU).
"""

import numpy as np
import pytest

import mdlc_b200
from mdlc_b200 import builders, passes
from mdlc_b200.compiler import Executable
from oracle import quant as oq
from oracle import reference as oref

pytestmark = pytest.mark.gpu

CASES = [
    ("conv_bn_relu", dict(n=2, cin=3, cout=16, h=12, w=12)),
    ("conv_bn_relu", dict(n=2, cin=32, cout=48, h=20, w=20, stride=2)),
    ("conv_bn_relu", dict(n=1, cin=64, cout=72, h=15, w=17, act="Relu6")),
    ("conv_bn_relu", dict(n=3, cin=16, cout=24, h=9, w=9, k=1, act=None)),
    ("residual_block", dict(n=2, c=16, h=16, w=16)),
    ("residual_block", dict(n=1, c=64, h=14, w=14)),
    ("mlp", dict(n=4, din=16, dh=32, dout=8)),
    ("resnet18", dict(batch=2, image=64)),
]


def _graph(name, kw):
    return passes.default_pipeline(builders.BUILDERS[name](**kw))


def _compare(exe, g, feeds):
    out = exe.run(feeds)
    want = oq.run_int8(g, exe.qplan, feeds)
    codes = exe.devices[0].read_tensors() if exe.keep_all else {}
    checked = 0
    for name, ref in want["__codes__"].items():
        if name not in codes:
            continue
        got = codes[name]
        ref = np.asarray(ref)
        if got.dtype in (np.uint8, np.int8):
            ref = ref.astype(np.int64)
            bad = np.argwhere(got.astype(np.int64) != ref)
            assert bad.size == 0, (f"{name}: {len(bad)} of {got.size} codes differ; first at {bad[0].tolist()}: "
                                   f"device {got[tuple(bad[0])]} oracle {ref[tuple(bad[0])]}")
        else:
            np.testing.assert_array_equal(got, ref.astype(np.float32), err_msg=name)
        checked += 1
    for o in g.outputs:
        np.testing.assert_array_equal(out[o], np.asarray(want[o], np.float32).reshape(out[o].shape), err_msg=o)
    return out, want, checked


@pytest.mark.parametrize("requant", ["fixed", "fp32"])
@pytest.mark.parametrize("name,kw", CASES, ids=[f"{n}-{i}" for i, (n, _) in enumerate(CASES)])
def test_int8_bit_exact_per_layer(name, kw, requant):
    """Every stored code and the logits, for both requantisation forms: the
    fixed-point multiplier + shift (the default, BASELINE config 3's form) and
    the fp32-scale opt-in."""
    g = _graph(name, kw)
    n = g.value_info[g.runtime_inputs[0]].shape[0]
    exe = Executable(g, dtype="int8", batch=n, keep_all=True, requant=requant)
    assert exe.qplan.requant == requant
    try:
        assert exe.fallbacks() == []
        feeds = builders.make_input(g, seed=11)
        out, _, checked = _compare(exe, g, feeds)
        assert checked >= 1
        # quantisation error only: the int8 result tracks the fp32 graph
        ref = oref.run(g, feeds)
        for o in g.outputs:
            rel = np.linalg.norm(out[o] - ref[o]) / max(np.linalg.norm(ref[o]), 1e-12)
            assert rel < 0.1, f"{o}: int8 vs fp32 relative error {rel:.3f}"
    finally:
        exe.close()


@pytest.fixture(scope="module")
def resnet18_int8_b1():
    g = _graph("resnet18", dict(batch=1))
    exe = mdlc_b200.compile(g, dtype="int8", batch=1)
    yield g, exe
    exe.close()


def test_int8_resnet18_224_b1_bit_exact(resnet18_int8_b1):
    """BASELINE config 3 at b=1: logits bit-exact against the integer oracle."""
    g, exe = resnet18_int8_b1
    feeds = builders.make_input(g, seed=5)
    out, want, _ = _compare(exe, g, feeds)
    ref = oref.run(g, feeds)["logits"]
    rel = np.linalg.norm(out["logits"] - ref) / np.linalg.norm(ref)
    assert rel < 0.1, f"int8 vs fp32 relative error {rel:.3f}"
    # the CUDA graph replays the same integer program
    ins = exe.pinned_inputs()
    ins["input"][...] = feeds["input"]
    exe.run_pinned(use_graph=True)
    np.testing.assert_array_equal(exe.pinned_outputs()["logits"], out["logits"])


def test_int8_resnet18_b1024_batch_invariance(resnet18_int8_b1):
    """BASELINE config 3 at b=1024: every image's logits are independent of the
    batch it runs in (rows of the b=1024 run equal the verified b=1 executable's
    under the same quantisation plan), so the b=1 oracle check covers them."""
    g1, exe1 = resnet18_int8_b1
    g = _graph("resnet18", dict(batch=1024))
    exe = mdlc_b200.compile(g, dtype="int8", batch=1024, calib=exe1.ranges)
    try:
        rng = np.random.default_rng(1024)
        x = rng.standard_normal((1024, 3, 224, 224), dtype=np.float32)
        out = exe.run({"input": x})["logits"]
        assert out.shape == (1024, 1000) and np.isfinite(out).all()
        for i in (0, 1, 255, 256, 600, 1023):
            one = exe1.run({"input": x[i:i + 1]})["logits"]
            np.testing.assert_array_equal(out[i:i + 1], one, err_msg=f"row {i}")
    finally:
        exe.close()


@pytest.mark.parametrize("shape", [(4, 256, 7, 7, 512, 3, 3, 1, 1), (2, 64, 20, 18, 200, 3, 3, 2, 1)],
                         ids=["512ch-7x7", "ragged-k200-s2"])
def test_int8_conv_same_bits_for_every_tile_config(shape):
    """An int8 conv (u8 codes x s8 weights, int32 accumulation, fp32 dequantised
    output) gives the same bits whichever tile configuration runs it, the
    192-wide tiles, the two-CTAs-per-SM ones and split-K (int32 partial sums)
    included: the integer sums are exact and the epilogue is per element."""
    from mdlc_b200 import _lib as L
    from mdlc_b200.tuner import ConvShape, _Bench
    ctx = L.Context(0)
    b = _Bench(ctx, ConvShape(*shape, dtype=L.U8))
    try:
        d = b.d
        rng = np.random.default_rng(7)
        x = rng.integers(0, 256, (d.n, d.h, d.w, d.c_stride), dtype=np.uint8)
        x[..., d.c:] = 0
        ctx.upload(b.x, x)
        outs = {}
        # (bn, stages, flags): tile configurations, and split-K into 2 and 7
        # slices (flags bits 8-15)
        for cfg in ((0, 0, 0), (256, 3, 0), (192, 3, 0), (128, 2, 0), (64, 3, 0), (128, 4, 0), (64, 8, 0),
                    (0, 0, 2 << 8), (64, 3, 7 << 8), (256, 3, 7 << 8)):
            b.run(L.TileCfg(bn=cfg[0], stages=cfg[1], flags=cfg[2]) if any(cfg) else None)
            ctx.sync()
            outs[cfg] = ctx.download(b.y, (d.n * d.oh * d.ow, d.k_stride), np.float32)[:, :d.k]
        ref = outs[(0, 0, 0)]
        assert np.isfinite(ref).all() and np.abs(ref).max() > 0
        for cfg, y in outs.items():
            np.testing.assert_array_equal(y, ref, err_msg=str(cfg))
    finally:
        b.close()
        ctx.close()
