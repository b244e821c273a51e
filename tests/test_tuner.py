"""Autotuner host logic (no GPU): the analytical ranking, the JSON cache and the
``tuner(kind, geom)`` hook contract (the reference's ``schedule_fn``,
mdlc/codegen/cuda/emit.py:27,100; cache and search, mdlc/autotuner/tuner.py:60-174)."""

import json

from mdlc_b200 import _lib as L
from mdlc_b200 import tuner as T


def _best(shape):
    cfg, _, ranking = T.tune(shape)          # no context: modeled
    assert [c for c, _ in ranking] and cfg == ranking[0][0]
    return cfg


def test_every_config_is_ranked_and_known():
    shape = T.ConvShape(8, 64, 28, 28, 64, 3, 3, 1, 1)
    _, _, ranking = T.tune(shape)
    assert sorted(c for c, _ in ranking) == sorted(T.CONFIGS)
    assert all(cfg in T.CTAS_PER_SM for cfg in T.CONFIGS)


def test_model_prefers_two_ctas_per_sm_for_narrow_layers():
    # ResNet-18 layers at b=256: narrow tiles are issue-bound with one CTA per SM
    assert _best(T.ConvShape(256, 64, 56, 56, 64, 3, 3, 1, 1)) == (64, 3)
    assert _best(T.ConvShape(256, 128, 28, 28, 128, 3, 3, 1, 1)) == (128, 2)
    # wide layers keep 256-wide tiles (the MMA covers the issuer's gaps)
    assert _best(T.ConvShape(256, 256, 14, 14, 256, 3, 3, 1, 1)) == (256, 3)
    assert _best(T.ConvShape(256, 512, 7, 7, 512, 3, 3, 1, 1)) == (256, 3)


def test_model_fp32_prefers_the_deeper_rings():
    # 3xTF32 runs one CTA per SM in every configuration, so the model follows the
    # ring depth, as measured on ResNet-18 fp32 b=256 (layer1 (64, 4), 128- and
    # 512-channel layers (128, 3))
    f32 = dict(dtype=L.F32)
    assert _best(T.ConvShape(256, 64, 56, 56, 64, 3, 3, 1, 1, **f32)) == (64, 4)
    assert _best(T.ConvShape(256, 128, 28, 28, 128, 3, 3, 1, 1, **f32)) == (128, 3)
    _, _, ranking = T.tune(T.ConvShape(8, 64, 28, 28, 64, 3, 3, 1, 1, **f32))
    assert sorted(c for c, _ in ranking) == sorted(T.CONFIGS_F32)


def test_model_counts_waves():
    shape = T.ConvShape(1, 512, 7, 7, 512, 3, 3, 1, 1)   # 1 M tile: only N tiles spread the work
    assert T.analytical_cost(shape, 64, 8) < T.analytical_cost(shape, 256, 3)


def test_cache_round_trip(tmp_path):
    path = tmp_path / "cache.json"
    c = T.TuneCache(str(path))
    shape = T.ConvShape(2, 64, 14, 14, 64, 3, 3, 1, 1)
    assert c.get(shape.key()) is None
    c.put(shape.key(), (64, 3), 1.5, False)
    c.save()
    assert json.loads(path.read_text())[shape.key()]["cfg"] == [64, 3]
    assert T.TuneCache(str(path)).get(shape.key()) == (64, 3)
    assert T.KERNEL_TAG in shape.key()


def test_hook_contract(tmp_path):
    tuner = T.Tuner(T.TuneCache(str(tmp_path / "c.json")))
    geom = dict(n=256, c=64, h=56, w=56, k=64, r=3, s=3, sh=1, sw=1, pt=1, pl=1, dh=1, groups=1, dtype=L.BF16)
    assert tuner("conv", geom) == (64, 3)
    assert tuner.cache.get(T.ConvShape(256, 64, 56, 56, 64, 3, 3, 1, 1).key()) == (64, 3)
    assert tuner("conv", dict(geom, groups=64)) is None        # depthwise: not a tensor-core conv
    assert tuner("pool", geom) is None
    assert tuner("conv", dict(geom, dh=2)) is None             # dilation: heuristic default
