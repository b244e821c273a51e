"""The stem rewrites, checked with the oracle's conv on CPU: the 2x2
space-to-depth form (a stride-2 conv over <= 4 channels becomes a stride-1
conv over 4x the channels) and the column pairing of that stride-1 conv (two
horizontally adjacent output pixels per GEMM row, over the same bytes read as
super-pixels of two input pixels)."""

import numpy as np
import pytest

from mdlc_b200 import lowering
from oracle import reference as oref


@pytest.mark.parametrize("S,pl,pr,C,cs,W", [(4, 2, 1, 12, 16, 112), (4, 2, 1, 12, 16, 14), (4, 1, 2, 12, 16, 10),
                                            (3, 1, 1, 8, 8, 12), (5, 2, 2, 3, 8, 16)])
def test_pair_weights_reproduce_the_conv(S, pl, pr, C, cs, W):
    rng = np.random.default_rng(S * 100 + W)
    N, H, K, R = 2, 6, 8, 4
    x = rng.standard_normal((N, C, H, W)).astype(np.float32)
    w = rng.standard_normal((K, C, R, S)).astype(np.float32)
    y = oref.conv(x, w, None, pads=[2, pl, 1, pr])
    ow = y.shape[3]
    assert ow % 2 == 0
    w2, s2, pl2 = lowering.pair_weights(w, cs, pl)
    assert w2.shape == (2 * K, 2 * cs, R, s2)
    # the same bytes: NHWC [N, H, W, cs] read as [N, H, W/2, 2cs]
    xn = np.zeros((N, H, W, cs), np.float32)
    xn[..., :C] = x.transpose(0, 2, 3, 1)
    xp = xn.reshape(N, H, W // 2, 2 * cs).transpose(0, 3, 1, 2)
    pr2 = (ow // 2 - 1) + s2 - W // 2 - pl2
    y2 = oref.conv(xp, w2, None, pads=[2, pl2, 1, pr2])
    # and the output [N, OH, OW/2, 2K] read back as [N, OH, OW, K]
    back = y2.transpose(0, 2, 3, 1).reshape(N, y.shape[2], ow, K).transpose(0, 3, 1, 2)
    np.testing.assert_allclose(back, y, rtol=1e-5, atol=1e-4)


def test_resnet18_stem_is_paired_space_to_depth():
    from mdlc_b200 import _lib as L
    from mdlc_b200 import builders, passes
    from mdlc_b200 import shapes as S
    g = passes.default_pipeline(builders.resnet18(batch=2, image=64))
    lo = lowering.lower(g, S.infer(g, None), L.BF16)
    stem = lo.steps[0]
    geom = lo.weights[stem.params["weight"]][0]
    assert stem.params.get("s2d") and stem.params.get("paired")
    # 7x7/2 over 3 channels -> 4x4/1 over 2x2 space-to-depth (16-channel pixels)
    # -> 4x3/1 over 32-channel super-pixels with 128 = 2 x 64 outputs
    assert (geom["r"], geom["s"], geom["c"], geom["cs"], geom["k"]) == (4, 3, 32, 32, 128)
    assert (geom["w"], geom["ow"], geom["pl"]) == (16, 16, 1)
    assert geom["flops"] == 2.0 * 2 * 32 * 32 * 64 * 3 * 49     # algorithmic work of the 7x7 node
    lo8 = lowering.lower(g, S.infer(g, None), L.U8)
    assert lo8.steps[0].params.get("s2d") and lo8.steps[0].params.get("paired")
    g8 = lo8.weights[lo8.steps[0].params["weight"]][0]
    assert (g8["cs"], g8["k"], g8["s"]) == (64, 128, 3)      # 32-byte int8 pixels -> 64-byte super-pixels
