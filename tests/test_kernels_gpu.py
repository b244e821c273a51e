"""Kernel-level parity through the C ABI (``libmdlc_b200.so``) against the oracle.

Each case builds NCHW fp32 inputs and OIHW weights, packs them through the
library's own packer, runs one entry point on ``cuda:0`` and compares with
:mod:`oracle.reference` evaluated on the *same* operands (bf16-rounded for the
bf16 kernels, so the remaining difference is fp32 accumulation order plus the
final bf16 rounding of the output).
"""

import numpy as np
import pytest

from oracle import reference as oref

from mdlc_b200 import _lib as L

pytestmark = pytest.mark.gpu


def bf16_bits(x):
    return (oref.round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def nhwc(x, cs):
    n, c, h, w = x.shape
    out = np.zeros((n, h, w, cs), dtype=x.dtype)
    out[..., :c] = x.transpose(0, 2, 3, 1)
    return out


@pytest.fixture(scope="module")
def ctx():
    c = L.Context(0)
    yield c
    c.close()


def _rnd8(v):
    return (v + 7) // 8 * 8


def run_conv(ctx, x, w, b, *, stride=1, pad=0, dil=1, groups=1, dtype="bf16", act=L.ACT_NONE,
             res=None, out_f32=False, cfg=None, clip=(0.0, 6.0), flags=0):
    n, c, h, wd = x.shape
    k, _, r, s = w.shape
    oh = (h + 2 * pad - dil * (r - 1) - 1) // stride + 1
    ow = (wd + 2 * pad - dil * (s - 1) - 1) // stride + 1
    cs, ks = _rnd8(c), _rnd8(k)
    et = L.BF16 if dtype == "bf16" else L.F32
    ot = L.F32 if (out_f32 or dtype == "f32") else L.BF16
    d = L.ConvDesc(n=n, h=h, w=wd, c=c, c_stride=cs, k=k, k_stride=ks, r=r, s=s, stride_h=stride,
                   stride_w=stride, pad_t=pad, pad_l=pad, dil_h=dil, dil_w=dil, oh=oh, ow=ow,
                   groups=groups, in_type=et, out_type=ot, res_stride=0, in_zp=0)
    wp = L.pack_weights(d, w)
    xh = nhwc(x, cs)
    xd = ctx.to_device(bf16_bits(xh) if et == L.BF16 else xh.astype(np.float32))
    wd_ = ctx.to_device(wp)
    bias = np.zeros(ks, np.float32)
    bias[:k] = b
    bd = ctx.to_device(bias)
    rd = 0
    if res is not None:
        rh = nhwc(res, ks)
        rd = ctx.to_device(bf16_bits(rh) if et == L.BF16 else rh.astype(np.float32))
    ebytes = 4 if ot == L.F32 else 2
    yd = ctx.alloc(n * oh * ow * ks * ebytes)
    ctx.memset(yd, 0xFF, n * oh * ow * ks * ebytes)   # poison: every element must be written
    epi = L.Epilogue(act=act, alpha=0.01, beta=0.5, clip_lo=clip[0], clip_hi=clip[1])
    tc = L.TileCfg(bn=cfg[0] if cfg else 0, stages=cfg[1] if cfg else 0, flags=flags) if (cfg or flags) else None
    ctx.conv2d(d, xd, wd_, bd, rd, yd, epi, tc)
    ctx.sync()
    if ot == L.F32:
        y = ctx.download(yd, (n, oh, ow, ks), np.float32)
    else:
        y = from_bf16_bits(ctx.download(yd, (n, oh, ow, ks), np.uint16))
    for p in (xd, wd_, bd, yd) + ((rd,) if rd else ()):
        ctx.free(p)
    assert np.all(y[..., k:] == 0), "padding channels must be written as zero"
    return y[..., :k].transpose(0, 3, 1, 2)


def oracle_conv(x, w, b, *, stride=1, pad=0, dil=1, groups=1, act=None, res=None, bf16=True, clip=(0.0, 6.0)):
    if bf16:
        x, w = oref.round_bf16(x), oref.round_bf16(w)
        res = None if res is None else oref.round_bf16(res)
    y = oref.conv(x, w, b, strides=[stride, stride], pads=[pad] * 4, dilations=[dil, dil], group=groups)
    if res is not None:
        y = y + res
    return oref.activation(act, y, {"clip_min": clip[0], "clip_max": clip[1], "alpha": 0.01, "beta": 0.5})


def check(got, want, rel):
    err = np.abs(got - want).max()
    scale = max(np.abs(want).max(), 1e-6)
    assert err <= rel * scale, f"max err {err:.3e} vs scale {scale:.3e} (rel {err / scale:.2e} > {rel})"


CONV_CASES = [
    # n, c, h, w, k, r, stride, pad, dil
    (1, 64, 14, 14, 64, 3, 1, 1, 1),
    (2, 64, 9, 11, 128, 3, 1, 1, 1),
    (2, 128, 7, 7, 256, 3, 1, 1, 1),
    (2, 256, 7, 7, 512, 3, 2, 1, 1),
    (3, 3, 23, 23, 64, 7, 2, 3, 1),       # stem-like, c=3 padded to 8
    (2, 64, 15, 15, 128, 1, 2, 0, 1),     # 1x1 stride-2 projection
    (1, 24, 10, 10, 40, 3, 1, 2, 2),      # dilation, ragged channels
    (5, 512, 1, 1, 1000, 1, 1, 0, 1),     # FC as 1x1 conv (k=1000 not a tile multiple)
    (1, 16, 5, 5, 8, 3, 1, 1, 1),         # tiny
]


@pytest.mark.parametrize("case", CONV_CASES, ids=[str(c) for c in CONV_CASES])
def test_conv_bf16_tcgen05(ctx, case):
    n, c, h, w, k, r, st, pad, dil = case
    rng = np.random.default_rng(sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    got = run_conv(ctx, x, wt, b, stride=st, pad=pad, dil=dil, act=L.ACT_RELU)
    want = oracle_conv(x, wt, b, stride=st, pad=pad, dil=dil, act="Relu")
    check(got, want, 1e-2)


EPI_ACTS = [
    # activation code, clip bounds, oracle activation name
    (L.ACT_NONE, (0.0, 6.0), None),
    (L.ACT_RELU, (0.0, 6.0), "Relu"),
    (L.ACT_CLIP, (0.0, 6.0), "Clip"),      # ReLU6: bounds exact in bf16 -> packed-pair clamp
    (L.ACT_CLIP, (-0.75, 1.5), "Clip"),    # exact, lower bound below zero
    (L.ACT_CLIP, (0.1, 2.0), "Clip"),      # 0.1 is not a bf16 value -> per-element fp32 clamp
    (L.ACT_GELU, (0.0, 6.0), "Gelu"),
    (L.ACT_SIGMOID, (0.0, 6.0), "Sigmoid"),
]


@pytest.mark.parametrize("k", [40, 72, 128])
@pytest.mark.parametrize("act", range(len(EPI_ACTS)))
def test_conv_bf16_epilogue_activations(ctx, act, k):
    """bf16 epilogue: bias + residual by paired fp32 adds, clamp activations on
    packed bf16 pairs (or per element when a bound is not exact in bf16), padding
    columns of a chunk past k zeroed (k = 40, 72: ragged 64-column chunks)."""
    code, clip, name = EPI_ACTS[act]
    n, c, h, w = 2, 32, 9, 10
    rng = np.random.default_rng(300 + 7 * act + k)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, 3, 3)) * np.sqrt(2.0 / (c * 9))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.2).astype(np.float32)
    res = rng.standard_normal((n, k, h, w)).astype(np.float32)
    got = run_conv(ctx, x, wt, b, stride=1, pad=1, act=code, res=res, clip=clip)
    want = oracle_conv(x, wt, b, stride=1, pad=1, act=name, res=res, clip=clip)
    check(got, want, 1e-2)
    if code == L.ACT_CLIP:
        assert got.min() >= clip[0] - 1e-6 and got.max() <= clip[1] + 1e-6


@pytest.mark.parametrize("cfg", [(64, 3), (128, 2), (256, 3), (192, 3), (64, 8), (128, 4)])
def test_conv_bf16_tile_configs(ctx, cfg):
    """Every tile configuration the tuner may pick gives the same answer (odd M, k tail)."""
    rng = np.random.default_rng(7)
    x = rng.standard_normal((3, 96, 13, 13)).astype(np.float32)
    wt = (rng.standard_normal((200, 96, 3, 3)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(200) * 0.1).astype(np.float32)
    res = rng.standard_normal((3, 200, 13, 13)).astype(np.float32)
    got = run_conv(ctx, x, wt, b, pad=1, act=L.ACT_RELU, res=res, cfg=cfg)
    want = oracle_conv(x, wt, b, pad=1, act="Relu", res=res)
    check(got, want, 1e-2)


IM2COL_CASES = [
    # n, c, h, w, k, r, stride, pad, dil  (inputs >= 128 KiB, c % 64 == 0: im2col-mode TMA)
    (4, 64, 32, 32, 64, 3, 1, 1, 1),
    (2, 128, 20, 21, 256, 3, 2, 1, 1),
    (3, 64, 17, 19, 128, 1, 2, 0, 1),
    (2, 256, 11, 9, 512, 3, 1, 1, 1),
    (2, 64, 23, 23, 64, 3, 1, 2, 2),
    (5, 192, 7, 7, 200, 3, 1, 1, 1),
    (8, 16, 40, 40, 64, 4, 1, 2, 1),      # c = 16: one 32-byte pixel per load (SW32 A tiles)
    (8, 16, 30, 30, 96, 1, 1, 0, 1),      # c = 16, 1x1: three padding taps per k-block
    (6, 32, 33, 31, 128, 3, 2, 1, 1),     # c = 32: 64-byte pixels (SW64 A tiles), stride 2
]


@pytest.mark.parametrize("case", IM2COL_CASES, ids=[str(c) for c in IM2COL_CASES])
def test_conv_im2col_tma_matches_gather(ctx, case):
    """The TMA im2col A operand and the cp.async gather load identical tiles, so
    the outputs are bit-identical; both match the oracle."""
    n, c, h, w, k, r, st, pad, dil = case
    rng = np.random.default_rng(100 + sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    oh = (h + 2 * pad - dil * (r - 1) - 1) // st + 1
    ow = (w + 2 * pad - dil * (r - 1) - 1) // st + 1
    res = rng.standard_normal((n, k, oh, ow)).astype(np.float32)
    tma = run_conv(ctx, x, wt, b, stride=st, pad=pad, dil=dil, act=L.ACT_RELU, res=res)
    gather = run_conv(ctx, x, wt, b, stride=st, pad=pad, dil=dil, act=L.ACT_RELU, res=res, flags=1)
    want = oracle_conv(x, wt, b, stride=st, pad=pad, dil=dil, act="Relu", res=res)
    scale = np.abs(want).max()
    bad_t = np.abs(tma - want).max(axis=1) > 1e-2 * scale          # (n, oh, ow) pixels that are wrong
    bad_g = np.abs(gather - want).max(axis=1) > 1e-2 * scale
    if bad_t.any() or bad_g.any():
        m_t = np.flatnonzero(bad_t.reshape(-1))
        print(f"TMA wrong pixels: {bad_t.sum()} / {bad_t.size}, first m {m_t[:20]}, tiles {np.unique(m_t // 128)[:20]}")
        print(f"gather wrong pixels: {bad_g.sum()}")
    check(gather, want, 1e-2)
    check(tma, want, 1e-2)
    np.testing.assert_array_equal(tma, gather)


POINTWISE_CASES = [
    # n, c, h, w, k   (1x1, stride 1, no padding: A by 2-D tiled TMA of the [M, cs] matrix)
    (4, 24, 28, 28, 144),     # MobileNetV2 expand: 24 channels (48-byte rows), one partial k-block
    (2, 56, 30, 30, 112),     # RepViT widths: 56 of 64 channels, ragged last M tile
    (2, 112, 14, 15, 56),     # two k-blocks, the second partial
    (3, 512, 1, 1, 1000),     # FC as a 1x1 conv over 1x1 images
]


@pytest.mark.parametrize("case", POINTWISE_CASES, ids=[str(c) for c in POINTWISE_CASES])
def test_conv_pointwise_tma_matches_gather(ctx, case):
    """Pointwise convs load A as a plain 2-D tile of the activation matrix
    (channels past cs read as zero); the result equals the cp.async gather's
    bit for bit and the oracle within tolerance."""
    n, c, h, w, k = case
    rng = np.random.default_rng(300 + sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, 1, 1)) * np.sqrt(2.0 / c)).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    res = rng.standard_normal((n, k, h, w)).astype(np.float32)
    tma = run_conv(ctx, x, wt, b, act=L.ACT_RELU, res=res)
    gather = run_conv(ctx, x, wt, b, act=L.ACT_RELU, res=res, flags=1)
    want = oracle_conv(x, wt, b, act="Relu", res=res)
    check(tma, want, 1e-2)
    np.testing.assert_array_equal(tma, gather)


HALO_CASES = [
    # n, c, h, w, k, r, pad   (stride 1, output >= 14x14: the halo-band main loop)
    (4, 16, 40, 40, 64, 4, 2),       # 32-byte pixels (the space-to-depth stem shape)
    (2, 32, 30, 26, 96, 3, 1),       # 64-byte pixels, ragged tiles
    (2, 16, 20, 20, 32, 5, 2),       # 32-byte pixels, 25 taps: the last k-block half padding
    (2, 64, 56, 56, 64, 3, 1),       # ResNet-18 layer1 (128-byte blocks on request)
    (2, 64, 20, 30, 128, 3, 1),      # ragged tile grid (12 of 16 rows, 6 of 8 columns in the last tiles)
    (1, 128, 28, 28, 128, 3, 1),     # two channel blocks per band
    (1, 256, 14, 14, 256, 3, 1),     # four channel blocks, 256-wide tiles
    (2, 64, 17, 15, 64, 5, 2),       # 5x5: the tallest band
    (1, 64, 16, 18, 64, 3, 0),       # no padding
]


@pytest.mark.parametrize("case", HALO_CASES, ids=[str(c) for c in HALO_CASES])
def test_conv_halo_band_matches_per_tap_paths(ctx, case):
    """Stride-1 convs read each input band once and every tap from shared memory
    (halo mode); the result matches the per-tap im2col-TMA and cp.async paths
    (bit for bit with one channel block, where the accumulation order is the
    same) and the oracle."""
    n, c, h, w, k, r, pad = case
    rng = np.random.default_rng(200 + sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    oh, ow = h + 2 * pad - r + 1, w + 2 * pad - r + 1
    res = rng.standard_normal((n, k, oh, ow)).astype(np.float32)
    halo = run_conv(ctx, x, wt, b, pad=pad, act=L.ACT_RELU, res=res, flags=4)
    per_tap = run_conv(ctx, x, wt, b, pad=pad, act=L.ACT_RELU, res=res, flags=2)
    gather = run_conv(ctx, x, wt, b, pad=pad, act=L.ACT_RELU, res=res, flags=1)
    want = oracle_conv(x, wt, b, pad=pad, act="Relu", res=res)
    check(halo, want, 1e-2)
    check(per_tap, want, 1e-2)
    np.testing.assert_array_equal(per_tap, gather)
    if c <= 64:   # one band per tile: same accumulation order as the per-tap loads
        np.testing.assert_array_equal(halo, per_tap)
    if c % 64 == 0 and k <= 64 and c * r * r <= 9 * 64:
        # the weights resident in shared memory: same products in the same order
        resident = run_conv(ctx, x, wt, b, pad=pad, act=L.ACT_RELU, res=res, flags=8)
        np.testing.assert_array_equal(resident, halo)


RESIDENT_CASES = [
    # n, c, h, w, k, act, residual   (64 input channels, 3x3, stride 1: the resident-weight halo path)
    (4, 64, 56, 56, 64, L.ACT_RELU, True),    # ResNet-18 layer1 conv2 shape, several tiles per SM
    (3, 64, 29, 37, 48, L.ACT_NONE, False),   # ragged tiles, k < 64 (padding columns)
    (1, 64, 14, 14, 64, L.ACT_CLIP, True),    # fewer tiles than SMs
    (2, 64, 30, 22, 64, L.ACT_GELU, False),   # heavy epilogue
]


@pytest.mark.parametrize("case", RESIDENT_CASES, ids=[str(c[:5]) for c in RESIDENT_CASES])
def test_conv_resident_weights(ctx, case):
    """Tile flags bit 3: the whole weight matrix stays in shared memory and each
    tile loads only its input band; equal to the per-tap path bit for bit (one
    channel block: same accumulation order) and to the oracle."""
    n, c, h, w, k, act, with_res = case
    rng = np.random.default_rng(400 + n + h + w + k)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, 3, 3)) * np.sqrt(2.0 / (c * 9))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    res = rng.standard_normal((n, k, h, w)).astype(np.float32) if with_res else None
    clip = (0.0, 6.0)
    resident = run_conv(ctx, x, wt, b, pad=1, act=act, res=res, flags=8, clip=clip)
    per_tap = run_conv(ctx, x, wt, b, pad=1, act=act, res=res, flags=2, clip=clip)
    np.testing.assert_array_equal(resident, per_tap)
    name = {L.ACT_RELU: "Relu", L.ACT_NONE: None, L.ACT_CLIP: "Clip", L.ACT_GELU: "Gelu"}[act]
    check(resident, oracle_conv(x, wt, b, pad=1, act=name, res=res, clip=clip), 1e-2)


SPLIT_CASES = [
    # n, c, h, w, k, r, stride, pad, splits
    (1, 512, 7, 7, 512, 3, 1, 1, 9),      # ResNet-18 layer4 at b=1
    (1, 256, 14, 14, 256, 3, 1, 1, 4),
    (1, 96, 9, 9, 200, 3, 1, 1, 3),       # ragged k (200 of 256 columns) and M (81 rows)
    (2, 64, 8, 8, 64, 3, 2, 1, 5),        # 9 k-blocks in 5 uneven slices, stride 2
]


@pytest.mark.parametrize("case", SPLIT_CASES, ids=[str(c) for c in SPLIT_CASES])
def test_conv_split_k(ctx, case):
    """Split-K: slices of the reduction on different CTAs, the tile's last one
    summing them in slice order. Matches the unsplit kernel (bf16 rounding of a
    differently ordered fp32 sum) and the oracle, and repeats bit for bit (the
    arrival counters are left at zero)."""
    n, c, h, w, k, r, st, pad, splits = case
    rng = np.random.default_rng(500 + sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    oh, ow = (h + 2 * pad - r) // st + 1, (w + 2 * pad - r) // st + 1
    res = rng.standard_normal((n, k, oh, ow)).astype(np.float32)
    split1 = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, res=res, flags=splits << 8)
    split2 = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, res=res, flags=splits << 8)
    whole = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, res=res)
    np.testing.assert_array_equal(split1, split2)
    check(split1, whole, 1e-2)
    check(split1, oracle_conv(x, wt, b, stride=st, pad=pad, act="Relu", res=res), 1e-2)
    # fp32 output (the FC / logits form) through the same split
    f1 = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, out_f32=True, flags=splits << 8)
    f0 = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, out_f32=True)
    check(f1, f0, 1e-4)


def test_conv_split_k_after_stale_counters(ctx):
    """A split-K call that gives up on a bounded wait leaves its tiles' arrival
    counters part-counted. The next split-K call must not be affected: the
    counters are planted non-zero (no wait is made to run out) and the split
    result must equal a clean split run bit for bit and the unsplit one."""
    n, c, h, w, k, r, st, pad, splits = SPLIT_CASES[0]
    rng = np.random.default_rng(4242)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * np.sqrt(2.0 / (c * r * r))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    clean = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, flags=splits << 8)
    for value in (1, 0x7F):
        ctx.poison_split_counters(value)
        got = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU, flags=splits << 8)
        np.testing.assert_array_equal(got, clean)
    whole = run_conv(ctx, x, wt, b, stride=st, pad=pad, act=L.ACT_RELU)
    check(clean, whole, 1e-2)


@pytest.mark.parametrize("act,name", [(L.ACT_NONE, None), (L.ACT_CLIP, "Clip"), (L.ACT_SIGMOID, "Sigmoid"),
                                      (L.ACT_GELU, "Gelu"), (L.ACT_HARD_SWISH, "HardSwish"),
                                      (L.ACT_LEAKY_RELU, "LeakyRelu"), (L.ACT_TANH, "Tanh")])
def test_conv_bf16_epilogue_activations(ctx, act, name):
    rng = np.random.default_rng(3)
    x = rng.standard_normal((2, 32, 8, 8)).astype(np.float32)
    wt = (rng.standard_normal((48, 32, 3, 3)) * 0.1).astype(np.float32)
    b = (rng.standard_normal(48) * 0.1).astype(np.float32)
    got = run_conv(ctx, x, wt, b, pad=1, act=act)
    want = oracle_conv(x, wt, b, pad=1, act=name)
    check(got, want, 1e-2)


def test_conv_bf16_fp32_output(ctx):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((4, 512, 1, 1)).astype(np.float32)
    wt = (rng.standard_normal((1000, 512, 1, 1)) * 0.06).astype(np.float32)
    b = (rng.standard_normal(1000) * 0.1).astype(np.float32)
    got = run_conv(ctx, x, wt, b, out_f32=True)
    want = oracle_conv(x, wt, b)
    check(got, want, 2e-3)   # no output rounding: only accumulation order differs


F32_CASES = [
    # n, c, h, w, k, r, stride, pad
    (2, 3, 11, 11, 16, 3, 1, 1),       # small: cp.async gather
    (1, 64, 9, 9, 64, 3, 2, 1),
    (3, 40, 6, 6, 24, 1, 1, 0),        # ragged channels
    (4, 64, 32, 32, 64, 3, 1, 1),      # im2col TMA, 32-channel (128-byte) blocks
    (8, 8, 40, 40, 64, 3, 1, 1),       # 32-byte pixels (c = 8)
    (6, 16, 33, 31, 128, 3, 2, 1),     # 64-byte pixels (c = 16), stride 2
    (4, 128, 20, 20, 256, 1, 1, 0),    # pointwise 2-D TMA, 256-wide tiles
    (2, 256, 7, 7, 512, 3, 1, 1),      # deep reduction (2304)
]


@pytest.mark.parametrize("case", F32_CASES, ids=[str(c) for c in F32_CASES])
def test_conv_fp32_3xtf32(ctx, case):
    """fp32 convolutions on the tensor cores (3xTF32) meet the reference's
    FP32_REDUCTION tier against the fp32 oracle."""
    n, c, h, w, k, r, st, pad = case
    rng = np.random.default_rng(5)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * 0.1).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    res = rng.standard_normal((n, k, (h + 2 * pad - r) // st + 1, (w + 2 * pad - r) // st + 1)).astype(np.float32)
    got = run_conv(ctx, x, wt, b, stride=st, pad=pad, dtype="f32", act=L.ACT_RELU, res=res)
    want = oracle_conv(x, wt, b, stride=st, pad=pad, act="Relu", res=res, bf16=False)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)   # FP32_REDUCTION tier


F32_DEEP_CASES = [
    # (n, c, h, w, k, r, stride, pad), (bn, stages)
    ((4, 64, 32, 32, 64, 3, 1, 1), (64, 4)),      # im2col TMA, 64-wide tiles, 4-stage ring
    ((3, 64, 19, 17, 40, 3, 2, 1), (64, 4)),      # stride 2, ragged output channels
    ((4, 64, 32, 32, 128, 3, 1, 1), (128, 3)),    # 128-wide tiles, 3-stage ring
    ((4, 256, 7, 7, 192, 3, 1, 1), (128, 3)),     # deep reduction (2304): promoted accumulator
    ((4, 128, 20, 20, 256, 1, 1, 0), (128, 3)),   # pointwise 2-D TMA
    ((3, 96, 11, 13, 64, 1, 1, 0), (64, 4)),
]


@pytest.mark.parametrize("case,cfg", F32_DEEP_CASES, ids=[f"{c}-{t}" for c, t in F32_DEEP_CASES])
def test_conv_fp32_deep_rings(ctx, case, cfg):
    """The deeper fp32 stage rings (64, 4) and (128, 3) at the FP32_REDUCTION tier."""
    n, c, h, w, k, r, st, pad = case
    rng = np.random.default_rng(6)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * 0.1).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    res = rng.standard_normal((n, k, (h + 2 * pad - r) // st + 1, (w + 2 * pad - r) // st + 1)).astype(np.float32)
    got = run_conv(ctx, x, wt, b, stride=st, pad=pad, dtype="f32", act=L.ACT_RELU, res=res, cfg=cfg)
    want = oracle_conv(x, wt, b, stride=st, pad=pad, act="Relu", res=res, bf16=False)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)   # FP32_REDUCTION tier


def test_conv_fp32_deep_ring_needs_tma_blocks(ctx):
    """(64, 4) exists for 128-byte channel blocks only: a gathered layer is refused."""
    rng = np.random.default_rng(7)
    x = rng.standard_normal((2, 3, 11, 11)).astype(np.float32)
    wt = (rng.standard_normal((16, 3, 3, 3)) * 0.1).astype(np.float32)
    with pytest.raises(L.MdlcError, match="128-byte channel blocks"):
        run_conv(ctx, x, wt, np.zeros(16, np.float32), pad=1, dtype="f32", cfg=(64, 4))


def test_conv_fp32_split_k(ctx):
    """3xTF32 with split-K: fp32 partial sums summed in slice order."""
    n, c, h, w, k, r, st, pad = 1, 512, 7, 7, 512, 3, 1, 1
    rng = np.random.default_rng(15)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, r, r)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    got = run_conv(ctx, x, wt, b, stride=st, pad=pad, dtype="f32", act=L.ACT_RELU, flags=6 << 8)
    want = oracle_conv(x, wt, b, stride=st, pad=pad, act="Relu", bf16=False)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


DW_CASES = [
    # n, c, h, w, r, stride, pad, residual   (3x3 dilation 1: the row-strip kernel; others generic)
    (2, 96, 13, 12, 3, 1, 1, False),
    (2, 96, 13, 12, 3, 2, 1, False),
    (1, 40, 35, 9, 3, 2, 1, False),      # 3 strips, ragged channel groups
    (2, 24, 20, 17, 3, 1, 0, True),      # no padding, residual
    (2, 32, 11, 10, 5, 1, 2, False),     # 5x5: generic kernel
    (2, 144, 29, 31, 3, 1, 1, True),     # 48-channel blocks, tiles past both image edges
    (1, 960, 9, 7, 3, 2, 1, False),      # 15 blocks of 64 channels, stride 2
    (3, 56, 33, 17, 3, 2, 1, True),      # one 56-channel block, odd sizes, stride 2
    (1, 24, 40, 40, 3, 1, 1, False),     # 24-channel pixels (48 bytes), several tiles
    (1, 20, 15, 15, 3, 1, 1, False),     # c % 4 != 0: the last 4-channel quad is ragged
    (2, 32, 112, 112, 3, 1, 1, False),   # MobileNetV2 block 1 (tall tiles, 64-byte pixels)
    (2, 96, 112, 112, 3, 2, 1, False),   # MobileNetV2 first stride-2 layer
    (2, 384, 14, 14, 3, 1, 1, True),     # late-stage layer, residual
    (2, 576, 14, 14, 3, 2, 1, False),
    (4, 960, 7, 7, 3, 1, 1, False),
]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("case", DW_CASES, ids=[str(c) for c in DW_CASES])
def test_depthwise(ctx, dtype, case):
    n, c, h, w, r, stride, pad, with_res = case
    rng = np.random.default_rng(9 + sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((c, 1, r, r)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(c) * 0.1).astype(np.float32)
    oh, ow = (h + 2 * pad - r) // stride + 1, (w + 2 * pad - r) // stride + 1
    res = rng.standard_normal((n, c, oh, ow)).astype(np.float32) if with_res else None
    got = run_conv(ctx, x, wt, b, stride=stride, pad=pad, groups=c, dtype=dtype, act=L.ACT_CLIP, res=res)
    # depthwise weights are kept in fp32; only activations are bf16
    xr = oref.round_bf16(x) if dtype == "bf16" else x
    y = oref.conv(xr, wt, b, strides=[stride] * 2, pads=[pad] * 4, group=c)
    if res is not None:
        y = y + (oref.round_bf16(res) if dtype == "bf16" else res)
    want = oref.clip(y, 0.0, 6.0)
    if dtype == "bf16":
        check(got, want, 1e-2)
    else:
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


DW_ACTS = [
    # activation, clip bounds, oracle
    (L.ACT_NONE, (0.0, 6.0), lambda y: y),
    (L.ACT_RELU, (0.0, 6.0), lambda y: np.maximum(y, 0.0)),
    (L.ACT_CLIP, (-1.0, 2.5), lambda y: np.clip(y, -1.0, 2.5)),   # bounds exact in bf16
    (L.ACT_CLIP, (0.1, 6.0), lambda y: np.clip(y, 0.1, 6.0)),     # 0.1 is not: per-element path
    (L.ACT_SIGMOID, (0.0, 6.0), lambda y: 1.0 / (1.0 + np.exp(-y))),
]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("act", range(len(DW_ACTS)))
def test_depthwise_activations(ctx, dtype, act):
    """Depthwise epilogue activations: clamps folded into packed bf16 pairs,
    or per element (general activations, or clip bounds not exact in bf16)."""
    code, clip, fn = DW_ACTS[act]
    n, c, h, w = 2, 44, 19, 23
    rng = np.random.default_rng(31 + act)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((c, 1, 3, 3)) * 0.4).astype(np.float32)
    b = (rng.standard_normal(c) * 0.1).astype(np.float32)
    for stride in (1, 2):
        got = run_conv(ctx, x, wt, b, stride=stride, pad=1, groups=c, dtype=dtype, act=code, clip=clip)
        xr = oref.round_bf16(x) if dtype == "bf16" else x
        want = fn(oref.conv(xr, wt, b, strides=[stride] * 2, pads=[1] * 4, group=c))
        if dtype == "bf16":
            check(got, want, 1e-2)
        else:
            np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


GROUPED_CASES = [
    # n, c, k, h, w, r, stride, pad, groups, residual
    (2, 64, 64, 11, 13, 3, 1, 1, 2, False),
    (2, 64, 96, 9, 9, 3, 2, 1, 4, True),       # k != c
    (1, 128, 128, 7, 8, 3, 1, 1, 16, False),    # groups = C/8
    (2, 24, 40, 10, 10, 1, 1, 0, 4, False),     # 1x1 grouped, ragged k stride
    (2, 16, 32, 12, 12, 3, 1, 1, 16, False),    # depth multiplier 2 (groups = C, K = 2C)
]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("case", GROUPED_CASES, ids=[str(c) for c in GROUPED_CASES])
def test_grouped_conv(ctx, dtype, case):
    """1 < groups < C (and channel multipliers) on the device: the reference
    runs these per group on the host (ops.py:68-78, emit.py:175-180)."""
    n, c, k, h, w, r, stride, pad, groups, with_res = case
    rng = np.random.default_rng(77 + sum(case))
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c // groups, r, r)) * np.sqrt(2.0 / (c // groups * r * r))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    oh, ow = (h + 2 * pad - r) // stride + 1, (w + 2 * pad - r) // stride + 1
    res = rng.standard_normal((n, k, oh, ow)).astype(np.float32) if with_res else None
    got = run_conv(ctx, x, wt, b, stride=stride, pad=pad, groups=groups, dtype=dtype, act=L.ACT_RELU, res=res)
    # grouped weights are kept in fp32; only activations are bf16
    xr = oref.round_bf16(x) if dtype == "bf16" else x
    y = oref.conv(xr, wt, b, strides=[stride] * 2, pads=[pad] * 4, group=groups)
    if res is not None:
        y = y + (oref.round_bf16(res) if dtype == "bf16" else res)
    want = np.maximum(y, 0)
    if dtype == "bf16":
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2)
    else:
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def _pool(ctx, x, kind, dtype, k=3, s=2, p=1):
    n, c, h, w = x.shape
    cs = _rnd8(c)
    oh, ow = ((h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1) if kind != 2 else (1, 1)
    dt = L.BF16 if dtype == "bf16" else L.F32
    d = L.PoolDesc(kind=kind, n=n, h=h, w=w, c=c, c_stride=cs, kh=k, kw=k, stride_h=s, stride_w=s,
                   pad_t=p, pad_l=p, oh=oh, ow=ow, count_include_pad=0, dtype=dt)
    xh = nhwc(x, cs)
    xd = ctx.to_device(bf16_bits(xh) if dt == L.BF16 else xh)
    eb = 2 if dt == L.BF16 else 4
    yd = ctx.alloc(n * oh * ow * cs * eb)
    ctx.pool2d(d, xd, yd)
    ctx.sync()
    y = ctx.download(yd, (n, oh, ow, cs), np.uint16 if dt == L.BF16 else np.float32)
    y = from_bf16_bits(y) if dt == L.BF16 else y
    ctx.free(xd)
    ctx.free(yd)
    return y[..., :c].transpose(0, 3, 1, 2)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_pools(ctx, dtype):
    rng = np.random.default_rng(13)
    x = rng.standard_normal((2, 20, 15, 14)).astype(np.float32)
    xr = oref.round_bf16(x) if dtype == "bf16" else x
    got = _pool(ctx, x, 0, dtype)
    np.testing.assert_array_equal(got, oref.maxpool(xr, kernel=[3, 3], strides=[2, 2], pads=[1] * 4))
    got = _pool(ctx, x, 1, dtype)
    want = oref.averagepool(xr, kernel=[3, 3], strides=[2, 2], pads=[1] * 4)
    check(got, want, 1e-2 if dtype == "bf16" else 1e-6)
    got = _pool(ctx, x, 2, dtype)
    want = oref.global_average_pool(xr)
    check(got, want, 1e-2 if dtype == "bf16" else 1e-6)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("shape,k,s,p", [((3, 64, 37, 30), 3, 2, 1), ((2, 24, 40, 41), 3, 2, 0),
                                         ((1, 16, 112, 112), 3, 2, 1), ((2, 8, 9, 10), 3, 1, 1),
                                         ((2, 40, 12, 12), 2, 2, 0)])
def test_maxpool_shapes(ctx, dtype, shape, k, s, p):
    """3x3/2 row-strip kernel (several strips, with and without padding) and the
    generic window kernel, bit-exact (max is exact in either precision)."""
    x = np.random.default_rng(29).standard_normal(shape).astype(np.float32)
    xr = oref.round_bf16(x) if dtype == "bf16" else x
    got = _pool(ctx, x, 0, dtype, k=k, s=s, p=p)
    np.testing.assert_array_equal(got, oref.maxpool(xr, kernel=[k, k], strides=[s, s], pads=[p] * 4))


@pytest.mark.parametrize("dtype", [L.U8, L.S8])
@pytest.mark.parametrize("shape,k,s,p", [((2, 64, 37, 30), 3, 2, 1), ((1, 16, 20, 20), 3, 2, 0),
                                         ((2, 32, 9, 10), 3, 1, 1)])
def test_maxpool_codes(ctx, dtype, shape, k, s, p):
    """8-bit max pooling on codes (strip kernel for 3x3/2, generic otherwise)."""
    n, c, h, w = shape
    rng = np.random.default_rng(37)
    npdt = np.uint8 if dtype == L.U8 else np.int8
    info = np.iinfo(npdt)
    x = rng.integers(info.min, info.max + 1, shape).astype(npdt)
    cs = (c + 15) // 16 * 16
    oh, ow = (h + 2 * p - k) // s + 1, (w + 2 * p - k) // s + 1
    d = L.PoolDesc(kind=0, n=n, h=h, w=w, c=c, c_stride=cs, kh=k, kw=k, stride_h=s, stride_w=s,
                   pad_t=p, pad_l=p, oh=oh, ow=ow, count_include_pad=0, dtype=dtype)
    xd = ctx.to_device(nhwc(x, cs))
    yd = ctx.alloc(n * oh * ow * cs)
    ctx.pool2d(d, xd, yd)
    ctx.sync()
    y = ctx.download(yd, (n, oh, ow, cs), npdt)[..., :c].transpose(0, 3, 1, 2)
    want = oref.maxpool(x.astype(np.float32), kernel=[k, k], strides=[s, s], pads=[p] * 4)
    np.testing.assert_array_equal(y.astype(np.float32), want)
    ctx.free(xd)
    ctx.free(yd)


def _s2d_ref(x):
    n, c, h, w = x.shape
    t = x.reshape(n, c, h // 2, 2, w // 2, 2).transpose(0, 2, 4, 3, 5, 1)   # n, Y, X, dy, dx, c
    return t.reshape(n, h // 2, w // 2, 4 * c)


@pytest.mark.parametrize("dtype", [L.BF16, L.F32, L.U8, L.S8])
@pytest.mark.parametrize("shape,cs", [((2, 3, 20, 18), 16), ((1, 4, 8, 6), 16), ((2, 1, 6, 4), 16),
                                      ((2, 3, 20, 18), 32), ((2, 5, 10, 12), 24),
                                      ((3, 3, 14, 28), 16), ((2, 3, 10, 24), 32)])   # two pixels per thread
def test_space_to_depth_input(ctx, dtype, shape, cs):
    """fp32 NCHW -> 2x2 space-to-depth NHWC (16-channel stem kernel and the
    generic one), quantising for 8-bit types."""
    x = np.random.default_rng(31).standard_normal(shape).astype(np.float32)
    n, c, h, w = shape
    q8 = dtype in (L.U8, L.S8)
    if q8:
        cs = max(cs, 16) if cs % 16 == 0 else 32
    zp = 0 if dtype == L.S8 else 77
    xd = ctx.to_device(x)
    eb = {L.BF16: 2, L.F32: 4, L.U8: 1, L.S8: 1}[dtype]
    yd = ctx.alloc(n * (h // 2) * (w // 2) * cs * eb)
    inv = 1.0 / np.float32(0.05)
    ctx.to_s2d(xd, n, c, h, w, yd, cs, dtype, float(np.float32(inv)), zp)
    ctx.sync()
    npdt = {L.BF16: np.uint16, L.F32: np.float32, L.U8: np.uint8, L.S8: np.int8}[dtype]
    y = ctx.download(yd, (n, h // 2, w // 2, cs), npdt)
    ref = _s2d_ref(x)
    if dtype == L.BF16:
        np.testing.assert_array_equal(y[..., :4 * c], bf16_bits(ref))
        assert np.all(y[..., 4 * c:] == 0)
    elif dtype == L.F32:
        np.testing.assert_array_equal(y[..., :4 * c], ref)
        assert np.all(y[..., 4 * c:] == 0)
    else:
        lo, hi = (-128, 127) if dtype == L.S8 else (0, 255)
        q = np.clip(np.rint(ref * np.float32(inv)).astype(np.int64) + zp, lo, hi)
        np.testing.assert_array_equal(y[..., :4 * c].astype(np.int64), q)
        assert np.all(y[..., 4 * c:] == 0)
    ctx.free(xd)
    ctx.free(yd)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_eltwise_program(ctx, dtype):
    """relu(a + b) * c with c broadcast per (n, channel), plus a second output."""
    rng = np.random.default_rng(17)
    n, c, h, w = 2, 36, 5, 7
    cs = _rnd8(c)
    a = rng.standard_normal((n, c, h, w)).astype(np.float32)
    b = rng.standard_normal((n, c, h, w)).astype(np.float32)
    g = rng.standard_normal((n, c, 1, 1)).astype(np.float32)
    dt = L.BF16 if dtype == "bf16" else L.F32
    conv = (lambda t: bf16_bits(t)) if dt == L.BF16 else (lambda t: t)
    ad, bd, gd = (ctx.to_device(conv(nhwc(t, cs))) for t in (a, b, g))
    eb = 2 if dt == L.BF16 else 4
    y0, y1 = ctx.alloc(n * h * w * cs * eb), ctx.alloc(n * h * w * cs * eb)
    prog = L.EwProg(n=n, hw=h * w, c=c, c_stride=cs, dtype=dt, n_inputs=3, n_outputs=2, n_instr=3)
    prog.bcast[0], prog.bcast[1], prog.bcast[2] = L.BC_FULL, L.BC_FULL, L.BC_NC
    prog.code[0] = L.EwInstr(op=L.EW_ADD, dst=3, src0=0, src1=1)
    prog.code[1] = L.EwInstr(op=L.EW_RELU, dst=4, src0=3, src1=0)
    prog.code[2] = L.EwInstr(op=L.EW_MUL, dst=5, src0=4, src1=2)
    prog.out_reg[0], prog.out_reg[1] = 5, 3
    ctx.eltwise(prog, [ad, bd, gd], [y0, y1])
    ctx.sync()
    outs = []
    for yd in (y0, y1):
        y = ctx.download(yd, (n, h, w, cs), np.uint16 if dt == L.BF16 else np.float32)
        y = from_bf16_bits(y) if dt == L.BF16 else y
        assert np.all(y[..., c:] == 0)
        outs.append(y[..., :c].transpose(0, 3, 1, 2))
    if dt == L.BF16:
        a, b, g = oref.round_bf16(a), oref.round_bf16(b), oref.round_bf16(g)
    s = a + b
    want0, want1 = np.maximum(s, 0) * g, s
    check(outs[0], want0, 1e-2 if dt == L.BF16 else 1e-6)
    check(outs[1], want1, 1e-2 if dt == L.BF16 else 1e-6)


@pytest.mark.parametrize("shape", [(3, 44, 6, 5), (8, 128, 56, 56)], ids=["padded", "multi-trip"])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("mode,op,post", [(L.BC_FULL, L.EW_ADD, L.EW_RELU), (L.BC_NC, L.EW_MUL, None),
                                          (L.BC_C, L.EW_SUB, L.EW_SIGMOID), (L.BC_SCALAR, L.EW_MUL, L.EW_CLIP)])
def test_eltwise_binary_fast_path(ctx, dtype, mode, op, post, shape):
    """Programs of the form [unary](in0 (op) in1), in1 broadcast full / per (n, c)
    / per c / scalar, take the register-resident fast path; same results. The
    second shape has no padding channels and more vectors than one grid-stride
    trip of the launch covers."""
    rng = np.random.default_rng(19 + mode)
    n, c, h, w = shape
    cs = _rnd8(c)
    dt = L.BF16 if dtype == "bf16" else L.F32
    a = rng.standard_normal((n, c, h, w)).astype(np.float32)
    bshape = {L.BC_FULL: (n, c, h, w), L.BC_NC: (n, c, 1, 1), L.BC_C: (1, c, 1, 1), L.BC_SCALAR: (1, 1, 1, 1)}[mode]
    b = rng.standard_normal(bshape).astype(np.float32)
    conv = (lambda t: bf16_bits(t)) if dt == L.BF16 else (lambda t: t)
    ad = ctx.to_device(conv(nhwc(a, cs)))
    if mode == L.BC_SCALAR:
        bd = ctx.to_device(conv(b.reshape(1)))
    elif mode == L.BC_C:
        bd = ctx.to_device(conv(nhwc(b, cs)).reshape(-1))
    else:
        bd = ctx.to_device(conv(nhwc(b, cs)))
    eb = 2 if dt == L.BF16 else 4
    yd = ctx.alloc(n * h * w * cs * eb)
    ctx.memset(yd, 0xFF, n * h * w * cs * eb)
    prog = L.EwProg(n=n, hw=h * w, c=c, c_stride=cs, dtype=dt, n_inputs=2, n_outputs=1,
                    n_instr=1 if post is None else 2)
    prog.bcast[0], prog.bcast[1] = L.BC_FULL, mode
    prog.code[0] = L.EwInstr(op=op, dst=2, src0=0, src1=1)
    if post is not None:
        prog.code[1] = L.EwInstr(op=post, dst=3, src0=2, src1=0, imm0=-0.5, imm1=0.75)
    prog.out_reg[0] = 2 if post is None else 3
    ctx.eltwise(prog, [ad, bd], [yd])
    ctx.sync()
    y = ctx.download(yd, (n, h, w, cs), np.uint16 if dt == L.BF16 else np.float32)
    y = from_bf16_bits(y) if dt == L.BF16 else y
    assert np.all(y[..., c:] == 0)
    got = y[..., :c].transpose(0, 3, 1, 2)
    if dt == L.BF16:
        a, b = oref.round_bf16(a), oref.round_bf16(b)
    r = {L.EW_ADD: a + b, L.EW_MUL: a * b, L.EW_SUB: a - b}[op]
    if post == L.EW_RELU:
        r = np.maximum(r, 0)
    elif post == L.EW_SIGMOID:
        r = 1 / (1 + np.exp(-r))
    elif post == L.EW_CLIP:
        r = np.clip(r, -0.5, 0.75)
    check(got, r, 1e-2 if dt == L.BF16 else 1e-6)
    for p_ in (ad, bd, yd):
        ctx.free(p_)


@pytest.mark.parametrize("dtype", [L.BF16, L.F32])
def test_layout_roundtrip(ctx, dtype):
    rng = np.random.default_rng(19)
    x = rng.standard_normal((3, 5, 7, 9)).astype(np.float32)
    xd = ctx.to_device(x)
    cs = 8
    eb = 2 if dtype == L.BF16 else 4
    yd = ctx.alloc(3 * 7 * 9 * cs * eb)
    zd = ctx.alloc(x.nbytes)
    ctx.to_nhwc(xd, 3, 5, 7, 9, yd, cs, dtype)
    ctx.to_nchw(yd, 3, 5, 7, 9, cs, dtype, zd)
    ctx.sync()
    z = ctx.download(zd, x.shape, np.float32)
    want = oref.round_bf16(x) if dtype == L.BF16 else x
    np.testing.assert_array_equal(z, want)
    for p in (xd, yd, zd):
        ctx.free(p)


def test_bounded_wait_reports_timeout(ctx):
    """A wait that can never complete gives up, sets the error word, and the
    context stays usable (no fault, no hang)."""
    ctx.timeout_probe(2000)   # 2 ms
    ctx.check(ctx.lib.mdlc_sync(ctx.h, 10000), "sync")
    assert ctx.check_flag() == L.DEVERR_WAIT_TIMEOUT
    assert ctx.check_flag() == 0        # reading clears the word
    test_layout_roundtrip(ctx, L.F32)   # still works afterwards


GEMM_CASES = [
    # m, n, k, lda, trans_b, alpha, dtype
    (37, 1000, 512, 512, 1, 1.0, "bf16"),     # FC layout (ONNX transB = 1), ragged m and n
    (64, 96, 200, 208, 0, 0.5, "bf16"),       # [k, n] operand, row padding in a, alpha folded
    (5, 24, 40, 40, 1, 2.0, "f32"),           # fp32: SIMT kernel
]


@pytest.mark.parametrize("case", GEMM_CASES, ids=[str(c) for c in GEMM_CASES])
def test_gemm_entry_point(ctx, case):
    """mdlc_gemm: y = act(alpha * a . op(b) + bias) against the oracle's Gemm."""
    m, n, k, lda, tb, alpha, dtype = case
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((n, k) if tb else (k, n)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    et = L.BF16 if dtype == "bf16" else L.F32
    d = L.GemmDesc(m=m, n=n, k=k, lda=lda, trans_a=0, trans_b=tb, alpha=alpha, in_type=et, out_type=et)
    bp = ctx.to_device(L.pack_gemm_weights(d, b))
    ah = np.zeros((m, lda), np.float32)
    ah[:, :k] = a
    ad = ctx.to_device(bf16_bits(ah) if et == L.BF16 else ah)
    bd = ctx.to_device(bias)
    ns = _rnd8(n)
    eb = 2 if et == L.BF16 else 4
    yd = ctx.alloc(m * ns * eb)
    ctx.memset(yd, 0xFF, m * ns * eb)
    ctx.gemm(d, ad, bp, bd, yd, L.Epilogue(act=L.ACT_RELU))
    ctx.sync()
    y = ctx.download(yd, (m, ns), np.uint16 if et == L.BF16 else np.float32)
    y = from_bf16_bits(y) if et == L.BF16 else y
    for p in (bp, ad, bd, yd):
        ctx.free(p)
    assert np.all(y[:, n:] == 0), "padding columns must be written as zero"
    ar = oref.round_bf16(a) if et == L.BF16 else a
    bw = np.float32(alpha) * (b if tb else b.T)
    br = oref.round_bf16(bw) if et == L.BF16 else bw
    want = np.maximum(ar @ br.T + bias, 0)
    if et == L.BF16:
        check(y[:, :n], want, 1e-2)
    else:
        np.testing.assert_allclose(y[:, :n], want, rtol=1e-4, atol=1e-4)


def test_gemm_rejects_trans_a(ctx):
    d = L.GemmDesc(m=4, n=8, k=8, lda=8, trans_a=1, trans_b=1, alpha=1.0, in_type=L.BF16, out_type=L.BF16)
    with pytest.raises(L.MdlcError, match="trans_a"):
        ctx.gemm(d, 0, 0, 0, 0)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_dwconv2d_entry_point(ctx, dtype):
    """mdlc_dwconv2d gives the bytes mdlc_conv2d gives for the same depthwise
    conv, and refuses a grouped conv that is not depthwise."""
    n, c, h, w = 2, 48, 15, 13
    rng = np.random.default_rng(48)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((c, 1, 3, 3)) * 0.3).astype(np.float32)
    b = (rng.standard_normal(c) * 0.1).astype(np.float32)
    et = L.BF16 if dtype == "bf16" else L.F32
    cs = _rnd8(c)
    d = L.ConvDesc(n=n, h=h, w=w, c=c, c_stride=cs, k=c, k_stride=cs, r=3, s=3, stride_h=2, stride_w=2,
                   pad_t=1, pad_l=1, dil_h=1, dil_w=1, oh=8, ow=7, groups=c, in_type=et, out_type=et)
    wp = ctx.to_device(L.pack_weights(d, wt))
    xh = nhwc(x, cs)
    xd = ctx.to_device(bf16_bits(xh) if et == L.BF16 else xh)
    bd = ctx.to_device(np.pad(b, (0, cs - c)))
    nb = n * 8 * 7 * cs * (2 if et == L.BF16 else 4)
    y1, y2 = ctx.alloc(nb), ctx.alloc(nb)
    epi = L.Epilogue(act=L.ACT_CLIP, clip_lo=0.0, clip_hi=6.0)
    ctx.conv2d(d, xd, wp, bd, 0, y1, epi)
    ctx.dwconv2d(d, xd, wp, bd, 0, y2, epi)
    ctx.sync()
    r1 = ctx.download(y1, (nb,), np.uint8)
    r2 = ctx.download(y2, (nb,), np.uint8)
    bad = L.ConvDesc(**{f: getattr(d, f) for f, _ in L.ConvDesc._fields_})
    bad.groups = c // 2
    with pytest.raises(L.MdlcError, match="groups"):
        ctx.dwconv2d(bad, xd, wp, bd, 0, y2, epi)
    for p in (wp, xd, bd, y1, y2):
        ctx.free(p)
    np.testing.assert_array_equal(r1, r2)


SE_CASES = [
    # n, c, rd, act1, act2
    (6, 56, 16, L.ACT_RELU, L.ACT_SIGMOID),       # RepViT stage 1 (n not a multiple of 4)
    (4, 448, 112, L.ACT_RELU, L.ACT_SIGMOID),     # RepViT stage 4
    (9, 100, 24, L.ACT_RELU, L.ACT_HARD_SIGMOID), # ragged channel stride, MobileNetV3-style gate
    (3, 2000, 500, L.ACT_NONE, L.ACT_SIGMOID),    # > 48 KB of shared memory
]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("case", SE_CASES, ids=[str(c[:3]) for c in SE_CASES])
def test_se_fc(ctx, dtype, case):
    """mdlc_se_fc: FC + act + FC + act on pooled activations against fp32 numpy
    (the hidden layer stays in fp32; bf16 rounds the input and the gate)."""
    n, c, rd, act1, act2 = case
    cs = _rnd8(c)
    rng = np.random.default_rng(n + c + rd)
    p = rng.standard_normal((n, c)).astype(np.float32)
    w1 = (rng.standard_normal((rd, c)) / np.sqrt(c)).astype(np.float32)
    b1 = (rng.standard_normal(rd) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((c, rd)) / np.sqrt(rd)).astype(np.float32)
    b2 = (rng.standard_normal(c) * 0.1).astype(np.float32)
    dt = L.BF16 if dtype == "bf16" else L.F32
    ph = np.zeros((n, cs), np.float32)
    ph[:, :c] = p
    pd = ctx.to_device(bf16_bits(ph) if dt == L.BF16 else ph)
    eb = 2 if dt == L.BF16 else 4
    gd = ctx.alloc(n * cs * eb)
    ctx.memset(gd, 0xFF, n * cs * eb)      # poison: padding channels must be written
    bufs = [ctx.to_device(a) for a in (w1, b1, np.ascontiguousarray(w2.T), b2)]
    d = L.SeDesc(n=n, c=c, c_stride=cs, rd=rd, dtype=dt, act1=act1, act2=act2, alpha1=0.01, beta1=0.5,
                 lo1=-np.inf, hi1=np.inf, alpha2=0.2, beta2=0.5, lo2=-np.inf, hi2=np.inf)
    ctx.se_fc(d, pd, *bufs, gd)
    ctx.sync()
    y = ctx.download(gd, (n, cs), np.uint16 if dt == L.BF16 else np.float32)
    y = from_bf16_bits(y) if dt == L.BF16 else y
    for b in [pd, gd] + bufs:
        ctx.free(b)
    assert np.all(y[:, c:] == 0)
    acts = {L.ACT_NONE: lambda v: v, L.ACT_RELU: lambda v: np.maximum(v, 0),
            L.ACT_SIGMOID: lambda v: 1 / (1 + np.exp(-v)),
            L.ACT_HARD_SIGMOID: lambda v: np.clip(0.2 * v + 0.5, 0, 1)}
    x = oref.round_bf16(p) if dt == L.BF16 else p
    h = acts[act1](x.astype(np.float64) @ w1.T.astype(np.float64) + b1)
    want = acts[act2](h @ w2.T.astype(np.float64) + b2)
    if dt == L.BF16:
        np.testing.assert_allclose(y[:, :c], want, rtol=1e-2, atol=4e-3)
    else:
        np.testing.assert_allclose(y[:, :c], want, rtol=1e-4, atol=1e-5)


SE_POOL_CASES = [
    # n, c, hw, rd   (the squeeze fused: activations [n][hw][c_stride] in)
    (5, 56, 56 * 56, 16),     # RepViT stage 1: 7 channel groups, 146 pixel slices (not a power of two)
    (4, 224, 14 * 14, 56),    # RepViT stage 3: 28 groups, 36 slices
    (3, 448, 7 * 7, 112),     # RepViT stage 4: 56 groups, 18 slices
    (2, 100, 9 * 11, 24),     # ragged channel stride (104), odd pixel count
    (3, 4000, 3 * 3, 1000),   # 500 groups (2 slices), > 48 KB of shared memory
]


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
@pytest.mark.parametrize("case", SE_POOL_CASES, ids=[str(c) for c in SE_POOL_CASES])
def test_se_fc_fused_squeeze(ctx, dtype, case):
    """mdlc_se_fc with hw > 1: the global average pool of the activations and
    both FCs in one kernel (the mean kept in fp32), against fp32 numpy."""
    n, c, hw, rd = case
    cs = _rnd8(c)
    rng = np.random.default_rng(n + c + hw + rd)
    x = rng.standard_normal((n, hw, c)).astype(np.float32) + 0.5
    w1 = (rng.standard_normal((rd, c)) / np.sqrt(c)).astype(np.float32)
    b1 = (rng.standard_normal(rd) * 0.1).astype(np.float32)
    w2 = (rng.standard_normal((c, rd)) / np.sqrt(rd)).astype(np.float32)
    b2 = (rng.standard_normal(c) * 0.1).astype(np.float32)
    dt = L.BF16 if dtype == "bf16" else L.F32
    xh = np.zeros((n, hw, cs), np.float32)
    xh[..., :c] = x
    xd = ctx.to_device(bf16_bits(xh) if dt == L.BF16 else xh)
    eb = 2 if dt == L.BF16 else 4
    gd = ctx.alloc(n * cs * eb)
    ctx.memset(gd, 0xFF, n * cs * eb)
    bufs = [ctx.to_device(a) for a in (w1, b1, np.ascontiguousarray(w2.T), b2)]
    d = L.SeDesc(n=n, c=c, c_stride=cs, rd=rd, dtype=dt, act1=L.ACT_RELU, act2=L.ACT_SIGMOID, alpha1=0.01,
                 beta1=0.5, lo1=-np.inf, hi1=np.inf, alpha2=0.2, beta2=0.5, lo2=-np.inf, hi2=np.inf, hw=hw)
    ctx.se_fc(d, xd, *bufs, gd)
    ctx.sync()
    y = ctx.download(gd, (n, cs), np.uint16 if dt == L.BF16 else np.float32)
    y = from_bf16_bits(y) if dt == L.BF16 else y
    for b in [xd, gd] + bufs:
        ctx.free(b)
    assert np.all(y[:, c:] == 0)
    xr = oref.round_bf16(x) if dt == L.BF16 else x
    p = xr.astype(np.float64).mean(axis=1)
    h = np.maximum(p @ w1.T.astype(np.float64) + b1, 0)
    want = 1 / (1 + np.exp(-(h @ w2.T.astype(np.float64) + b2)))
    if dt == L.BF16:
        np.testing.assert_allclose(y[:, :c], want, rtol=1e-2, atol=4e-3)
    else:
        np.testing.assert_allclose(y[:, :c], want, rtol=1e-4, atol=1e-5)


def test_se_fc_fused_squeeze_needs_alignment(ctx):
    """The activations to pool are read 16 bytes at a time: a misaligned base is refused."""
    n, c, hw, rd = 2, 64, 16, 16
    xd = ctx.alloc(n * hw * c * 2 + 64)
    gd = ctx.alloc(n * c * 2)
    bufs = [ctx.to_device(np.zeros(s, np.float32)) for s in (rd * c, rd, rd * c, c)]
    d = L.SeDesc(n=n, c=c, c_stride=c, rd=rd, dtype=L.BF16, act1=L.ACT_RELU, act2=L.ACT_SIGMOID, hw=hw)
    with pytest.raises(L.MdlcError, match="16-byte aligned"):
        ctx.se_fc(d, xd + 2, *bufs, gd)
    for b in [xd, gd] + bufs:
        ctx.free(b)
