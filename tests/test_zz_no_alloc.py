"""The allocation-free split-K convolution entry point, through the C ABI.

``mdlc_conv2d_splitk_noalloc`` is for callers that cannot call cudaMalloc --
a plug-in that only borrows a stream from a host framework whose memory
manager owns all device memory, or a service with a device memory budget fixed
at start-up -- and so cannot create an ``mdlc_ctx`` either. It keeps its
scratch in a fixed array of the library's device image. This file is collected
last, so a run stopping at its first failure has run every other test; it
passes alone in a fresh process as well as after the others.
"""

import ctypes as C

import numpy as np
import pytest

from mdlc_b200 import _lib as L
from oracle import reference as oref

pytestmark = pytest.mark.gpu


def _bf16_bits(x):
    return (oref.round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def _from_bf16_bits(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def _nhwc(x, cs):
    n, c, h, w = x.shape
    out = np.zeros((n, h, w, cs), dtype=x.dtype)
    out[..., :c] = x.transpose(0, 2, 3, 1)
    return out


def test_splitk_noalloc_matches_conv2d_on_two_calls():
    """Two calls in a row of the allocation-free entry point (on the caller's
    stream) give what mdlc_conv2d gives for the same split-K conv, and what the
    oracle gives, within the bf16 tolerance of the kernel tests; the status
    query reports no device-side error after each."""
    ctx = L.Context(0)
    lib = L.load()
    n, c, h, w, k, splits = 1, 512, 7, 7, 512, 9       # ResNet-18 layer4 at b=1, 8 k-blocks a slice
    rng = np.random.default_rng(77)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((k, c, 3, 3)) * np.sqrt(2.0 / (c * 9))).astype(np.float32)
    b = (rng.standard_normal(k) * 0.1).astype(np.float32)
    res = rng.standard_normal((n, k, h, w)).astype(np.float32)
    d = L.ConvDesc(n=n, h=h, w=w, c=c, c_stride=c, k=k, k_stride=k, r=3, s=3, stride_h=1, stride_w=1,
                   pad_t=1, pad_l=1, dil_h=1, dil_w=1, oh=h, ow=w, groups=1, in_type=L.BF16, out_type=L.BF16,
                   res_stride=0, in_zp=0)
    bufs = []
    try:
        xd = ctx.to_device(_bf16_bits(_nhwc(x, c)))
        wd = ctx.to_device(L.pack_weights(d, wt))
        bd = ctx.to_device(b)
        rd = ctx.to_device(_bf16_bits(_nhwc(res, k)))
        nbytes = n * h * w * k * 2
        y_ref, y_new = ctx.alloc(nbytes), ctx.alloc(nbytes)
        bufs = [xd, wd, bd, rd, y_ref, y_new]
        epi = L.Epilogue(act=L.ACT_RELU)
        ctx.conv2d(d, xd, wd, bd, rd, y_ref, epi, L.TileCfg(bn=0, stages=0, flags=splits << 8))
        ctx.sync()
        want = _from_bf16_bits(ctx.download(y_ref, (n, h, w, k), np.uint16))
        xr, wr, rr = oref.round_bf16(x), oref.round_bf16(wt), oref.round_bf16(res)
        oracle = oref.conv(xr, wr, b, strides=[1, 1], pads=[1, 1, 1, 1]) + rr
        oracle = np.maximum(oracle, 0).transpose(0, 2, 3, 1)
        stream = C.c_void_p()
        assert lib.mdlc_get_stream(ctx.h, C.byref(stream)) == 0
        msg = C.create_string_buffer(256)
        for call in range(2):
            ctx.memset(y_new, 0xFF, nbytes)           # poison: the call must write every element
            st = lib.mdlc_conv2d_splitk_noalloc(C.byref(d), C.c_void_p(xd), C.c_void_p(wd), C.c_void_p(bd),
                                                C.c_void_p(rd), C.c_void_p(y_new), C.byref(epi), splits,
                                                stream, msg, len(msg))
            assert st == 0, msg.value.decode()
            ctx.sync()
            got = _from_bf16_bits(ctx.download(y_new, (n, h, w, k), np.uint16))
            err = np.abs(got - want).max()
            assert err <= 1e-2 * np.abs(want).max(), f"call {call}: max err {err}"
            # and directly against the oracle on the same bf16-rounded operands
            err_o = np.abs(got - oracle).max()
            assert err_o <= 1e-2 * np.abs(oracle).max(), f"call {call}: max err vs oracle {err_o}"
            flag = C.c_int(-1)
            assert lib.mdlc_conv2d_splitk_noalloc_status(stream, C.byref(flag), msg, len(msg)) == 0, msg.value
            assert flag.value == 0, f"call {call}: device error word {flag.value}"
    finally:
        for p in bufs:
            ctx.free(p)
        ctx.close()


def test_splitk_noalloc_rejects_what_it_cannot_hold():
    """Requests beyond the fixed scratch, or outside the entry point's scope,
    fail with a status and a message before any launch."""
    lib = L.load()
    msg = C.create_string_buffer(256)
    big = L.ConvDesc(n=64, h=56, w=56, c=64, c_stride=64, k=64, k_stride=64, r=3, s=3, stride_h=1, stride_w=1,
                     pad_t=1, pad_l=1, dil_h=1, dil_w=1, oh=56, ow=56, groups=1, in_type=L.BF16,
                     out_type=L.BF16, res_stride=0, in_zp=0)
    ctx = L.Context(0)
    try:
        stream = C.c_void_p()
        assert lib.mdlc_get_stream(ctx.h, C.byref(stream)) == 0
        dummy = ctx.alloc(1 << 16)
        # 1568 tiles x 9 slices of 128 x 64 fp32 partials: far beyond 8 MiB
        st = lib.mdlc_conv2d_splitk_noalloc(C.byref(big), C.c_void_p(dummy), C.c_void_p(dummy), None, None,
                                            C.c_void_p(dummy), None, 9, stream, msg, len(msg))
        assert st == L.ERR_INVALID and b"workspace" in msg.value, msg.value
        q8 = L.ConvDesc(**{f: getattr(big, f) for f, _ in L.ConvDesc._fields_})
        q8.in_type = L.U8
        st = lib.mdlc_conv2d_splitk_noalloc(C.byref(q8), C.c_void_p(dummy), C.c_void_p(dummy), None, None,
                                            C.c_void_p(dummy), None, 2, stream, msg, len(msg))
        assert st == L.ERR_UNSUPPORTED and b"bf16" in msg.value
        st = lib.mdlc_conv2d_splitk_noalloc(C.byref(big), C.c_void_p(dummy), C.c_void_p(dummy), None, None,
                                            C.c_void_p(dummy), None, 1, stream, msg, len(msg))
        assert st == L.ERR_INVALID and b"splits" in msg.value
        ctx.free(dummy)
    finally:
        ctx.close()
