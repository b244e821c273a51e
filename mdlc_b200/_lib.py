"""ctypes binding of ``libmdlc_b200.so`` (declared in ``include/mdlc_b200.h``).

The structures below mirror the header field-for-field. Every call's status
is checked; a non-zero status raises :class:`MdlcError` carrying the
library's last error message. There is no fallback: if the library is missing
or no B200 is present, loading fails loudly.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# MDLC_B200_LIB=check selects the bounds-checked build (python -m mdlc_b200.build --check)
LIB_PATH = os.path.join(HERE, "libmdlc_b200_check.so" if os.environ.get("MDLC_B200_LIB") == "check"
                        else "libmdlc_b200.so")

OK, ERR_INVALID, ERR_CUDA, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_DEVICE, ERR_NOMEM = 0, -1, -2, -3, -4, -5, -6
STREAM_COMPUTE, STREAM_COPY = 0, 1
DEVERR_NONE, DEVERR_WAIT_TIMEOUT, DEVERR_BOUNDS, DEVERR_INJECTED = 0, 1, 2, 3
F32, BF16, S8, U8, S32 = 0, 1, 2, 3, 4
(ACT_NONE, ACT_RELU, ACT_CLIP, ACT_SIGMOID, ACT_TANH, ACT_LEAKY_RELU, ACT_HARD_SIGMOID,
 ACT_HARD_SWISH, ACT_GELU) = range(9)
(EW_ADD, EW_SUB, EW_MUL, EW_DIV, EW_ADDI, EW_SUBI, EW_RSUBI, EW_MULI, EW_DIVI, EW_RDIVI,
 EW_RELU, EW_CLIP, EW_SIGMOID, EW_TANH, EW_LEAKY_RELU, EW_HARD_SIGMOID, EW_HARD_SWISH, EW_ERF,
 EW_GELU, EW_MAX, EW_MIN) = range(21)
EW_MAX_INPUTS, EW_MAX_OUTPUTS, EW_MAX_INSTR = 4, 2, 24
BC_FULL, BC_NC, BC_C, BC_SCALAR = 0, 1, 2, 3

ELEM_BYTES = {F32: 4, BF16: 2, S8: 1, U8: 1, S32: 4}


class MdlcError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"mdlc_b200 error {status}: {msg}")
        self.status = status


class Epilogue(C.Structure):
    _fields_ = [("act", C.c_int32), ("alpha", C.c_float), ("beta", C.c_float),
                ("clip_lo", C.c_float), ("clip_hi", C.c_float),
                ("rq_scale", C.c_void_p),
                ("out_zp", C.c_int32), ("qmin", C.c_int32), ("qmax", C.c_int32),
                ("res_zp", C.c_int32), ("res_scale", C.c_float), ("res_signed", C.c_int32),
                ("deq_scale", C.c_void_p), ("deq_bias", C.c_void_p),
                ("rq_mult", C.c_void_p), ("rq_res_mult", C.c_void_p), ("rq_shift", C.c_void_p)]


class ConvDesc(C.Structure):
    _fields_ = [(f, C.c_int32) for f in (
        "n", "h", "w", "c", "c_stride", "k", "k_stride", "r", "s", "stride_h", "stride_w",
        "pad_t", "pad_l", "dil_h", "dil_w", "oh", "ow", "groups", "in_type", "out_type",
        "res_stride", "in_zp")]


class GemmDesc(C.Structure):
    _fields_ = [("m", C.c_int32), ("n", C.c_int32), ("k", C.c_int32), ("lda", C.c_int32),
                ("trans_a", C.c_int32), ("trans_b", C.c_int32), ("alpha", C.c_float),
                ("in_type", C.c_int32), ("out_type", C.c_int32)]


class TileCfg(C.Structure):
    _fields_ = [("bn", C.c_int32), ("stages", C.c_int32), ("flags", C.c_int32)]


class PoolDesc(C.Structure):
    _fields_ = [(f, C.c_int32) for f in (
        "kind", "n", "h", "w", "c", "c_stride", "kh", "kw", "stride_h", "stride_w", "pad_t",
        "pad_l", "oh", "ow", "count_include_pad", "dtype", "in_zp", "out_zp", "rq_mult",
        "rq_shift")]


class EwInstr(C.Structure):
    _fields_ = [("op", C.c_int8), ("dst", C.c_int8), ("src0", C.c_int8), ("src1", C.c_int8),
                ("imm0", C.c_float), ("imm1", C.c_float)]


class EwProg(C.Structure):
    _fields_ = [("n", C.c_int32), ("hw", C.c_int32), ("c", C.c_int32), ("c_stride", C.c_int32),
                ("dtype", C.c_int32), ("n_inputs", C.c_int32), ("n_outputs", C.c_int32),
                ("n_instr", C.c_int32), ("bcast", C.c_int32 * EW_MAX_INPUTS),
                ("out_reg", C.c_int32 * EW_MAX_OUTPUTS), ("code", EwInstr * EW_MAX_INSTR)]


class CopyDesc(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("in_dims", C.c_int32 * 4), ("in_cs", C.c_int32),
                ("out_dims", C.c_int32 * 4), ("out_cs", C.c_int32), ("src_dim", C.c_int32 * 4),
                ("offset", C.c_int32 * 4), ("mode", C.c_int32), ("pad_mode", C.c_int32), ("value", C.c_float)]


class SoftmaxDesc(C.Structure):
    _fields_ = [("dtype", C.c_int32), ("dims", C.c_int32 * 4), ("cs", C.c_int32), ("axis", C.c_int32)]


class SeDesc(C.Structure):
    _fields_ = [("n", C.c_int32), ("c", C.c_int32), ("c_stride", C.c_int32), ("rd", C.c_int32),
                ("dtype", C.c_int32), ("act1", C.c_int32), ("act2", C.c_int32),
                ("alpha1", C.c_float), ("beta1", C.c_float), ("lo1", C.c_float), ("hi1", C.c_float),
                ("alpha2", C.c_float), ("beta2", C.c_float), ("lo2", C.c_float), ("hi2", C.c_float),
                ("hw", C.c_int32)]


# exported symbol -> (argtypes, restype); the CPU test suite checks every
# function declared in include/mdlc_b200.h is exported and listed here.
_P, _I, _S = C.c_void_p, C.c_int, C.c_size_t
SIGNATURES = {
    "mdlc_version": ([], C.c_int),
    "mdlc_device_count": ([C.POINTER(C.c_int)], C.c_int),
    "mdlc_ctx_create": ([C.c_int, C.POINTER(C.c_void_p)], C.c_int),
    "mdlc_ctx_destroy": ([_P], C.c_int),
    "mdlc_last_error": ([_P], C.c_char_p),
    "mdlc_get_stream": ([_P, C.POINTER(C.c_void_p)], C.c_int),
    "mdlc_alloc": ([_P, _S, C.POINTER(C.c_void_p)], C.c_int),
    "mdlc_free": ([_P, _P], C.c_int),
    "mdlc_host_alloc": ([_P, _S, C.POINTER(C.c_void_p)], C.c_int),
    "mdlc_host_free": ([_P, _P], C.c_int),
    "mdlc_upload": ([_P, _P, _P, _S], C.c_int),
    "mdlc_download": ([_P, _P, _P, _S], C.c_int),
    "mdlc_memset": ([_P, _P, C.c_int, _S], C.c_int),
    "mdlc_sync": ([_P, C.c_int], C.c_int),
    "mdlc_check_flag": ([_P, C.POINTER(C.c_int)], C.c_int),
    "mdlc_upload_on": ([_P, C.c_int, _P, _P, _S], C.c_int),
    "mdlc_download_on": ([_P, C.c_int, _P, _P, _S], C.c_int),
    "mdlc_fence_record": ([_P, C.c_int, C.c_int], C.c_int),
    "mdlc_fence_wait": ([_P, C.c_int, C.c_int], C.c_int),
    "mdlc_fence_sync": ([_P, C.c_int, C.c_int], C.c_int),
    "mdlc_conv2d": ([_P, C.POINTER(ConvDesc), _P, _P, _P, _P, _P, C.POINTER(Epilogue),
                     C.POINTER(TileCfg)], C.c_int),
    "mdlc_conv_weight_bytes": ([C.POINTER(ConvDesc), C.POINTER(C.c_size_t)], C.c_int),
    "mdlc_pack_conv_weights": ([C.POINTER(ConvDesc), _P, _P], C.c_int),
    "mdlc_pool2d": ([_P, C.POINTER(PoolDesc), _P, _P], C.c_int),
    "mdlc_dwconv2d": ([_P, C.POINTER(ConvDesc), _P, _P, _P, _P, _P, C.POINTER(Epilogue)], C.c_int),
    "mdlc_conv2d_splitk_noalloc": ([C.POINTER(ConvDesc), _P, _P, _P, _P, _P, C.POINTER(Epilogue), C.c_int, _P,
                                    C.c_char_p, C.c_size_t], C.c_int),
    "mdlc_conv2d_splitk_noalloc_status": ([_P, C.POINTER(C.c_int), C.c_char_p, C.c_size_t], C.c_int),
    "mdlc_gemm_weight_bytes": ([C.POINTER(GemmDesc), C.POINTER(C.c_size_t)], C.c_int),
    "mdlc_pack_gemm_weights": ([C.POINTER(GemmDesc), _P, _P], C.c_int),
    "mdlc_gemm": ([_P, C.POINTER(GemmDesc), _P, _P, _P, _P, C.POINTER(Epilogue), C.POINTER(TileCfg)], C.c_int),
    "mdlc_eltwise": ([_P, C.POINTER(EwProg), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)], C.c_int),
    "mdlc_nchw_to_nhwc": ([_P, _P, _I, _I, _I, _I, _P, _I, _I, C.c_float, _I], C.c_int),
    "mdlc_nhwc_to_nchw": ([_P, _P, _I, _I, _I, _I, _I, _I, _P, C.c_float, _I], C.c_int),
    "mdlc_nchw_to_s2d": ([_P, _P, _I, _I, _I, _I, _P, _I, _I, C.c_float, _I], C.c_int),
    "mdlc_copy4d": ([_P, C.POINTER(CopyDesc), _P, _P], C.c_int),
    "mdlc_softmax": ([_P, C.POINTER(SoftmaxDesc), _P, _P], C.c_int),
    "mdlc_se_fc": ([_P, C.POINTER(SeDesc), _P, _P, _P, _P, _P, _P], C.c_int),
    "mdlc_graph_begin": ([_P], C.c_int),
    "mdlc_graph_end": ([_P], C.c_int),
    "mdlc_graph_launch": ([_P], C.c_int),
    "mdlc_graph_reset": ([_P], C.c_int),
    "mdlc_event_record": ([_P, C.c_int], C.c_int),
    "mdlc_event_record_on": ([_P, C.c_int, C.c_int], C.c_int),
    "mdlc_event_elapsed": ([_P, C.c_int, C.c_int, C.POINTER(C.c_float)], C.c_int),
    "mdlc_launch_count": ([_P, C.POINTER(C.c_longlong)], C.c_int),
    "mdlc_debug_timeout_probe": ([_P, C.c_int], C.c_int),
    "mdlc_debug_poison_split_counters": ([_P, C.c_int], C.c_int),
}

_lib = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Load the prebuilt library (no JIT, no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise MdlcError(ERR_UNSUPPORTED,
                            f"{path} not built; run `python -m mdlc_b200.build` (nvcc, sm_100a)")
        lib = C.CDLL(path)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
    return _lib


def device_count() -> int:
    n = C.c_int(0)
    load().mdlc_device_count(C.byref(n))
    return n.value


class Context:
    """One device + stream (``mdlc_ctx``). Owns device allocations made through it."""

    def __init__(self, device: int = 0):
        self.lib = load()
        h = C.c_void_p()
        st = self.lib.mdlc_ctx_create(int(device), C.byref(h))
        if st != OK:
            raise MdlcError(st, f"mdlc_ctx_create(device={device}) failed (is a B200 visible?)")
        self.h = h
        self.device = device
        self._allocs = set()
        self._host_allocs = set()

    # -- status ---------------------------------------------------------
    def check(self, st: int, what: str = "") -> None:
        if st != OK:
            raise MdlcError(st, f"{what}: {self.lib.mdlc_last_error(self.h).decode()}")

    def check_flag(self) -> int:
        v = C.c_int(0)
        self.check(self.lib.mdlc_check_flag(self.h, C.byref(v)), "check_flag")
        return v.value

    def sync(self, timeout_ms: int = 60000) -> None:
        self.check(self.lib.mdlc_sync(self.h, int(timeout_ms)), "sync")
        flag = self.check_flag()
        if flag:
            raise MdlcError(ERR_DEVICE, f"device error word = {flag}")

    # -- memory ---------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        p = C.c_void_p()
        self.check(self.lib.mdlc_alloc(self.h, C.c_size_t(int(nbytes)), C.byref(p)), "alloc")
        self._allocs.add(p.value)
        return p.value

    def free(self, ptr: int) -> None:
        if ptr in self._allocs:
            self._allocs.discard(ptr)
            self.check(self.lib.mdlc_free(self.h, C.c_void_p(ptr)), "free")

    def host_alloc(self, nbytes: int) -> int:
        p = C.c_void_p()
        self.check(self.lib.mdlc_host_alloc(self.h, C.c_size_t(int(nbytes)), C.byref(p)), "host_alloc")
        self._host_allocs.add(p.value)
        return p.value

    def host_free(self, ptr: int) -> None:
        if ptr in self._host_allocs:
            self._host_allocs.discard(ptr)
            self.check(self.lib.mdlc_host_free(self.h, C.c_void_p(ptr)), "host_free")

    def upload(self, dev: int, arr: np.ndarray) -> None:
        arr = np.ascontiguousarray(arr)
        self.check(self.lib.mdlc_upload(self.h, C.c_void_p(dev), arr.ctypes.data_as(C.c_void_p),
                                        C.c_size_t(arr.nbytes)), "upload")
        self.check(self.lib.mdlc_sync(self.h, 60000), "sync after upload")

    def upload_async(self, dev: int, host_ptr: int, nbytes: int) -> None:
        self.check(self.lib.mdlc_upload(self.h, C.c_void_p(dev), C.c_void_p(host_ptr),
                                        C.c_size_t(nbytes)), "upload")

    def download(self, dev: int, shape, dtype) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        self.check(self.lib.mdlc_download(self.h, out.ctypes.data_as(C.c_void_p), C.c_void_p(dev),
                                          C.c_size_t(out.nbytes)), "download")
        self.sync()
        return out

    def download_async(self, host_ptr: int, dev: int, nbytes: int) -> None:
        self.check(self.lib.mdlc_download(self.h, C.c_void_p(host_ptr), C.c_void_p(dev),
                                          C.c_size_t(nbytes)), "download")

    # -- copy stream and fences (transfers overlapped with compute) ------
    def upload_on(self, stream: int, dev: int, host_ptr: int, nbytes: int) -> None:
        self.check(self.lib.mdlc_upload_on(self.h, int(stream), C.c_void_p(dev), C.c_void_p(host_ptr),
                                           C.c_size_t(nbytes)), "upload_on")

    def download_on(self, stream: int, host_ptr: int, dev: int, nbytes: int) -> None:
        self.check(self.lib.mdlc_download_on(self.h, int(stream), C.c_void_p(host_ptr), C.c_void_p(dev),
                                             C.c_size_t(nbytes)), "download_on")

    def fence_record(self, fence: int, stream: int) -> None:
        self.check(self.lib.mdlc_fence_record(self.h, int(fence), int(stream)), "fence_record")

    def fence_wait(self, fence: int, stream: int) -> None:
        self.check(self.lib.mdlc_fence_wait(self.h, int(fence), int(stream)), "fence_wait")

    def fence_sync(self, fence: int, timeout_ms: int = 60000) -> None:
        self.check(self.lib.mdlc_fence_sync(self.h, int(fence), int(timeout_ms)), "fence_sync")

    def memset(self, dev: int, value: int, nbytes: int) -> None:
        self.check(self.lib.mdlc_memset(self.h, C.c_void_p(dev), int(value), C.c_size_t(nbytes)), "memset")

    def to_device(self, arr: np.ndarray) -> int:
        arr = np.ascontiguousarray(arr)
        p = self.alloc(max(arr.nbytes, 16))
        self.upload(p, arr)
        return p

    # -- kernels --------------------------------------------------------
    def conv2d(self, desc: ConvDesc, x, w, bias, res, y, epi: Epilogue | None = None,
               cfg: TileCfg | None = None) -> None:
        self.check(self.lib.mdlc_conv2d(self.h, C.byref(desc), C.c_void_p(x), C.c_void_p(w),
                                        C.c_void_p(bias or 0), C.c_void_p(res or 0), C.c_void_p(y),
                                        C.byref(epi) if epi is not None else None,
                                        C.byref(cfg) if cfg is not None else None), "conv2d")

    def dwconv2d(self, desc: ConvDesc, x, w, bias, res, y, epi: Epilogue | None = None) -> None:
        self.check(self.lib.mdlc_dwconv2d(self.h, C.byref(desc), C.c_void_p(x), C.c_void_p(w),
                                          C.c_void_p(bias or 0), C.c_void_p(res or 0), C.c_void_p(y),
                                          C.byref(epi) if epi is not None else None), "dwconv2d")

    def gemm(self, desc: GemmDesc, a, b_packed, bias, y, epi: Epilogue | None = None,
             cfg: TileCfg | None = None) -> None:
        self.check(self.lib.mdlc_gemm(self.h, C.byref(desc), C.c_void_p(a), C.c_void_p(b_packed),
                                      C.c_void_p(bias or 0), C.c_void_p(y),
                                      C.byref(epi) if epi is not None else None,
                                      C.byref(cfg) if cfg is not None else None), "gemm")

    def pool2d(self, desc: PoolDesc, x, y) -> None:
        self.check(self.lib.mdlc_pool2d(self.h, C.byref(desc), C.c_void_p(x), C.c_void_p(y)), "pool2d")

    def eltwise(self, prog: EwProg, inputs, outputs) -> None:
        ins = (C.c_void_p * EW_MAX_INPUTS)(*([C.c_void_p(p) for p in inputs] +
                                            [C.c_void_p(0)] * (EW_MAX_INPUTS - len(inputs))))
        outs = (C.c_void_p * EW_MAX_OUTPUTS)(*([C.c_void_p(p) for p in outputs] +
                                              [C.c_void_p(0)] * (EW_MAX_OUTPUTS - len(outputs))))
        self.check(self.lib.mdlc_eltwise(self.h, C.byref(prog), ins, outs), "eltwise")

    def copy4d(self, desc: CopyDesc, x, y) -> None:
        self.check(self.lib.mdlc_copy4d(self.h, C.byref(desc), C.c_void_p(x), C.c_void_p(y)), "copy4d")

    def softmax(self, desc: SoftmaxDesc, x, y) -> None:
        self.check(self.lib.mdlc_softmax(self.h, C.byref(desc), C.c_void_p(x), C.c_void_p(y)), "softmax")

    def se_fc(self, desc: SeDesc, pooled, w1, b1, w2t, b2, gate) -> None:
        self.check(self.lib.mdlc_se_fc(self.h, C.byref(desc), C.c_void_p(pooled), C.c_void_p(w1),
                                       C.c_void_p(b1 or None), C.c_void_p(w2t), C.c_void_p(b2 or None),
                                       C.c_void_p(gate)), "se_fc")

    def to_nhwc(self, x, n, c, h, w, y, cs, dtype, inv_scale=1.0, zp=0) -> None:
        self.check(self.lib.mdlc_nchw_to_nhwc(self.h, C.c_void_p(x), n, c, h, w, C.c_void_p(y), cs, dtype,
                                              C.c_float(inv_scale), zp), "nchw_to_nhwc")

    def to_s2d(self, x, n, c, h, w, y, cs, dtype, inv_scale=1.0, zp=0) -> None:
        self.check(self.lib.mdlc_nchw_to_s2d(self.h, C.c_void_p(x), n, c, h, w, C.c_void_p(y), cs, dtype,
                                             C.c_float(inv_scale), zp), "nchw_to_s2d")

    def to_nchw(self, x, n, c, h, w, cs, dtype, y, scale=1.0, zp=0) -> None:
        self.check(self.lib.mdlc_nhwc_to_nchw(self.h, C.c_void_p(x), n, c, h, w, cs, dtype, C.c_void_p(y),
                                              C.c_float(scale), zp), "nhwc_to_nchw")

    # -- graphs / timing -----------------------------------------------
    def graph_begin(self):
        self.check(self.lib.mdlc_graph_begin(self.h), "graph_begin")

    def graph_end(self):
        self.check(self.lib.mdlc_graph_end(self.h), "graph_end")

    def graph_launch(self):
        self.check(self.lib.mdlc_graph_launch(self.h), "graph_launch")

    def graph_reset(self):
        self.check(self.lib.mdlc_graph_reset(self.h), "graph_reset")

    def event_record(self, slot: int, stream: int = 0):
        if stream:
            self.check(self.lib.mdlc_event_record_on(self.h, int(slot), int(stream)), "event_record_on")
        else:
            self.check(self.lib.mdlc_event_record(self.h, int(slot)), "event_record")

    def event_elapsed(self, a: int, b: int) -> float:
        ms = C.c_float(0)
        self.check(self.lib.mdlc_event_elapsed(self.h, int(a), int(b), C.byref(ms)), "event_elapsed")
        return ms.value

    def launch_count(self) -> int:
        v = C.c_longlong(0)
        self.check(self.lib.mdlc_launch_count(self.h, C.byref(v)), "launch_count")
        return v.value

    def stream(self) -> int:
        s = C.c_void_p()
        self.check(self.lib.mdlc_get_stream(self.h, C.byref(s)), "get_stream")
        return s.value or 0

    def timeout_probe(self, limit_us: int) -> None:
        self.check(self.lib.mdlc_debug_timeout_probe(self.h, int(limit_us)), "timeout_probe")

    def poison_split_counters(self, value: int) -> None:
        self.check(self.lib.mdlc_debug_poison_split_counters(self.h, int(value)), "poison_split_counters")

    def close(self) -> None:
        if getattr(self, "h", None):
            for p in list(self._allocs):
                self.lib.mdlc_free(self.h, C.c_void_p(p))
            for p in list(self._host_allocs):
                self.lib.mdlc_host_free(self.h, C.c_void_p(p))
            self._allocs.clear()
            self._host_allocs.clear()
            self.lib.mdlc_ctx_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def weight_bytes(desc: ConvDesc) -> int:
    n = C.c_size_t(0)
    st = load().mdlc_conv_weight_bytes(C.byref(desc), C.byref(n))
    if st != OK:
        raise MdlcError(st, "conv_weight_bytes: unsupported conv configuration")
    return n.value


def gemm_weight_bytes(desc: GemmDesc) -> int:
    n = C.c_size_t(0)
    st = load().mdlc_gemm_weight_bytes(C.byref(desc), C.byref(n))
    if st != OK:
        raise MdlcError(st, "gemm_weight_bytes: unsupported GEMM configuration")
    return n.value


def pack_gemm_weights(desc: GemmDesc, b: np.ndarray) -> np.ndarray:
    """Pack B ([n, k] when ``desc.trans_b``, else [k, n]) scaled by ``desc.alpha`` (host)."""
    shape = (desc.n, desc.k) if desc.trans_b else (desc.k, desc.n)
    b = np.ascontiguousarray(b, dtype=np.float32)
    if b.shape != shape:
        raise ValueError(f"B has shape {b.shape}, descriptor wants {shape}")
    out = np.empty(gemm_weight_bytes(desc), dtype=np.uint8)
    st = load().mdlc_pack_gemm_weights(C.byref(desc), b.ctypes.data_as(C.c_void_p),
                                       out.ctypes.data_as(C.c_void_p))
    if st != OK:
        raise MdlcError(st, "pack_gemm_weights failed")
    return out


def pack_weights(desc: ConvDesc, w_oihw: np.ndarray) -> np.ndarray:
    """Pack OIHW fp32 weights (or int8 codes as float) into the kernel layout (host)."""
    w = np.ascontiguousarray(w_oihw, dtype=np.float32)
    out = np.empty(weight_bytes(desc), dtype=np.uint8)
    st = load().mdlc_pack_conv_weights(C.byref(desc), w.ctypes.data_as(C.c_void_p),
                                       out.ctypes.data_as(C.c_void_p))
    if st != OK:
        raise MdlcError(st, "pack_conv_weights failed")
    return out
