"""The C ABI library loads and exports every function the header declares
(no GPU needed: nothing here launches a kernel)."""

import os
import re

import numpy as np
import pytest

from conftest import ROOT
from mdlc_b200 import _lib as L

HEADER = os.path.join(ROOT, "include", "mdlc_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\s*\*?\s*(mdlc_\w+)\s*\(", text, flags=re.M)))


def test_library_exports_every_declared_function():
    lib = L.load()
    names = declared_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
        assert n in L.SIGNATURES, f"{n} has no ctypes signature"
    assert set(L.SIGNATURES) <= set(names)


def test_struct_layouts_match_header():
    # field counts mirror the header structs; sizes follow from int32/float/pointer fields
    import ctypes as C
    assert C.sizeof(L.ConvDesc) == 22 * 4
    assert C.sizeof(L.PoolDesc) == 20 * 4
    assert C.sizeof(L.TileCfg) == 12
    assert C.sizeof(L.EwInstr) == 12
    assert C.sizeof(L.EwProg) == 8 * 4 + 4 * 4 + 2 * 4 + 24 * 12
    assert C.sizeof(L.Epilogue) == 5 * 4 + 4 + 8 + 4 * 4 + 4 + 4 + 2 * 8  # padding before the first pointer


def test_version_and_no_device_here():
    lib = L.load()
    assert lib.mdlc_version() == 100
    if L.device_count() == 0:
        with pytest.raises(L.MdlcError):
            L.Context(0)


@pytest.mark.parametrize("path", ["tc", "f32", "dw"])
def test_weight_packing_layouts(path):
    """Host-side packer: reference OIHW -> kernel layouts (no device needed)."""
    rng = np.random.default_rng(0)
    if path == "dw":
        c = 24
        w = rng.standard_normal((c, 1, 3, 3)).astype(np.float32)
        d = L.ConvDesc(n=1, h=5, w=5, c=c, c_stride=24, k=c, k_stride=24, r=3, s=3, stride_h=1, stride_w=1,
                       pad_t=1, pad_l=1, dil_h=1, dil_w=1, oh=5, ow=5, groups=c, in_type=L.BF16,
                       out_type=L.BF16)
        p = L.pack_weights(d, w).view(np.float32).reshape(9, 24)
        np.testing.assert_array_equal(p, w.reshape(c, 9).T)
        return
    c, k = 3, 10
    w = rng.standard_normal((k, c, 3, 3)).astype(np.float32)
    et = L.BF16 if path == "tc" else L.F32
    d = L.ConvDesc(n=1, h=5, w=5, c=c, c_stride=8, k=k, k_stride=16, r=3, s=3, stride_h=1, stride_w=1,
                   pad_t=1, pad_l=1, dil_h=1, dil_w=1, oh=5, ow=5, groups=1, in_type=et, out_type=et)
    p = L.pack_weights(d, w)
    if path == "tc":
        from oracle.reference import round_bf16
        kg_pad = 128  # 9 taps x 8 channels = 72 -> padded to 128 (two 64-element k-blocks)
        q = p.view(np.uint16).reshape(k, kg_pad)
        f = (q.astype(np.uint32) << 16).view(np.float32)
        want = np.zeros((k, kg_pad), np.float32)
        want[:, :72] = np.pad(round_bf16(w).transpose(0, 2, 3, 1), ((0, 0), (0, 0), (0, 0), (0, 5))).reshape(k, 72)
        np.testing.assert_array_equal(f, want)
    else:
        q = p.view(np.float32).reshape(72, 16)
        want = np.zeros((72, 16), np.float32)
        want[:, :k] = np.pad(w.transpose(2, 3, 1, 0), ((0, 0), (0, 0), (0, 5), (0, 0))).reshape(72, k)
        np.testing.assert_array_equal(q, want)
