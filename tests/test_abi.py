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


STRUCTS = {"mdlc_epilogue": "Epilogue", "mdlc_conv_desc": "ConvDesc", "mdlc_tile_cfg": "TileCfg",
           "mdlc_pool_desc": "PoolDesc", "mdlc_ew_instr": "EwInstr", "mdlc_ew_prog": "EwProg",
           "mdlc_gemm_desc": "GemmDesc", "mdlc_copy_desc": "CopyDesc", "mdlc_softmax_desc": "SoftmaxDesc",
           "mdlc_se_desc": "SeDesc"}


def test_struct_layouts_match_header(tmp_path):
    """Every ctypes mirror has the size and field offsets the C compiler gives
    the header's struct (a C program including include/mdlc_b200.h prints them)."""
    import ctypes as C
    import shutil
    import subprocess
    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler")
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "mdlc_b200.h"', "int main(void) {"]
    for cname, pname in STRUCTS.items():
        lines.append(f'printf("{pname} size %zu\\n", sizeof({cname}));')
        for field, _ in getattr(L, pname)._fields_:
            lines.append(f'printf("{pname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run([gcc, "-I", inc, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.split("\n")
    checked = 0
    for line in filter(None, out):
        pname, field, value = line.split()
        cls = getattr(L, pname)
        got = C.sizeof(cls) if field == "size" else getattr(cls, field).offset
        assert got == int(value), f"{pname}.{field}: ctypes {got}, C {value}"
        checked += 1
    assert checked == sum(1 + len(getattr(L, p)._fields_) for p in STRUCTS.values())


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
        # fp32 (3xTF32): [hi matrix][lo matrix], each [k][kg_pad] with 32-element k-blocks
        kg_pad = 96   # 72 -> three 32-element k-blocks
        q = p.view(np.float32).reshape(2, k, kg_pad)
        full = np.zeros((k, kg_pad), np.float32)
        full[:, :72] = np.pad(w.transpose(0, 2, 3, 1), ((0, 0), (0, 0), (0, 0), (0, 5))).reshape(k, 72)
        hi = (full.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)
        np.testing.assert_array_equal(q[0], hi)
        np.testing.assert_array_equal(q[1], full - hi)
        assert np.all((q[0].view(np.uint32) & 0x1FFF) == 0)              # hi is exactly a tf32 value
        np.testing.assert_array_equal(q[0].astype(np.float64) + q[1], full.astype(np.float64))  # split is exact
