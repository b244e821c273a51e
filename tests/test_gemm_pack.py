"""Host-side GEMM weight packing through the C ABI (no GPU needed).

``mdlc_pack_gemm_weights`` maps a Gemm's B operand onto the 1x1-convolution
weight layout: transB selects [n, k] or [k, n] storage and alpha is folded into
the packed values (mdlc/codegen/cuda/emit.py:211-244 takes the same attributes).
"""

import numpy as np
import pytest

from mdlc_b200 import _lib as L


def _desc(**kw):
    base = dict(m=16, n=24, k=40, lda=40, trans_a=0, trans_b=1, alpha=1.0, in_type=L.BF16, out_type=L.BF16)
    base.update(kw)
    return L.GemmDesc(**base)


@pytest.mark.parametrize("et", [L.BF16, L.F32, L.U8])
def test_trans_b_is_a_layout_choice(et):
    rng = np.random.default_rng(3)
    b = rng.integers(-100, 100, (24, 40)).astype(np.float32)     # [n, k]
    p1 = L.pack_gemm_weights(_desc(trans_b=1, in_type=et, out_type=et, lda=48 if et == L.U8 else 40), b)
    p0 = L.pack_gemm_weights(_desc(trans_b=0, in_type=et, out_type=et, lda=48 if et == L.U8 else 40), b.T.copy())
    np.testing.assert_array_equal(p1, p0)


def test_alpha_is_folded_into_the_weights():
    rng = np.random.default_rng(4)
    b = rng.standard_normal((24, 40)).astype(np.float32)
    np.testing.assert_array_equal(L.pack_gemm_weights(_desc(alpha=2.0), b),
                                  L.pack_gemm_weights(_desc(alpha=1.0), 2.0 * b))


def test_bad_descriptors_are_rejected():
    with pytest.raises(L.MdlcError):
        L.gemm_weight_bytes(_desc(trans_a=1))
    with pytest.raises(L.MdlcError):
        L.gemm_weight_bytes(_desc(k=0))
    with pytest.raises(ValueError):
        L.pack_gemm_weights(_desc(), np.zeros((40, 24), np.float32))   # wrong orientation for trans_b=1
