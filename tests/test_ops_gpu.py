"""Softmax, Transpose, Concat, Pad, BatchNormalization and Gemm transA=1 on
the device (the reference GPU executor ran these on the host,
mdlc/codegen/cuda/emit.py:32-35), against the oracle (ops.py semantics)."""

import numpy as np
import pytest

from mdlc_b200 import builders, compile, passes
from oracle import reference as oref
from test_ops_cpu import KINDS, ops_graph

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", KINDS)
def test_op_graph_matches_oracle(kind):
    g = passes.default_pipeline(ops_graph(kind))
    feeds = builders.make_input(g, seed=3)
    want = oref.run(g, feeds)["y"]
    emu = oref.run(g, feeds, bf16_emulation=True)["y"]
    scale = float(np.abs(want).max())
    for dtype in ("fp32", "bf16"):
        exe = compile(g, dtype=dtype)
        try:
            assert exe.fallbacks() == []
            got = exe.run(feeds)["y"]
        finally:
            exe.close()
        assert got.shape == want.shape
        if dtype == "fp32":
            np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4, err_msg=kind)
        else:
            np.testing.assert_allclose(got, emu, rtol=2e-2, atol=2e-2 * scale, err_msg=kind)
