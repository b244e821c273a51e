"""The bounds-checked build (``python -m mdlc_b200.build --check``,
``-DMDLC_CHECK``) runs the kernel tests' small shapes with every computed
global-memory index checked against its tensor's extent; a violation would
record ``MDLC_DEVERR_BOUNDS`` in the context's error word, which every
``Context.sync()`` turns into a test failure. The checked library is loaded in
a child process (``MDLC_B200_LIB=check``), one library per process."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CHECK_LIB = os.path.join(ROOT, "mdlc_b200", "libmdlc_b200_check.so")


@pytest.mark.skipif(not os.path.exists(CHECK_LIB), reason="checked build not built")
def test_kernel_shapes_under_bounds_checks():
    env = dict(os.environ, MDLC_B200_LIB="check")
    probe = subprocess.run([sys.executable, "-c", "from mdlc_b200 import _lib; print(_lib.load()._name)"],
                           cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert probe.returncode == 0 and probe.stdout.strip().endswith("libmdlc_b200_check.so"), probe.stderr
    r = subprocess.run([sys.executable, "-m", "pytest", "tests/test_kernels_gpu.py", "-x", "-p",
                        "no:cacheprovider", "-k",
                        "conv_bf16_tcgen05 or tile_configs or split_k or im2col or pointwise or depthwise "
                        "or grouped or fp32 or gemm or pools or eltwise"],
                       cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout
