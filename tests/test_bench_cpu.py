"""bench.py's own consistency, checked without a GPU: every function it calls
by name is defined in it or imported (a renamed helper fails here, not on
the GPU box), and the per-kernel-class table arithmetic."""

import ast
import builtins
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_bench_calls_only_defined_names():
    tree = ast.parse(open(os.path.join(ROOT, "bench.py")).read())
    defined = set(dir(builtins))
    for n in ast.walk(tree):
        if isinstance(n, (ast.FunctionDef, ast.ClassDef)):
            defined.add(n.name)
        elif isinstance(n, (ast.Import, ast.ImportFrom)):
            defined.update((a.asname or a.name).split(".")[0] for a in n.names)
        elif isinstance(n, ast.Name) and isinstance(n.ctx, ast.Store):
            defined.add(n.id)
        elif isinstance(n, ast.arg):
            defined.add(n.arg)
    called = {n.func.id for n in ast.walk(tree) if isinstance(n, ast.Call) and isinstance(n.func, ast.Name)}
    assert called - defined == set()


def test_kernel_table_fractions():
    sys.path.insert(0, ROOT)
    import bench
    table = {"conv_tc": {"launches": 2, "ms": 2.0, "bytes": 0, "flops": 2e12, "bound": "tensor"},
             "maxpool": {"launches": 1, "ms": 1.0, "bytes": 5e9, "flops": 0.0, "bound": "hbm"}}
    out = bench.kernel_table(table, 4.0, 1000.0, 5000.0)
    assert list(out) == ["conv_tc", "maxpool"]                 # by time
    assert out["conv_tc"]["achieved_tflops"] == 1000.0 and out["conv_tc"]["frac"] == 1.0
    assert out["maxpool"]["achieved_gbs"] == 5000.0 and out["maxpool"]["frac"] == 1.0
    assert out["conv_tc"]["share"] == 0.5 and out["conv_tc"]["avg_launch_us"] == 1000.0
