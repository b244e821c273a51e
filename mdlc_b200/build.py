"""Build ``libmdlc_b200.so`` (all CUDA kernels, sm_100a) in-tree.

    python -m mdlc_b200.build [--verbose] [--check]

``--check`` builds the bounds-checked variant ``libmdlc_b200_check.so``
(``-DMDLC_CHECK``: computed global-memory indices are checked against the
tensors' extents; a violation records ``MDLC_DEVERR_BOUNDS`` and skips the
access). ``_lib`` loads it when ``MDLC_B200_LIB=check``.

Each ``csrc/*.cu`` is compiled by nvcc in parallel into ``_build/`` and linked
into ``mdlc_b200/libmdlc_b200.so`` next to this file, which is where
:mod:`mdlc_b200._lib` loads it from. Rebuilds only when a source or header is
newer than the library.
"""

from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libmdlc_b200.so")
CHECK_BUILD = os.path.join(ROOT, "_build_check")
CHECK_LIB = os.path.join(HERE, "libmdlc_b200_check.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def up_to_date(lib: str = LIB) -> bool:
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, extra=(), check: bool = False) -> str:
    lib, bdir = (CHECK_LIB, CHECK_BUILD) if check else (LIB, BUILD)
    if check:
        extra = (*extra, "-DMDLC_CHECK")
    if not force and up_to_date(lib):
        return lib
    os.makedirs(bdir, exist_ok=True)

    headers = [p for p in _deps() if not p.endswith(".cu")]
    newest_header = max((os.path.getmtime(p) for p in headers), default=0.0)
    flags_file = os.path.join(bdir, "flags.txt")
    flags = " ".join([*ARCH, *FLAGS, *extra])
    same_flags = os.path.exists(flags_file) and open(flags_file).read() == flags

    def compile_one(src):
        obj = os.path.join(bdir, os.path.basename(src) + ".o")
        # incremental: an object newer than its source and every header is reused
        if (not force and same_flags and os.path.exists(obj) and
                os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header)):
            return obj, ""
        cmd = [NVCC, *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(compile_one, _sources()))
    with open(flags_file, "w") as f:
        f.write(flags)
    if verbose:
        for _, log in results:
            sys.stderr.write(log)
    tmp = lib + ".tmp"
    cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *[o for o, _ in results], "-lcudart_static", "-ldl", "-lrt",
           "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, lib)
    return lib


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    ap.add_argument("--check", action="store_true", help="the bounds-checked variant (-DMDLC_CHECK)")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, check=args.check))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
