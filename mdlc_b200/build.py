"""Build ``libmdlc_b200.so`` (all CUDA kernels, sm_100a) in-tree.

    python -m mdlc_b200.build [--verbose] [--check]

``--check`` builds the bounds-checked variant ``libmdlc_b200_check.so``
(``-DMDLC_CHECK``: computed global-memory indices are checked against the
tensors' extents; a violation records ``MDLC_DEVERR_BOUNDS`` and skips the
access). ``_lib`` loads it when ``MDLC_B200_LIB=check``.

Each ``csrc/*.cu`` is compiled by nvcc in parallel into ``_build/`` and linked
into ``mdlc_b200/libmdlc_b200.so`` next to this file, which is where
:mod:`mdlc_b200._lib` loads it from. Incremental by content: each object
records a digest of its source, every header and the flags, taken before it
is compiled, and the library the digest of its objects' digests (in
``manifest.json`` of the build folder), so a file edited while a build runs
is compiled again by the next build.
"""

from __future__ import annotations

import argparse
import glob
import hashlib
import json
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


def _digest(*parts: bytes) -> str:
    h = hashlib.sha256()
    for p in parts:
        h.update(len(p).to_bytes(8, "little"))
        h.update(p)
    return h.hexdigest()


def _read(path: str) -> bytes:
    with open(path, "rb") as f:
        return f.read()


def _keys(flags: str) -> tuple:
    """(source basename -> digest, library digest) of the files as they are now."""
    headers = sorted(p for p in _deps() if not p.endswith(".cu"))
    hdr = _digest(*[p.encode() + b"\0" + _read(p) for p in headers])
    keys = {os.path.basename(s): _digest(flags.encode(), hdr.encode(), _read(s)) for s in _sources()}
    return keys, _digest(*[f"{k}={v}".encode() for k, v in sorted(keys.items())])


def _manifest(bdir: str) -> dict:
    try:
        with open(os.path.join(bdir, "manifest.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


def up_to_date(lib: str = LIB, check: bool = False) -> bool:
    bdir = CHECK_BUILD if check else BUILD
    if not os.path.exists(lib):
        return False
    _, lib_key = _keys(" ".join([*ARCH, *FLAGS, *(("-DMDLC_CHECK",) if check else ())]))
    return _manifest(bdir).get("__lib__") == lib_key


def build(force: bool = False, verbose: bool = False, extra=(), check: bool = False) -> str:
    lib, bdir = (CHECK_LIB, CHECK_BUILD) if check else (LIB, BUILD)
    if check:
        extra = (*extra, "-DMDLC_CHECK")
    os.makedirs(bdir, exist_ok=True)
    flags = " ".join([*ARCH, *FLAGS, *extra])
    keys, lib_key = _keys(flags)          # digests of the inputs as this build reads them
    manifest = _manifest(bdir)
    if not force and os.path.exists(lib) and manifest.get("__lib__") == lib_key:
        return lib

    def compile_one(src):
        name = os.path.basename(src)
        obj = os.path.join(bdir, name + ".o")
        if not force and os.path.exists(obj) and manifest.get(name) == keys[name]:
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
    with open(os.path.join(bdir, "manifest.json"), "w") as f:
        json.dump({**keys, "__lib__": lib_key}, f, indent=1, sort_keys=True)
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
