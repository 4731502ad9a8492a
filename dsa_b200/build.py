"""Build libdsa_b200.so in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into
``dsa_b200/_build/`` and linked into ``dsa_b200/libdsa_b200.so`` (static
cudart, so the library depends only on the driver). Objects are rebuilt when
their source or any ``csrc`` header is newer.

``--bounds-check`` builds the debugging variant
``dsa_b200/libdsa_b200_checked.so`` (same ABI, ``-DDSA_BOUNDS_CHECK``):
every gathered row index, batch row, shared-memory stage destination and
tensor-memory column is checked, and a failed check sets bit 4 of the
status word instead of trapping.

Usage: ``python -m dsa_b200.build [--force] [--verbose] [--bounds-check]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libdsa_b200.so")
LIB_CHECKED = os.path.join(HERE, "libdsa_b200_checked.so")
BUILD_CHECKED = os.path.join(BUILD, "checked")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-fvisibility=hidden", "-I", CSRC, "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the sm_100a library cannot be built")


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src: str, force: bool, verbose: bool, extra=(), build_dir=BUILD) -> str:
    obj = os.path.join(build_dir, src[:-3] + ".o")
    path = os.path.join(CSRC, src)
    if (not force and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(path), _headers_mtime())):
        return obj
    cmd = [nvcc(), *ARCH_FLAGS, *CFLAGS, *extra, "-c", path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False, bounds_check: bool = False) -> str:
    """Compile and link the library (or its bounds-checking variant); returns its path."""
    build_dir, lib = (BUILD_CHECKED, LIB_CHECKED) if bounds_check else (BUILD, LIB)
    extra = ("-DDSA_BOUNDS_CHECK",) if bounds_check else ()
    os.makedirs(build_dir, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, verbose, extra, build_dir), srcs))
    if (force or not os.path.exists(lib)
            or os.path.getmtime(lib) < max(os.path.getmtime(o) for o in objs)):
        tmp = lib + ".tmp"
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lcuda"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--bounds-check", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, bounds_check=args.bounds_check))
