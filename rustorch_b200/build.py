"""Build librustorch_b200.so (sm_100a) in-tree with nvcc.

    python -m rustorch_b200.build [--force] [--verbose]

Each csrc/*.cu and csrc/*.cpp compiles to _build/*.o in parallel, then links into
rustorch_b200/librustorch_b200.so (NCCL is dlopen'ed at first use).  A source is
recompiled when it or any header is newer than its object, and the library is
relinked when any object changed.  Objects and the library are stamped with the time
their compile started, so a file edited while a build runs is seen as newer by the
next build.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys
import time

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "librustorch_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "-I" + os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + [
        os.path.join(ROOT, "include", "rustorch_b200.h")]


def _obj(src: str) -> str:
    return os.path.join(BUILD, os.path.basename(src).rsplit(".", 1)[0] + ".o")


def _stale(src: str, newest_header: float) -> bool:
    obj = _obj(src)
    if not os.path.exists(obj):
        return True
    return os.path.getmtime(obj) < max(os.path.getmtime(src), newest_header)


def needs_build() -> bool:
    """The library is missing or older than a source or header (objects are
    not needed to use a library that is up to date)."""
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    return any(os.path.getmtime(p) > t for p in _sources() + _headers() + [__file__])


def _compile(src: str, verbose: bool) -> str:
    obj = _obj(src)
    t0 = time.time()
    cmd = [_nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stdout + r.stderr)
    os.utime(obj, (t0, t0))
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdr = max(os.path.getmtime(p) for p in _headers())
    todo = [s for s in srcs if force or verbose or _stale(s, hdr)]
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            list(ex.map(lambda s: _compile(s, verbose), todo))
    objs = [_obj(s) for s in srcs]
    tmp = LIB + ".tmp"
    cmd = [_nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-lcudart_static",
                                                               "-lrt", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp = max(os.path.getmtime(o) for o in objs)
    os.utime(LIB, (stamp, stamp))
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
