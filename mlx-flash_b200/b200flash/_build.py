"""Build libb200flash.so (all CUDA sources for sm_100a) in-tree.

    python -m b200flash._build          # from mlx-flash_b200/
    python mlx-flash_b200/b200flash/_build.py

Objects go to ``mlx-flash_b200/_build/``; the shared library is written next
to this file as ``lib/libb200flash.so`` so it travels with the source tree.
Sources are recompiled only when they (or a header) are newer than their object.
"""

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
PROJ = os.path.dirname(PKG)
REPO = os.path.dirname(PROJ)
CSRC = os.path.join(PROJ, "csrc")
INCLUDE = os.path.join(REPO, "include")
BUILD = os.path.join(PROJ, "_build")
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libb200flash.so")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
         "--expt-relaxed-constexpr", f"-I{INCLUDE}", f"-I{CSRC}"]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max((os.path.getmtime(h) for h in hs), default=0.0)


def _compile(src, hdr_mtime, verbose):
    s = os.path.join(CSRC, src)
    o = os.path.join(BUILD, src[:-3] + ".o")
    if os.path.exists(o) and os.path.getmtime(o) >= max(os.path.getmtime(s), hdr_mtime):
        return o, False
    cmd = [NVCC, *ARCH, *FLAGS, "-c", s, "-o", o]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return o, True


def build(verbose: bool = False, jobs: int = 0) -> str:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``lib/libb200flash.so``."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    hdr = _headers_mtime()
    srcs = _sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, hdr, verbose), srcs))
    objs = [o for o, _ in results]
    changed = any(ch for _, ch in results)
    if changed or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
