"""Build libtqb200.so (CUDA sm_100a) in-tree with nvcc.

Every csrc/*.cu compiles for ``-gencode arch=compute_100a,code=sm_100a`` and
links into tiny-llm_b200/libtqb200.so next to this file, so the library
travels with the source tree.  Objects are rebuilt only when a source or
header is newer.  ``python tiny-llm_b200/build.py [-v]`` runs it by hand.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtqb200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def nccl_dirs():
    """NCCL headers and library shipped with torch's nvidia-nccl wheel."""
    try:
        import nvidia.nccl as n  # type: ignore
        base = list(n.__path__)[0]
    except Exception:
        return None, None
    inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
        return inc, lib
    return None, None


def _flags():
    inc, _ = nccl_dirs()
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]
    if inc:
        f += ["-I", inc, "-DTQB200_HAVE_NCCL=1"]
    return f


def _newer(src: str, dst: str, deps) -> bool:
    if not os.path.exists(dst):
        return True
    t = os.path.getmtime(dst)
    return any(os.path.getmtime(d) > t for d in [src] + list(deps))


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    cc = nvcc()
    flags = _flags() + (["-Xptxas", "-v"] if ptxas_verbose else [])
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(OBJ, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if _newer(s, o, headers) or ptxas_verbose:
            jobs.append([cc] + flags + ["-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        outs = list(ex.map(run, jobs))
    if verbose or ptxas_verbose:
        for o in outs:
            if o.strip():
                print(o)
    if jobs or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        _, nlib = nccl_dirs()
        link = [cc] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcuda"]
        if nlib:
            link += ["-L", nlib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + nlib]
        run(link)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
