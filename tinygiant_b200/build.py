"""Builds tinygiant_b200/libtinygiant.so (CUDA for sm_100a + host C++).

    python -m tinygiant_b200.build [-v] [--force]

The library is built in-tree so it travels with the repository to a GPU
host.  nvcc cross-compiles for sm_100a without a GPU present.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libtinygiant.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# --fmad=false: the kernels reproduce the reference's separately rounded
# float operations; a contracted a*b+c would change results.
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "-I", str(ROOT / "include")]
SOURCES = ["tg_kernels.cu", "tg_moe.cu", "tg_route.cu", "tg_runtime.cu", "tg_layer.cu", "tg_step.cu", "tg_gemm.cu",
           "tg_attention.cu", "tg_noalloc.cu"]
HEADERS = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "tinygiant.h"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src, verbose):
    obj = BUILD / (src + ".o")
    deps = [CSRC / src] + HEADERS
    if not _stale(obj, deps):
        return obj, False
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", str(CSRC / src), "-o", str(obj)]
    if src.endswith(".cu"):
        cmd[1:1] = ["-x", "cu"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj, True


def build(verbose=False, force=False):
    BUILD.mkdir(exist_ok=True)
    if force:
        for o in BUILD.glob("*.o"):
            o.unlink()
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    objs = [o for o, _ in results]
    if any(changed for _, changed in results) or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "--cudart", "static", "-o", str(LIB)] + [str(o) for o in objs] + [
            "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.force))
