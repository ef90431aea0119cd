"""Builds libzilla_b200.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m zillaphp_b200.build          # incremental
    python -m zillaphp_b200.build --clean

Objects go to zillaphp_b200/_build/, the library to zillaphp_b200/lib/.
NCCL (data-parallel runner) is linked from the nvidia-nccl wheel that ships
with PyTorch; the library resolves it through an rpath.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libzilla_b200.so")
ROOT = os.path.dirname(PKG)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-I" + os.path.join(ROOT, "include")]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _nccl() -> tuple[str, str] | None:
    """(include dir, lib dir) of the NCCL wheel, if present."""
    try:
        import nvidia.nccl as n  # type: ignore
        base = list(n.__path__)[0]
    except Exception:
        return None
    inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
    if os.path.exists(os.path.join(inc, "nccl.h")) and glob.glob(os.path.join(lib, "libnccl.so*")):
        return inc, lib
    return None


def _compile(src: str, obj: str, extra: list[str]) -> None:
    cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")


def build(clean: bool = False, verbose: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    newest_header = max((os.path.getmtime(h) for h in headers), default=0)
    nccl = _nccl()
    extra = ["-DZB_HAVE_NCCL=1", "-I" + nccl[0]] if nccl else []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        if not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s), newest_header):
            jobs.append((s, o))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        futs = [ex.submit(_compile, s, o, extra) for s, o in jobs]
        for f in futs:
            f.result()
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        link = [_nvcc(), *ARCH, "-shared", "-o", LIB, *objs]
        if nccl:
            libfile = sorted(glob.glob(os.path.join(nccl[1], "libnccl.so*")))[0]
            link += ["-L" + nccl[1], "-l:" + os.path.basename(libfile), "-Xlinker", "-rpath=" + nccl[1]]
        r = subprocess.run(link, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(clean="--clean" in sys.argv, verbose=True)
