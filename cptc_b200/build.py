"""Builds the native parts of cptc_b200 in-tree.

  cptc_b200/_lib/libcptc_host.so  host-only library (generators, .tns I/O, binary cache)
  cptc_b200/_lib/libcptc.so       the CUDA engine (sm_100a) with the C ABI
  cptc_b200/_lib/cptc_opt         the command-line driver

Kernels are compiled for sm_100a only (``-gencode arch=compute_100a,
code=sm_100a``); nvcc cross-compiles without a GPU.  Objects go to
cptc_b200/_build/.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "_lib"
OBJ = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
HOST_SRCS = ["host/gen.cpp", "host/tns.cpp", "host/bincache.cpp", "host/reorder.cpp"]
CUDA_SRCS = [
    "cuda/views.cu",
    "cuda/mttkrp_sparse.cu",
    "cuda/tiles.cu",
    "cuda/tiles_pool.cu",
    "cuda/units.cu",
    "cuda/als_kernels.cu",
    "cuda/comm.cu",
    "cuda/shard.cu",
    "cuda/reorder_gpu.cu",
    "cuda/engine.cu",
    "cuda/noalloc.cu",
    "cuda/probe.cu",
]


def _nccl_paths() -> tuple[str, str]:
    """Header and library folders of the NCCL that torch loads."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia.nccl")
    if spec is None or not spec.submodule_search_locations:
        raise RuntimeError("nvidia.nccl (torch's NCCL) not found")
    base = Path(list(spec.submodule_search_locations)[0])
    return str(base / "include"), str(base / "lib")


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[0]} ... {cmd[-1]}")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _headers() -> list[Path]:
    hs = list((CSRC).rglob("*.hpp")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return hs


def build_host(verbose: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / "libcptc_host.so"
    srcs = [CSRC / s for s in HOST_SRCS]
    if _stale(out, srcs + _headers()):
        _run(["g++", "-O3", "-std=c++17", "-fPIC", "-fopenmp", "-shared", "-o", str(out)]
             + [str(s) for s in srcs], verbose)
    return out


def build_cuda(verbose: bool = False, jobs: int | None = None) -> Path:
    LIB.mkdir(exist_ok=True)
    OBJ.mkdir(exist_ok=True)
    nccl_inc, nccl_lib = _nccl_paths()
    hdrs = _headers()
    cflags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fopenmp", "-ccbin", "g++",
              f"-I{nccl_inc}", f"-I{ROOT / 'include'}"] + ARCH
    objs = []
    todo = []
    for s in CUDA_SRCS + HOST_SRCS:
        src = CSRC / s
        obj = OBJ / (s.replace("/", "_") + ".o")
        objs.append(obj)
        if _stale(obj, [src] + hdrs):
            if s.endswith(".cu"):
                cmd = ["nvcc"] + cflags + ["-c", str(src), "-o", str(obj)]
            else:
                cmd = ["g++", "-O3", "-std=c++17", "-fPIC", "-fopenmp", f"-I{ROOT / 'include'}",
                       "-c", str(src), "-o", str(obj)]
            todo.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        list(ex.map(lambda c: _run(c, verbose), todo))
    out = LIB / "libcptc.so"
    if todo or _stale(out, objs):
        _run(["nvcc", "-shared", "-ccbin", "g++", "--cudart", "static"] + ARCH
             + [str(o) for o in objs]
             + ["-o", str(out), f"-L{nccl_lib}", "-l:libnccl.so.2", "-lgomp",
                "-Xlinker", f"-rpath={nccl_lib}"], verbose)
    return out


def build_cli(verbose: bool = False) -> Path:
    out = LIB / "cptc_opt"
    src = CSRC / "cli" / "cptc_opt.cpp"
    if src.exists() and _stale(out, [src, LIB / "libcptc.so"] + _headers()):
        _run(["g++", "-O2", "-std=c++17", f"-I{ROOT / 'include'}", str(src), "-o", str(out),
              f"-L{LIB}", "-lcptc", f"-Wl,-rpath,{LIB}", "-fopenmp"], verbose)
    return out


def build_gen(verbose: bool = False) -> Path:
    """cptc_gen: the .tns generator as a self-contained executable (the
    generator and writer sources compiled in, no library of this project
    loaded at run time)."""
    LIB.mkdir(exist_ok=True)
    out = LIB / "cptc_gen"
    srcs = [CSRC / "cli" / "cptc_gen.cpp", CSRC / "host" / "gen.cpp", CSRC / "host" / "tns.cpp"]
    if _stale(out, srcs + _headers()):
        _run(["g++", "-O3", "-std=c++17", "-fopenmp", f"-I{ROOT / 'include'}"]
             + [str(s) for s in srcs] + ["-o", str(out)], verbose)
    return out


def build_all(verbose: bool = False) -> None:
    build_host(verbose)
    build_cuda(verbose)
    build_cli(verbose)
    build_gen(verbose)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built", LIB)
