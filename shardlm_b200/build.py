"""Build libshardlm_cuda.so (sm_100a) and the CPU oracle library.

The CUDA library is compiled in-tree with nvcc so the shared object travels with the repository
snapshot: ``shardlm_b200/lib/libshardlm_cuda.so``. The oracle (test infrastructure, never linked
by the library) is compiled with g++ into ``oracle/_build/liboracle.so``.
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
LIBDIR = PKG / "lib"
OBJDIR = PKG / "_build"
LIB = LIBDIR / "libshardlm_cuda.so"
INCLUDE = ROOT / "include"

ORACLE_DIR = ROOT / "oracle"
ORACLE_LIB = ORACLE_DIR / "_build" / "liboracle.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libshardlm_cuda.so")


def _nccl_include() -> list[str]:
    try:
        import nvidia.nccl  # type: ignore

        for p in nvidia.nccl.__path__:
            inc = Path(p) / "include"
            if (inc / "nccl.h").exists():
                return ["-I", str(inc)]
    except Exception:
        pass
    if Path("/usr/include/nccl.h").exists():
        return []
    raise RuntimeError("nccl.h not found")


def _newest(paths) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def library_stale() -> bool:
    if not LIB.exists():
        return True
    return _newest(_sources() + _headers()) > LIB.stat().st_mtime


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libshardlm_cuda.so."""
    if not force and not library_stale():
        return LIB
    nvcc = _nvcc()
    OBJDIR.mkdir(parents=True, exist_ok=True)
    LIBDIR.mkdir(parents=True, exist_ok=True)
    inc = ["-I", str(INCLUDE)] + _nccl_include()
    hdr_time = _newest(_headers())

    def compile_one(src: Path) -> Path:
        obj = OBJDIR / (src.stem + ".o")
        if force or not obj.exists() or max(src.stat().st_mtime, hdr_time) > obj.stat().st_mtime:
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *inc, "-c", str(src), "-o", str(obj)]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout, r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def oracle_stale() -> bool:
    if not ORACLE_LIB.exists():
        return True
    srcs = list(ORACLE_DIR.glob("*.cpp")) + list(ORACLE_DIR.glob("*.h"))
    return _newest(srcs) > ORACLE_LIB.stat().st_mtime


def build_oracle(force: bool = False) -> Path:
    """Compile the CPU oracle with the float rules of the reference (no contraction, no fast-math)."""
    if not force and not oracle_stale():
        return ORACLE_LIB
    r = subprocess.run(["make", "-C", str(ORACLE_DIR)], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return ORACLE_LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build_library(force=force, verbose=True))
    print(build_oracle(force=force))
