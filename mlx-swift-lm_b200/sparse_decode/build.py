"""Build libsparse_decode.so (sm_100a) in-tree with nvcc.

The library is compiled from mlx-swift-lm_b200/csrc: one object per storage
format (sd_inst.cu with SD_E/SD_BITS), plus the C ABI (sd_api.cu). The CUDA
runtime is linked statically, so the .so only needs the driver at run time.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent          # mlx-swift-lm_b200/
CSRC = PKG_DIR / "csrc"
BUILD = PKG_DIR / "_build"
LIB = PKG_DIR / "libsparse_decode.so"
INCLUDE = PKG_DIR.parent / "include"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         f"-I{INCLUDE}", f"-I{CSRC}"]
FORMATS = [(e, b) for b in (0, 4, 8) for e in (0, 1, 2)]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        INCLUDE / "sparse_decode.h"]


def _stale(target: Path) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in _sources())


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel object and link the shared library; returns its path."""
    if not force and not _stale(LIB):
        return LIB
    BUILD.mkdir(exist_ok=True)
    jobs = []
    for e, b in FORMATS:
        obj = BUILD / f"sd_inst_e{e}_b{b}.o"
        jobs.append([NVCC, *ARCH, *FLAGS, f"-DSD_E={e}", f"-DSD_BITS={b}", "-c", str(CSRC / "sd_inst.cu"),
                     "-o", str(obj)])
    jobs.append([NVCC, *ARCH, *FLAGS, "-c", str(CSRC / "sd_api.cu"), "-o", str(BUILD / "sd_api.o")])
    with cf.ThreadPoolExecutor(max_workers=max(2, os.cpu_count() or 2)) as ex:
        for f in cf.as_completed([ex.submit(_run, j) for j in jobs]):
            f.result()
            if verbose:
                print(".", end="", flush=True)
    objs = [str(BUILD / f"sd_inst_e{e}_b{b}.o") for e, b in FORMATS] + [str(BUILD / "sd_api.o")]
    tmp = LIB.with_suffix(".so.tmp")
    _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart=static"])
    tmp.replace(LIB)
    if verbose:
        print(f" built {LIB}")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
