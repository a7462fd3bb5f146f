"""Build libsparse_decode.so (sm_100a) in-tree with nvcc.

The library is compiled from mlx-swift-lm_b200/csrc: one object per storage
format (sd_inst.cu with SD_E/SD_BITS), plus the C ABI (sd_api.cu). The CUDA
runtime is linked statically, so the .so only needs the driver at run time.

`build(phase_timing=True)` makes a second library, libsparse_decode_phases.so,
compiled with -DSD_PHASE_TIMING: the decode kernel then writes per-phase
timestamps (sparse_decode.phase_profile reads them). The product library has
no stamps.
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
LIB_PHASES = PKG_DIR / "libsparse_decode_phases.so"
INCLUDE = PKG_DIR.parent / "include"

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         f"-I{INCLUDE}", f"-I{CSRC}"]
FORMATS = [(e, b) for b in (0, 4, 8) for e in (0, 1, 2)]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [
        INCLUDE / "sparse_decode.h"]


def _kernel_sources() -> list[Path]:
    """What the kernel objects (sd_inst.cu) depend on: everything but sd_api.cu."""
    return [s for s in _sources() if s.name not in ("sd_api.cu", "sparse_decode.h")]


def _api_sources() -> list[Path]:
    return [CSRC / "sd_api.cu", CSRC / "sd_format.h", CSRC / "sd_params.h", CSRC / "sd_kernels.h",
            INCLUDE / "sparse_decode.h"]


def _stale(target: Path, sources: list[Path] | None = None) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in (sources if sources is not None else _sources()))


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False, phase_timing: bool = False) -> Path:
    """Compile every kernel object and link the shared library; returns its path."""
    lib = LIB_PHASES if phase_timing else LIB
    bdir = PKG_DIR / "_build_phases" if phase_timing else BUILD
    flags = FLAGS + (["-DSD_PHASE_TIMING"] if phase_timing else [])
    bdir.mkdir(exist_ok=True)
    jobs = []
    for e, b in FORMATS:
        obj = bdir / f"sd_inst_e{e}_b{b}.o"
        if force or _stale(obj, _kernel_sources()):
            jobs.append([NVCC, *ARCH, *flags, f"-DSD_E={e}", f"-DSD_BITS={b}", "-c", str(CSRC / "sd_inst.cu"),
                         "-o", str(obj)])
    if force or _stale(bdir / "sd_api.o", _api_sources()):
        jobs.append([NVCC, *ARCH, *flags, "-c", str(CSRC / "sd_api.cu"), "-o", str(bdir / "sd_api.o")])
    with cf.ThreadPoolExecutor(max_workers=max(2, os.cpu_count() or 2)) as ex:
        for f in cf.as_completed([ex.submit(_run, j) for j in jobs]):
            f.result()
            if verbose:
                print(".", end="", flush=True)
    objs = [str(bdir / f"sd_inst_e{e}_b{b}.o") for e, b in FORMATS] + [str(bdir / "sd_api.o")]
    if not force and not jobs and not _stale(lib, [Path(o) for o in objs]):
        return lib
    tmp = lib.with_suffix(".so.tmp")
    _run([NVCC, *ARCH, "-shared", "-o", str(tmp), *objs, "-cudart=static"])
    tmp.replace(lib)
    if verbose:
        print(f" built {lib}")
    return lib


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, phase_timing="--phases" in sys.argv)
