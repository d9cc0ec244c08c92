"""Builds libflashmlp_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m flashmlp_b200.build`` (or ``__graft_entry__.build()``). The library is
written next to this file so it travels with the source tree; nothing is installed.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR.parent / "_build"
LIB_NAME = "libflashmlp_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
SOURCES = ["fmlp_fwd.cu", "fmlp_fwd_pair.cu", "fmlp_fwd2sm.cu", "fmlp_fwd_fp8.cu", "fmlp_bwd.cu", "fmlp_bwd256.cu", "fmlp_capi.cu",
           "fmlp_noalloc.cu", "fmlp_comm.cu", "fmlp_tf32.cu", "fmlp_dxgemm.cu", "fmlp_dwgemm256.cu"]
HEADERS = ["fmlp_ptx.cuh", "fmlp_act.cuh", "fmlp_kernels.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC or put CUDA's bin directory on PATH")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [PKG_DIR.parent / "include" / "flashmlp_b200.h"]
    objs = []
    jobs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD_DIR / (Path(src).stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(s), "-o", str(o)]
            jobs.append((src, cmd, o))

    def run(job):
        src, cmd, o = job
        r = subprocess.run(cmd, capture_output=True, text=True)
        log = BUILD_DIR / (Path(src).stem + ".ptxas.log")
        log.write_text(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr[-8000:]}")
        return src

    with cf.ThreadPoolExecutor(max_workers=len(jobs) or 1) as ex:
        for src in ex.map(run, jobs):
            if verbose:
                print(f"[flashmlp_b200.build] compiled {src}", file=sys.stderr)

    if force or jobs or _stale(LIB_PATH, objs):
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", *map(str, objs), "-o", str(LIB_PATH)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr[-8000:]}")
        if verbose:
            print(f"[flashmlp_b200.build] linked {LIB_PATH}", file=sys.stderr)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
