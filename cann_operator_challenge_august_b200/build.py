"""Build recipe for the in-tree CUDA library (sm_100a only).

    python -m cann_operator_challenge_august_b200.build     # or build() from Python

produces ``cann_operator_challenge_august_b200/libcgdr_fwd_h.so``: the C ABI
of include/cgdr_fwd_h.h with the tensor-core and general kernels, and
``runner/cgdr_fwd_h_case``: the golden-case runner (a plain C++ program over
that C ABI).  nvcc cross-compiles without a GPU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
LIB = PKG / "libcgdr_fwd_h.so"
SOURCES = [PKG / "csrc" / n for n in ("cgdr_fwd_h.cu", "cgdr_chunk_o.cu", "cgdr_wy.cu", "cgdr_gdr.cu", "host_util.cu")]
RUNNER_SRC = PKG / "runner" / "cgdr_fwd_h_case.cpp"
RUNNER = PKG / "runner" / "cgdr_fwd_h_case"
HEADERS = sorted((PKG / "csrc").glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-O3",
    "-Xptxas", "-v",
    "--expt-relaxed-constexpr",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA library cannot be built")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(src.stat().st_mtime > t for src in SOURCES + HEADERS)


def runner_needs_build() -> bool:
    if not RUNNER.exists():
        return True
    t = RUNNER.stat().st_mtime
    return any(src.stat().st_mtime > t for src in (RUNNER_SRC, LIB, ROOT / "include" / "cgdr_fwd_h.h"))


def build_runner(force: bool = False) -> Path:
    """Links the case runner against the in-tree library (found at run time
    through an $ORIGIN-relative rpath, so the tree can move)."""
    if not force and not runner_needs_build():
        return RUNNER
    # host code only: no device target to compile, so nvcc's default-target notice is moot
    cmd = [nvcc(), "-O2", "-std=c++17", "-Wno-deprecated-gpu-targets", "-o", str(RUNNER), str(RUNNER_SRC),
           "-L", str(PKG), "-lcgdr_fwd_h", "-Xlinker", "-rpath,$ORIGIN/.."]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = PKG / "build.log"
    with log.open("a") as f:
        f.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"building the case runner failed (exit {res.returncode}); see {log}")
    return RUNNER


def build(force: bool = False, verbose: bool = False) -> Path:
    if force or needs_build():
        cmd = [nvcc(), *NVCC_FLAGS, "-o", str(LIB), *map(str, SOURCES)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        log = PKG / "build.log"
        log.write_text(" ".join(cmd) + "\n" + res.stdout + res.stderr)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError(f"nvcc failed (exit {res.returncode}); see {log}")
        if verbose:
            sys.stdout.write(res.stderr)
    build_runner(force=force)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
