"""Build the sm_100a shared library ``lib/libpa_b200.so`` in-tree with nvcc.

The library exports the C ABI declared in ``include/paged_attention_b200.h``.
It links only the CUDA runtime (the driver's tensor-map encoder is fetched at
run time through ``cudaGetDriverEntryPoint``), so it loads on a machine
without a GPU and can be built there (nvcc cross-compiles for sm_100a).
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libpa_b200.so"

SOURCES = ["pa_capi.cu", "pa_kv_append.cu", "pa_decode_mma.cu", "pa_decode_f32.cu", "pa_static_ws.cu",
           "pa_prefill_mma.cu", "pa_prefill_umma.cu", "pa_prefill_umma2.cu"]
HEADERS = ["pa_common.cuh", "pa_internal.h", "pa_tile_math.cuh"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS]
    files.append(REPO_DIR / "include" / "paged_attention_b200.h")
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    lib_mtime = LIB_PATH.stat().st_mtime
    return any(f.stat().st_mtime > lib_mtime for f in _inputs())


def build_library(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile every CUDA source into ``lib/libpa_b200.so`` (skipped when up to date)."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        _nvcc(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "--expt-relaxed-constexpr",
        "-shared",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-Xcompiler",
        "-Wall",
        f"-I{REPO_DIR / 'include'}",
        *(extra_flags or []),
        *[str(CSRC / s) for s in SOURCES],
        "-o",
        str(tmp),
        "-lcudart",
    ]
    if verbose:
        print(" ".join(cmd))
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{proc.stdout}\n{proc.stderr}")
    if verbose and (proc.stdout or proc.stderr):
        print(proc.stdout, proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    path = build_library(force="--force" in sys.argv, verbose=True,
                         extra_flags=["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None)
    print(path)
