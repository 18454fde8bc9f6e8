"""Builds libb200kv.so (the C-ABI CUDA library) in-tree for sm_100a.

Usage: ``python -m torch_spyre_b200.build [--verbose]``.  The shared library is
written next to this file (``torch_spyre_b200/lib/libb200kv.so``) so it travels
with the source tree; nothing is installed.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libb200kv.so"
INCLUDE = PKG_DIR.parent / "include"

SOURCES = [
    "capi.cu",
    "kv_relayout.cu",
    "decode_attention.cu",
    "decode_mma.cu",
    "decode_simt.cu",
    "decode_noalloc.cu",
    "stick_relayout.cu",
    "fp8_ops.cu",
    "peer_allreduce.cu",
    "nvls_allreduce.cu",
    "rope.cu",
    "lse_combine.cu",
    "oproj_allreduce.cu",
]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libb200kv")
    return cand


def _needs_rebuild() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return any(p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every CUDA source of the library into one shared object."""
    if not force and not _needs_rebuild():
        return LIB_PATH
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [
        nvcc_path(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "--expt-relaxed-constexpr",
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-shared",
        f"-I{INCLUDE}",
        "-o",
        str(tmp),
        *[str(CSRC / s) for s in SOURCES],
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed ({proc.returncode}):\n{' '.join(cmd)}\n{proc.stderr}")
    if verbose:
        sys.stderr.write(proc.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="--verbose" in sys.argv)
    print(LIB_PATH)
