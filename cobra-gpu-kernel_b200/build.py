"""Build recipe for the sm_100a shared library (``_lib/libcobra_b200.so``).

One translation unit (``csrc/capi.cu``) holds the C ABI and every kernel. It is
compiled with nvcc for ``sm_100a`` only (tcgen05 / TMA are sm_100a features),
position-independent, with the CUDA runtime linked statically so the library
loads through ctypes without a toolkit on the library path.

A content hash of the sources and flags is stored next to the library; the
loader rebuilds when the hash differs and nvcc is available, and refuses to
run otherwise.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libcobra_b200.so"
STAMP = OUT_DIR / "build.sha"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-Xcompiler", "-fvisibility=hidden",
]


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def source_hash() -> str:
    h = hashlib.sha256()
    for p in _sources():
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def nvcc_path() -> str | None:
    cand = os.environ.get("NVCC") or shutil.which("nvcc")
    if cand:
        return cand
    p = Path("/usr/local/cuda/bin/nvcc")
    return str(p) if p.exists() else None


def is_current() -> bool:
    return LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or stale; returns its path."""
    if not force and is_current():
        return LIB
    nvcc = nvcc_path()
    if nvcc is None:
        raise RuntimeError("nvcc not found: cannot build the sm_100a library " f"({LIB})")
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc, *NVCC_FLAGS, "-o", str(tmp), str(CSRC / "capi.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose:
        print(res.stderr)
    os.replace(tmp, LIB)
    STAMP.write_text(source_hash() + "\n")
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
