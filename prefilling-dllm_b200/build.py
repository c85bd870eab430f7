"""Build step: compile the sm_100a kernels and their C-ABI into libpdllm_b200.so next to this file.

`nvcc` cross-compiles without a GPU, so this runs on a CPU-only machine. The result is loaded by
`_lib.py` through ctypes; nothing in the package JIT-compiles at import time.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from typing import List, Optional

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
CSRC_DIR = os.path.join(PKG_DIR, "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(PKG_DIR), "include")
LIB_NAME = "libpdllm_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
STAMP_PATH = os.path.join(PKG_DIR, ".libpdllm_b200.srchash")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--shared", "-Xcompiler", "-fPIC",
    "-Xptxas", "-v",
]


def _sources() -> List[str]:
    files = [os.path.join(CSRC_DIR, name) for name in sorted(os.listdir(CSRC_DIR)) if name.endswith((".cu", ".cuh"))]
    files.append(os.path.join(INCLUDE_DIR, "pdllm_b200.h"))
    return files


def source_hash() -> str:
    digest = hashlib.sha256()
    for path in _sources():
        with open(path, "rb") as handle:
            digest.update(os.path.basename(path).encode())
            digest.update(handle.read())
    digest.update(" ".join(NVCC_FLAGS).encode())
    return digest.hexdigest()


def find_nvcc() -> Optional[str]:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and os.path.exists(candidate):
            return candidate
    return None


def is_current() -> bool:
    if not (os.path.exists(LIB_PATH) and os.path.exists(STAMP_PATH)):
        return False
    with open(STAMP_PATH) as handle:
        return handle.read().strip() == source_hash()


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile if the sources changed since the last build; return the library path."""
    if not force and is_current():
        return LIB_PATH
    nvcc = find_nvcc()
    if nvcc is None:
        raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit to build libpdllm_b200.so")
    tmp_out = LIB_PATH + ".tmp"
    cmd = [nvcc, *NVCC_FLAGS, "-I", INCLUDE_DIR, "-o", tmp_out, os.path.join(CSRC_DIR, "pdllm_abi.cu")]
    proc = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if verbose or proc.returncode != 0:
        sys.stderr.write(proc.stdout)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed with exit code {proc.returncode}: {' '.join(cmd)}")
    with open(os.path.join(PKG_DIR, "ptxas_info.log"), "w") as handle:
        handle.write(proc.stdout)
    os.replace(tmp_out, LIB_PATH)
    with open(STAMP_PATH, "w") as handle:
        handle.write(source_hash())
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
