"""Build recipe of the native library (sm_100a only).

    python -m leanstream_b200.build        # -> leanstream_b200/libleanstream_b200.so

The shared object is built in-tree so that it travels with the repository
snapshot; nothing is JIT-compiled at import time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libleanstream_b200.so"
SOURCES = ("ls_kernel.cu", "ls_kernel_traced.cu", "ls_backend.cu", "ls_aux.cu", "ls_stream.cu", "ls_batch.cu")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def needs_build(target: Path = LIBRARY) -> bool:
    if not target.exists():
        return True
    stamp = target.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + [CSRC / "ls_internal.h", ROOT / "include" / "leanstream_b200.h"]
    return any(p.stat().st_mtime > stamp for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIBRARY
    cmd = [
        nvcc(), *ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v",
        "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
        "-I", str(ROOT / "include"),
        *[str(CSRC / s) for s in SOURCES],
        "-o", str(LIBRARY) + ".tmp",
    ]
    proc = subprocess.run(cmd, cwd=str(PACKAGE), capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + proc.stdout + proc.stderr)
    if verbose:
        sys.stdout.write(proc.stderr)
    os.replace(str(LIBRARY) + ".tmp", LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
