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


def _flags():
    return [*ARCH, "-O3", "-std=c++17", "-lineinfo", "-Xptxas", "-v", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
            "-I", str(ROOT / "include")]


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every source to an object under _build/ (in parallel; an
    object is rebuilt when its source or a shared header is newer), then
    links the shared library."""
    if not force and not needs_build():
        return LIBRARY
    from concurrent.futures import ThreadPoolExecutor

    objdir = PACKAGE / "_build"
    objdir.mkdir(exist_ok=True)
    headers = [CSRC / "ls_internal.h", ROOT / "include" / "leanstream_b200.h", CSRC / "ls_kernel.cu"]
    newest_header = max(h.stat().st_mtime for h in headers)

    def compile_one(src: str):
        obj = objdir / (Path(src).stem + ".o")
        srcp = CSRC / src
        if not force and obj.exists() and obj.stat().st_mtime > max(srcp.stat().st_mtime, newest_header):
            return obj, ""
        proc = subprocess.run([nvcc(), *_flags(), "-c", str(srcp), "-o", str(obj) + ".tmp"], cwd=str(PACKAGE),
                              capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n" + proc.stdout + proc.stderr)
        os.replace(str(obj) + ".tmp", obj)
        return obj, proc.stderr

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as pool:
        results = list(pool.map(compile_one, SOURCES))
    cmd = [nvcc(), *ARCH, "-shared", *[str(o) for o, _ in results], "-o", str(LIBRARY) + ".tmp"]
    proc = subprocess.run(cmd, cwd=str(PACKAGE), capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("nvcc link failed:\n" + proc.stdout + proc.stderr)
    if verbose:
        for _, log in results:
            sys.stdout.write(log)
    os.replace(str(LIBRARY) + ".tmp", LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose=True)
    print(path)
