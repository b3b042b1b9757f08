"""In-tree build of the CUDA extension ``_nnb.so`` for sm_100a.

``nvcc -gencode arch=compute_100a,code=sm_100a`` over ``csrc/*.cu``; the
library is written next to this file so that it travels with the source tree.
"""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
SOURCES = ("capi.cu", "simt_ops.cu", "window.cu", "tc_conv.cu", "noalloc.cu", "restore.cu", "preprocess.cu")
OUTPUT = PACKAGE / "_nnb.so"
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(home) / "bin" / "nvcc"
    return str(candidate) if candidate.exists() else "nvcc"


def build_extension(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``_nnb.so`` if it is missing or older than a source; return its path."""
    sources = [PACKAGE / "csrc" / name for name in SOURCES]
    deps = sources + list((PACKAGE / "csrc").glob("*.cuh")) + [PACKAGE.parent / "include" / "nnb.h"]
    if not force and OUTPUT.exists():
        newest = max(p.stat().st_mtime for p in deps if p.exists())
        if OUTPUT.stat().st_mtime >= newest:
            return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc(), *FLAGS, "-o", str(tmp), *map(str, sources)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr[-4000:]}")
    if verbose and result.stderr:
        print(result.stderr)
    tmp.replace(OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    print(build_extension(force=True, verbose=True))
