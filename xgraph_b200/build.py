"""Build libxgraph_b200.so in-tree with nvcc for sm_100a (B200).

    python -m xgraph_b200.build [--verbose]

The library holds every kernel and the C ABI (include/xgraph_b200.h); it links only the
CUDA runtime.  It is written next to this file so that it travels with the source tree.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
SOURCES = [HERE / "csrc" / "engine.cu", HERE / "csrc" / "build.cu"]
DEPENDS = SOURCES + [HERE / "csrc" / "core.cuh", HERE / "csrc" / "layout.h", ROOT / "include" / "xgraph_b200.h"]
OUTPUT = HERE / "libxgraph_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build the engine")
    return found


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and OUTPUT.exists() and OUTPUT.stat().st_mtime >= max(p.stat().st_mtime for p in DEPENDS):
        return OUTPUT
    command = [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-Xcompiler", "-fvisibility=hidden", "-I", str(ROOT / "include"),
        "-o", str(OUTPUT.with_suffix(".tmp.so")), *map(str, SOURCES),
    ]
    if verbose:
        command.insert(1, "-Xptxas=-v")
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{result.stderr}")
    if verbose:
        sys.stderr.write(result.stderr)
    os.replace(OUTPUT.with_suffix(".tmp.so"), OUTPUT)
    return OUTPUT


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force or args.verbose, verbose=args.verbose))


if __name__ == "__main__":
    main()
