"""Build recipe of libekv_b200.so: every .cu under csrc/ in one nvcc call, for sm_100a only.

The library links the shared CUDA runtime, so it shares torch's current device, streams and
context in the serving process. It is built in-tree, next to ``ekv/_lib.py``, which loads it.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PACKAGE_DIR = os.path.dirname(os.path.abspath(__file__))
SOURCE_DIR = os.path.join(os.path.dirname(PACKAGE_DIR), "csrc")
INCLUDE_DIR = os.path.join(os.path.dirname(os.path.dirname(PACKAGE_DIR)), "include")
OUTPUT = os.path.join(PACKAGE_DIR, "libekv_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(found):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libekv_b200.so")
    return found


def command(output: str = OUTPUT, extra: list[str] | None = None) -> list[str]:
    sources = sorted(glob.glob(os.path.join(SOURCE_DIR, "*.cu")))
    return [
        nvcc(),
        *ARCH_FLAGS,
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-shared",
        "-cudart",
        "shared",
        f"-I{INCLUDE_DIR}",
        *(extra or []),
        "-o",
        output,
        *sources,
    ]


def stale(output: str = OUTPUT) -> bool:
    """True when the library is missing or older than a source or the header."""
    if not os.path.exists(output):
        return True
    built = os.path.getmtime(output)
    inputs = glob.glob(os.path.join(SOURCE_DIR, "*")) + glob.glob(os.path.join(INCLUDE_DIR, "*.h"))
    return any(os.path.getmtime(path) > built for path in inputs)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if a source changed (or ``force``); return its path."""
    if not force and not stale():
        return OUTPUT
    cmd = command()
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stderr[-4000:]}")
    return OUTPUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
