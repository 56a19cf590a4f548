"""Build libintp_b200.so (sm_100a) in-tree with nvcc.

The library is compiled straight from ``csrc/*.cu`` with
``-gencode arch=compute_100a,code=sm_100a`` and linked as a plain shared
object; Python reaches it through ctypes (``intp_preliminary_b200._lib``).
The output lives next to the sources so it travels with the repository
snapshot to the GPU host.

Usage: ``python -m intp_preliminary_b200.build [--force] [--verbose]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = PACKAGE_DIR.parent / "include"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_PATH = LIB_DIR / "libintp_b200.so"
SOURCES = ("capi.cu", "look_attention_simt.cu", "look_attention_tc.cu", "look_attention_short.cu", "negative_l1.cu",
           "noalloc.cu", "share_vit_ops.cu", "backward.cu", "backward_tc.cu", "backward_fused.cu", "gemm_epilogue.cu", "dense_look_grid.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _inputs() -> list[Path]:
    files = [CSRC / name for name in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    return files


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(path.stat().st_mtime > built for path in _inputs())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the library if it is missing or older than its sources."""
    if not force and not is_stale():
        return LIB_PATH
    LIB_DIR.mkdir(exist_ok=True)
    objects = []
    nvcc = _nvcc()
    common = [
        nvcc, "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS,
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "-I", str(INCLUDE), "-I", str(CSRC),
    ]
    if verbose:
        common += ["-Xptxas", "-v"]
    for name in SOURCES:
        obj = LIB_DIR / (Path(name).stem + ".o")
        cmd = [*common, "-c", str(CSRC / name), "-o", str(obj)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or result.returncode != 0:
            sys.stderr.write(result.stdout + result.stderr)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed on {name}")
        objects.append(str(obj))
    tmp = LIB_DIR / "libintp_b200.so.tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objects, "-lcudart"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB_PATH)
    for obj in objects:
        Path(obj).unlink(missing_ok=True)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
