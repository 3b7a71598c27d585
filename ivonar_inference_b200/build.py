"""Build recipe for libivonar_b200.so (nvcc, sm_100a only).

The library is built in-tree (``ivonar_inference_b200/libivonar_b200.so``) so it travels with the
source tree; nothing is JIT-compiled at run time.
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
INCLUDE = ROOT / "include"
LIBRARY = PACKAGE / "libivonar_b200.so"

SOURCES = ("ivb_unit.cu", "ivb_decoder.cu", "ivb_splitk.cu", "ivb_gemm.cu", "ivb_prefill.cu", "ivb_batch.cu")
ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-cudart",
    "shared",
    "--expt-relaxed-constexpr",
)


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    candidate = Path("/usr/local/cuda/bin/nvcc")
    if candidate.exists():
        return str(candidate)
    raise RuntimeError("nvcc was not found; the sm_100a library cannot be built")


def _inputs() -> list[Path]:
    return [CSRC / name for name in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "ivonar_b200.h"]


def up_to_date() -> bool:
    if not LIBRARY.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in _inputs())


def build(force: bool = False, verbose: bool = False, extra: tuple[str, ...] = ()) -> Path:
    """Compile every .cu source into one shared library for sm_100a; returns its path."""

    if not force and up_to_date():
        return LIBRARY
    objects = []
    build_dir = PACKAGE / "_build"
    build_dir.mkdir(exist_ok=True)
    compiler = nvcc()
    for name in SOURCES:
        obj = build_dir / (Path(name).stem + ".o")
        cmd = [compiler, *ARCH_FLAGS, *NVCC_FLAGS, *extra, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(CSRC / name), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    temporary = LIBRARY.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [compiler, *ARCH_FLAGS, "-shared", "-cudart", "shared", *objects, "-o", str(temporary)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    temporary.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, extra=tuple(a for a in sys.argv[1:] if a.startswith("-X")))
    print(LIBRARY)
