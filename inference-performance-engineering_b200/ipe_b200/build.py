"""Build the sm_100a shared library `ipe_b200/lib/libipe_b200.so` in-tree with nvcc.

    python -m ipe_b200.build            # from inference-performance-engineering_b200/

Each `csrc/*.cu` compiles to an object for `-gencode arch=compute_100a,code=sm_100a` (the only
target: tcgen05 and TMA need the `a` variant), then one `-shared` link with the CUDA runtime linked
statically. Nothing else is built; no JIT cache is used.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent  # inference-performance-engineering_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB_DIR = PACKAGE / "lib"
LIBRARY = LIB_DIR / "libipe_b200.so"
BUILD_DIR = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build ipe_b200")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    return not target.exists() or any(d.stat().st_mtime > target.stat().st_mtime for d in deps)


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    flags = FLAGS + list(extra_flags or [])
    compiler = nvcc()

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        if _stale(obj, [src, *headers]):
            cmd = [compiler, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            result = subprocess.run(cmd, capture_output=True, text=True)
            if result.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{result.stderr}")
            if verbose and result.stderr:
                print(result.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, sources()))
    if _stale(LIBRARY, objects):
        cmd = [compiler, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stderr}")
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, extra_flags=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None))
