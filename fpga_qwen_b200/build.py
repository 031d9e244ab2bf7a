"""Build recipe for libqattn.so (in-tree, sm_100a only).

    python -m fpga_qwen_b200.build          # or: import fpga_qwen_b200.build; build()

Compiles every ``csrc/*.cu`` with nvcc for ``compute_100a``/``sm_100a`` and links one
shared library next to this file. The CUDA runtime is linked statically; the driver API
is reached through ``cudaGetDriverEntryPoint`` at run time, so the library needs only
``libcuda.so`` from the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libqattn.so"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + sorted(CSRC.glob("*.cuh")) + sorted((PKG.parent / "include").glob("*.h"))
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    objs = []

    def compile_one(src: Path):
        obj = BUILD / (src.stem + ".o")
        if _stale(obj, src):
            cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            res = subprocess.run(cmd, capture_output=True, text=True)
            log = BUILD / (src.stem + ".ptxas.txt")
            log.write_text(res.stdout + res.stderr)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr[-4000:]}")
            if verbose:
                print(res.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-Xcompiler", "-fPIC",
               "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
