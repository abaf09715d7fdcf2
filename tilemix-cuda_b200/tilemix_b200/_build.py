"""In-tree build of libtilemix_b200.so (sm_100a only) and the demo driver.

The shared library is written next to this file so it travels with the source
tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
PROJECT = PKG.parent                     # tilemix-cuda_b200/
REPO = PROJECT.parent
CSRC = PROJECT / "csrc"
INCLUDE = REPO / "include"
LIB = PKG / "libtilemix_b200.so"
DEMO = PROJECT / "src" / "main.cu"
DEMO_BIN = PKG / "tilemix_demo"

SOURCES = ["quantize.cu", "attention.cu", "api.cu", "noalloc.cu", "policy.cu", "backward.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/*.cu into libtilemix_b200.so (skipped when up to date)."""
    inputs = [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    if force or _stale(LIB, inputs):
        objdir = PROJECT / "_build"
        objdir.mkdir(exist_ok=True)
        objs = []
        for src in SOURCES:
            obj = objdir / (Path(src).stem + ".o")
            cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                   f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(CSRC / src), "-o", str(obj)]
            _run(cmd, verbose)
            objs.append(str(obj))
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs], verbose)
        tmp.replace(LIB)
    if force or _stale(DEMO_BIN, [DEMO, LIB]):
        _run([nvcc(), *ARCH, "-O2", "-std=c++17", f"-I{INCLUDE}", str(DEMO), "-o", str(DEMO_BIN),
              f"-L{PKG}", "-ltilemix_b200", f"-Xlinker=-rpath,{PKG}"], verbose)
    return LIB


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed ({res.returncode}): {' '.join(cmd)}\n{res.stdout}")


if __name__ == "__main__":
    import sys
    print(build(force="--force" in sys.argv, verbose=True))
