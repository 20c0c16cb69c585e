"""Build libb200exec.so in-tree with nvcc for sm_100a.

    python lets-build-a-runtime_b200/build.py        # or build() from Python

Every ``csrc/*.cu`` is compiled to an object (in parallel, skipped when up
to date) and linked into ``lib/libb200exec.so`` next to this file.  nvcc
cross-compiles without a GPU, so this runs on CPU-only machines too.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libb200exec.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-I", str(REPO / "include"), "-I", str(CSRC)]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.h")) + list((REPO / "include").glob("*.h"))
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    nvcc = _nvcc()
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    flags = NVCC_FLAGS + (extra_flags or [])

    def compile_one(src: Path) -> Path:
        obj = OBJ / (src.stem + ".o")
        if _stale(src, obj):
            cmd = [nvcc, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
            if verbose and r.stderr:
                print(r.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static",
               "-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    import sys
    print(build(verbose="-v" in sys.argv))
