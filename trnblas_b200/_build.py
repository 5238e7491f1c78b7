"""Build the sm_100a shared library `trnblas_b200/_lib/libtrnblas_b200.so`.

One nvcc invocation per translation unit, then one link; all code is compiled
for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`). The library has
no torch dependency: it exports the C ABI declared in include/trnblas_b200.h.
Run `python -m trnblas_b200._build` (or `__graft_entry__.build()`).
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
LIBDIR = PKG / "_lib"
LIBNAME = "libtrnblas_b200.so"
ROOT = PKG.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{ROOT / 'include'}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.hpp"), ROOT / "include" / "trnblas_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps if d.exists())


def build(verbose: bool = False, ptxas_info: bool = False, force: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link the shared library."""
    out = LIBDIR / LIBNAME
    objdir = LIBDIR / "obj"
    objdir.mkdir(parents=True, exist_ok=True)
    cc = nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []

    def compile_one(src: Path) -> Path:
        obj = objdir / (src.stem + ".o")
        if force or ptxas_info or _stale(obj, src):
            cmd = [cc, *ARCH, *NVFLAGS, *extra, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
            if ptxas_info or verbose:
                sys.stdout.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(compile_one, sources()))
    if force or not out.exists() or any(o.stat().st_mtime > out.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-o", str(out), *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv, force="-f" in sys.argv))
