"""Build libcc1d.so, the sm_100a kernel library behind causal_conv1d_cute, in place.

Usage: python build.py [--force] [--jobs N] [--verbose-ptxas]

Every csrc/*.cu file is compiled to an object under _build/ (in parallel, only when the source or
a header is newer than the object) and linked with the static CUDA runtime into
causal_conv1d_cute/libcc1d.so, next to the Python package that loads it. nvcc cross-compiles for
sm_100a, so the build runs on a machine without a GPU.
"""

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OBJ = HERE / "_build"
LIB = HERE / "causal_conv1d_cute" / "libcc1d.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}"]


def _nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def _stale(obj, deps):
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force=False, jobs=None, ptxas_verbose=False):
    """Compile the kernels and link libcc1d.so; return its path."""
    OBJ.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    nvcc = _nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []

    def compile_one(src):
        obj = OBJ / (src.stem + ".o")
        if not force and not _stale(obj, [src, *headers]):
            return obj, None
        cmd = [nvcc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        return obj, r.stderr if ptxas_verbose else None

    with ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as pool:
        results = list(pool.map(compile_one, sources))
    for _, log in results:
        if log:
            sys.stderr.write(log)
    objs = [o for o, _ in results]
    if force or _stale(LIB, objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main():
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--force", action="store_true")
    p.add_argument("--jobs", type=int, default=None)
    p.add_argument("--verbose-ptxas", action="store_true")
    args = p.parse_args()
    print(build(args.force, args.jobs, args.verbose_ptxas))


if __name__ == "__main__":
    main()
