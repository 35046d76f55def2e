"""Builds libffb200.so in-tree (fastforward_b200/libffb200.so) with nvcc for sm_100a.

Each `csrc/*.cu` compiles to a relocatable object under `fastforward_b200/_build/`
(rebuilt only when it or a header is newer than its object), then one nvcc call device-
links them into the shared library.  Run `python -m fastforward_b200.build [--force]`.
"""
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libffb200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc():
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libffb200.so")
    return cand


def _headers():
    return list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale(src, obj, newest_header):
    return (not obj.exists()) or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)


def build(force=False, verbose=False, jobs=None):
    OBJ.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0)
    cc = nvcc()
    todo = [s for s in sources if force or _stale(s, OBJ / (s.stem + ".o"), newest_header)]

    def compile_one(src):
        obj = OBJ / (src.stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        return src.name, r.stderr

    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        for name, err in ex.map(compile_one, todo):
            if verbose and err:
                print(f"== {name}\n{err}", file=sys.stderr)
    objs = [OBJ / (s.stem + ".o") for s in sources]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [cc, *ARCH, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(LIB),
               "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
