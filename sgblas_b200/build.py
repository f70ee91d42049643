"""Builds libsgblas.so (the product) in-tree with nvcc for sm_100a.

    python sgblas_b200/build.py [-v]     (a script: it must not import the package,
                                          whose import loads the library it builds)

Every translation unit under sgblas_b200/csrc is compiled for
``-gencode arch=compute_100a,code=sm_100a`` with ``-lineinfo`` and linked into
``sgblas_b200/lib/libsgblas.so`` together with a static CUDA runtime, so the
library does not depend on whichever libcudart another package (torch) loaded.
Objects are rebuilt only when a source or header is newer than the object.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OBJ = PKG / "_build"
LIB = PKG / "lib" / "libsgblas.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libsgblas.so")


def _sources() -> list[pathlib.Path]:
    return sorted(p for p in CSRC.iterdir() if p.suffix in (".cu", ".cpp"))


def _headers() -> list[pathlib.Path]:
    hs = [p for p in CSRC.iterdir() if p.suffix in (".cuh", ".hpp", ".h")]
    hs += list((INCLUDE / "sgblas").glob("*.h"))
    return hs


def _compile(src: pathlib.Path, verbose: bool) -> pathlib.Path:
    obj = OBJ / (src.name + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [_nvcc(), *COMMON, *ARCH, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"] if verbose else []
    else:
        cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}", f"-I{CSRC}",
               "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose: bool = False) -> pathlib.Path:
    OBJ.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    link_deps = [o.stat().st_mtime for o in objs] + [(CSRC / "exports.map").stat().st_mtime,
                                                      pathlib.Path(__file__).stat().st_mtime]
    if LIB.exists() and LIB.stat().st_mtime >= max(link_deps):
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    # Only the C API is exported (csrc/exports.map).
    cmd = [_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
           *map(str, objs), "-ldl", "-lpthread", "-lrt",
           "-Xlinker", f"--version-script={CSRC / 'exports.map'}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"linking libsgblas.so failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
