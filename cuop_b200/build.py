"""Ahead-of-time build of libcuopx.so (sm_100a) in-tree.

`python -m cuop_b200.build` compiles every CUDA/C++ source of the library with
nvcc for `-gencode arch=compute_100a,code=sm_100a` into
cuop_b200/libcuopx.so, and writes the ptxas register/spill report to
cuop_b200/_build/ptxas.log.  No JIT, no torch extension cache: the .so lives
next to this file so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from typing import Optional
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libcuopx.so"
BUILD_DIR = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", f"-I{ROOT / 'include'}",
          f"-I{ROOT / 'include' / 'cuop'}", f"-I{CSRC}"]

# Device code is one translation unit (see csrc/cuopx_unity.cu); the C++17
# operator/plugin facade is plain host code compiled by nvcc's host compiler.
CUDA_SOURCES = ["cuopx_unity.cu"]
HOST_SOURCES = sorted(p.name for p in (CSRC / "host").glob("*.cpp")) if (CSRC / "host").exists() else []


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: cannot build libcuopx.so")


def _sources() -> list[Path]:
    out = [CSRC / s for s in CUDA_SOURCES]
    out += [CSRC / "host" / s for s in HOST_SOURCES]
    return out


def _deps() -> list[Path]:
    deps = list(CSRC.rglob("*.cu")) + list(CSRC.rglob("*.cuh")) + list(CSRC.rglob("*.h"))
    deps += list((CSRC / "host").glob("*.cpp")) + list((ROOT / "include").rglob("*.h*"))
    return deps


def needs_rebuild() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


CORE_SRC = CSRC / "python" / "core.cpp"


def core_module_path() -> Path:
    import sysconfig

    return PKG / ("core" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build_core_module(force: bool = False, verbose: bool = False) -> Optional[Path]:
    """pybind11 module `cuop_b200.core` (the reference's Python operator
    classes over the C++ facade), linked against libcuopx.so; None when
    pybind11 is not importable."""
    import sysconfig

    try:
        import pybind11
    except ImportError:
        return None
    out = core_module_path()
    deps = [CORE_SRC, LIB] + list((ROOT / "include").rglob("*.h*"))
    if not force and out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    cmd = [_nvcc(), "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", f"-I{pybind11.get_include()}",
           f"-I{sysconfig.get_paths()['include']}", f"-I{ROOT / 'include'}", f"-I{ROOT / 'include' / 'cuop'}",
           str(CORE_SRC), "-o", str(out), f"-L{PKG}", "-lcuopx", "-Xlinker", "-rpath=$ORIGIN"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building {out.name} failed:\n{r.stderr[-4000:]}")
    return out


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_rebuild():
        build_core_module(verbose=verbose)
        return LIB
    BUILD_DIR.mkdir(exist_ok=True)
    nvcc = _nvcc()
    objs = []
    log = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        if src.suffix == ".cpp":  # host-only C++: nvcc hands it to the host compiler
            cmd = [nvcc, *COMMON, "-c", str(src), "-o", str(obj)]
        else:
            cmd = [nvcc, *ARCH, *COMMON, "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        r = subprocess.run(cmd, capture_output=True, text=True)
        log.append(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
        if r.returncode != 0:
            (BUILD_DIR / "ptxas.log").write_text("\n".join(log))
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr[-4000:]}")
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log.append(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
    (BUILD_DIR / "ptxas.log").write_text("\n".join(log))
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, LIB)
    build_core_module(force=True, verbose=verbose)
    return LIB


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
