"""Build ``libgdn_b200.so`` (all CUDA sources of ``csrc/``) for sm_100a with nvcc.

The library is written next to this file so it travels with the source tree;
intermediate objects go to ``_build/``.  Sources are compiled in parallel with
relocatable device code and device-linked into one shared object that exports
only the C ABI of ``include/gdn_b200.h``.  When ``tvm_ffi`` is installed, the
TVM-FFI module ``libgdn_b200_tvm_ffi.so`` (``csrc/gdn_tvm_ffi.cc``, host C++
over that C ABI) is built next to it.

    python build.py [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD_DIR = HERE / "_build"
LIB_NAME = "libgdn_b200.so"
LIB_PATH = HERE / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps_mtime() -> float:
    files = [f for f in CSRC.glob("*") if f.suffix != ".cc"] + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files if f.is_file())


def is_stale() -> bool:
    return not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < _deps_mtime()


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose or res.stderr.strip():
        sys.stderr.write(res.stderr)
    return obj


TVM_SRC = CSRC / "gdn_tvm_ffi.cc"
TVM_LIB_PATH = HERE / "libgdn_b200_tvm_ffi.so"


def tvm_ffi_paths():
    """(include dirs, lib dir) of the installed tvm_ffi package, or None if it is absent."""
    try:
        import tvm_ffi.libinfo as info
    except ImportError:
        return None
    lib = Path(info.find_libtvm_ffi()).parent
    return [str(p) for p in info.include_paths()], str(lib)


def build_tvm_ffi(force: bool = False) -> Path | None:
    """The TVM-FFI module (host C++ over the C ABI), when tvm_ffi is installed."""
    paths = tvm_ffi_paths()
    if paths is None:
        return None
    if not force and TVM_LIB_PATH.exists() and TVM_LIB_PATH.stat().st_mtime >= max(
            TVM_SRC.stat().st_mtime, LIB_PATH.stat().st_mtime, (INCLUDE / "gdn_b200.h").stat().st_mtime):
        return TVM_LIB_PATH
    incs, libdir = paths
    cuda = Path(nvcc()).resolve().parent.parent
    tmp = TVM_LIB_PATH.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", *[f"-I{i}" for i in incs], f"-I{cuda / 'include'}",
           str(TVM_SRC), "-o", str(tmp), f"-L{HERE}", "-lgdn_b200", "-Wl,-rpath,$ORIGIN",
           f"-L{libdir}", "-ltvm_ffi", f"-Wl,-rpath,{libdir}", f"-L{cuda / 'lib64'}", "-lcudart",
           f"-Wl,-rpath,{cuda / 'lib64'}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"TVM-FFI module build failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, TVM_LIB_PATH)
    return TVM_LIB_PATH


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library if any source is newer than it, then the TVM-FFI module."""
    _build_lib(force, verbose)
    build_tvm_ffi(force)
    return LIB_PATH


def _build_lib(force: bool, verbose: bool) -> Path:
    if not force and not is_stale():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objs),
           "-o", str(tmp), "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))
