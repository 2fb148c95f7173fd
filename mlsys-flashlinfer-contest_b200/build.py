"""Build the gdn_b200 CUDA library (libgdn_b200.so) for sm_100a, in-tree.

    python mlsys-flashlinfer-contest_b200/build.py [--force] [-j N]

Each csrc/*.cu compiles to _build/<name>.o with
``nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo``, and the objects
link into gdn_b200/libgdn_b200.so (static CUDA runtime, no other dependency).
A source is recompiled when it or any csrc header is newer than its object.
nvcc cross-compiles, so no GPU is needed to build.

csrc/gdn_torch.cpp, the torch-tensor binding of that C ABI, compiles with g++
against the installed torch headers into gdn_b200/_gdn_torch.so (linked to
libgdn_b200.so through an $ORIGIN rpath).

csrc/gdn_tvm_ffi.cc, the TVM-FFI module (the binding the reference's Solutions
load with tvm_ffi.load_module), compiles with g++ against the installed tvm_ffi
headers into gdn_b200/gdn_tvm_ffi.so, linked to libgdn_b200.so and libtvm_ffi.so.
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
BUILD = HERE / "_build"
LIB = HERE / "gdn_b200" / "libgdn_b200.so"
TORCH_EXT = HERE / "gdn_b200" / "_gdn_torch.so"
TVM_FFI_MOD = HERE / "gdn_b200" / "gdn_tvm_ffi.so"
REPO = HERE.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                     "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(REPO / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _compile(src: Path, extra, verbose: bool):
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and verbose:
        print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose: bool = False, extra=()) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((REPO / "include").glob("*.h"))
    newest_hdr = max((h.stat().st_mtime for h in headers), default=0.0)
    todo = []
    for s in sources:
        obj = BUILD / (s.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, newest_hdr):
            todo.append(s)
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(lambda s: _compile(s, list(extra), verbose), todo))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if todo or force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    build_torch_ext(force=force, verbose=verbose)
    build_tvm_ffi(force=force, verbose=verbose)
    return LIB


def build_torch_ext(force: bool = False, verbose: bool = False) -> Path:
    """g++ build of the torch-tensor binding (a CPython extension module)."""
    src = CSRC / "gdn_torch.cpp"
    deps = [src, REPO / "include" / "gdn_b200.h", LIB]
    if not force and TORCH_EXT.exists() and TORCH_EXT.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return TORCH_EXT
    import sysconfig
    import torch
    from torch.utils import cpp_extension as ce
    torch_lib = Path(torch.__file__).resolve().parent / "lib"
    cuda_inc = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "include"
    incs = [p for p in ce.include_paths("cpu")] + [str(cuda_inc), sysconfig.get_paths()["include"],
                                                  str(REPO / "include")]
    tmp = TORCH_EXT.with_suffix(".so.tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           "-DTORCH_EXTENSION_NAME=_gdn_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{p}" for p in incs], str(src), "-o", str(tmp),
           f"-L{torch_lib}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           f"-L{LIB.parent}", "-lgdn_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch binding build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TORCH_EXT)
    return TORCH_EXT


def build_tvm_ffi(force: bool = False, verbose: bool = False) -> Path:
    """g++ build of the TVM-FFI module (host code only: every export forwards to
    the C ABI of libgdn_b200.so)."""
    src = CSRC / "gdn_tvm_ffi.cc"
    deps = [src, REPO / "include" / "gdn_b200.h", LIB]
    if not force and TVM_FFI_MOD.exists() and TVM_FFI_MOD.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return TVM_FFI_MOD
    import tvm_ffi.libinfo as tl
    ffi_lib = Path(tl.find_libtvm_ffi()).resolve()
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    incs = [tl.find_include_path(), tl.find_dlpack_include_path(), str(cuda / "include"),
            str(REPO / "include")]
    tmp = TVM_FFI_MOD.with_suffix(".so.tmp")
    cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-fPIC", "-shared",
           *[f"-I{p}" for p in incs], str(src), "-o", str(tmp),
           f"-L{ffi_lib.parent}", "-ltvm_ffi", f"-L{cuda / 'lib64'}", "-lcudart",
           f"-L{LIB.parent}", "-lgdn_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{ffi_lib.parent}",
           f"-Wl,-rpath,{cuda / 'lib64'}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"TVM-FFI module build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, TVM_FFI_MOD)
    return TVM_FFI_MOD


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, jobs=a.j, verbose=a.v or a.ptxas_v, extra=extra))
