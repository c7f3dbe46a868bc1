"""Builds libveda_cuda.so (the sm_100a kernels behind include/veda_cuda.h) and libveda.so (the
C++23 host library: veda::core / autograd / optim / train over the kernels) in-tree.

    python -m veda_b200.build            # both libraries, incremental
    python -m veda_b200.build --force    # rebuild everything

Every .cu file is compiled with `-gencode arch=compute_100a,code=sm_100a -lineinfo -O3` (sm_100a
only: no PTX for other targets, no multi-arch fat binary). Outputs land next to this file, so
they travel with the repository snapshot to a GPU box.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = CSRC / "host"
OBJ = PKG / "_build"
INCLUDE = ROOT / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_LIB = "libveda_cuda.so"
HOST_LIB = "libveda.so"


def _nccl_paths():
    """Include and library dirs for NCCL: the copy bundled with torch if present (the one the
    Python process loads), else the system one."""
    try:
        import nvidia.nccl  # type: ignore
        base = Path(list(nvidia.nccl.__path__)[0])
        if (base / "include" / "nccl.h").exists():
            return base / "include", base / "lib"
    except Exception:
        pass
    return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _headers(folder: Path):
    return list(folder.glob("*.cuh")) + list(folder.glob("*.hpp")) + list(INCLUDE.rglob("*.h")) + \
        list(INCLUDE.rglob("*.hpp"))


def build_cuda(force=False, verbose=False, jobs=None) -> Path:
    OBJ.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers(CSRC)
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                    "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC)]
    if verbose:
        flags += ["-Xptxas", "-v"]

    def compile_one(src: Path):
        obj = OBJ / (src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            out = _run([NVCC] + flags + ["-c", str(src), "-o", str(obj)])
            if verbose and out.strip():
                print(f"--- {src.name}\n{out}")
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, sources))
    lib = PKG / CUDA_LIB
    if force or _stale(lib, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "shared", "-o", str(lib)] +
             [str(o) for o in objs] +
             ["-Xlinker", f"-rpath,{CUDA_HOME / 'lib64'}", "-ldl"])
    return lib


def build_host(force=False, jobs=None) -> Path:
    """The C++23 host library (include/veda/*.hpp, csrc/host/*.cpp) linked against
    libveda_cuda.so, cudart and NCCL."""
    sources = sorted(HOST.glob("*.cpp"))
    if not sources:
        return None
    OBJ.mkdir(exist_ok=True)
    nccl_inc, nccl_lib = _nccl_paths()
    headers = _headers(HOST)
    cxx = os.environ.get("CXX", "g++")
    flags = ["-std=c++23", "-O2", "-fPIC", "-pthread", "-I", str(INCLUDE),
             "-I", str(CUDA_HOME / "include"), "-I", str(nccl_inc)]

    def compile_one(src: Path):
        obj = OBJ / ("host_" + src.stem + ".o")
        if force or _stale(obj, [src] + headers):
            _run([cxx] + flags + ["-c", str(src), "-o", str(obj)])
        return obj

    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        objs = list(ex.map(compile_one, sources))
    lib = PKG / HOST_LIB
    cuda_lib = PKG / CUDA_LIB
    if force or _stale(lib, objs + [cuda_lib]):
        nccl_so = next(iter(sorted(nccl_lib.glob("libnccl.so*"))), None)
        link_nccl = [str(nccl_so)] if nccl_so else ["-lnccl"]
        _run([cxx, "-shared", "-o", str(lib)] + [str(o) for o in objs] +
             ["-L", str(PKG), "-lveda_cuda", "-L", str(CUDA_HOME / "lib64"), "-lcudart"] +
             link_nccl +
             ["-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{CUDA_HOME / 'lib64'}",
              f"-Wl,-rpath,{nccl_lib}", "-pthread"])
    return lib


def build_all(force=False, verbose=False):
    build_cuda(force=force, verbose=verbose)
    build_host(force=force)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    build_all(force=a.force, verbose=a.verbose)
    print("built", PKG / CUDA_LIB, PKG / HOST_LIB)


if __name__ == "__main__":
    sys.exit(main())
