"""In-tree build of the native library and its PyTorch operator shim.

  libffa_b200.so   C ABI (include/ffa_b200.h): host planner + sm_100a kernels,
                   built with nvcc -gencode arch=compute_100a,code=sm_100a.
  _ffa_torch.so    torch.ops.ffa_b200.* operators over that C ABI.

Both land next to this file so they travel with the source tree; the Python
package loads them from here and fails loudly when they are missing.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
BUILD = HERE / "_build"
LIB = HERE / "libffa_b200.so"
SHIM = HERE / "_ffa_torch.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _cuda_home() -> str:
    return os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _stale(output: Path, inputs: list[Path]) -> bool:
    if not output.exists():
        return True
    mtime = output.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in inputs)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"build step failed ({proc.returncode}): {' '.join(cmd)}\n"
                           f"{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def build_library(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    sources = [CSRC / "ffa_kernels.cu", CSRC / "ffa_long.cu", CSRC / "ffa_window.cu", CSRC / "ffa_host.cpp",
               CSRC / "ffa_noalloc.cu"]
    headers = [CSRC / "ffa_internal.h", CSRC / "ffa_device.cuh", INCLUDE / "ffa_b200.h"]
    if not (force or _stale(LIB, sources + headers)):
        return LIB
    BUILD.mkdir(exist_ok=True)
    nvcc = f"{_cuda_home()}/bin/nvcc"
    common = ["-std=c++17", "-O3", f"-I{INCLUDE}", f"-I{CSRC}",
              "-Xcompiler", "-fPIC,-fvisibility=hidden"]
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        cmd = [nvcc, "-c", str(src), "-o", str(obj), *common]
        cmd += ARCH
        if src.suffix == ".cu":
            cmd += ["-lineinfo", "--fmad=false"]
            if ptxas_info:
                cmd += ["-Xptxas", "-v"]
        out = _run(cmd, verbose)
        if ptxas_info and out.strip():
            print(out)
        objs.append(str(obj))
    tmp = LIB.with_name(LIB.name + f".{os.getpid()}.tmp")
    _run([nvcc, "-shared", *ARCH, "-o", str(tmp), *objs, "-cudart", "static"], verbose)
    tmp.replace(LIB)
    return LIB


def build_shim(force: bool = False, verbose: bool = False) -> Path:
    src = CSRC / "ffa_torch.cpp"
    if not (force or _stale(SHIM, [src, INCLUDE / "ffa_b200.h", LIB])):
        return SHIM
    import torch
    from torch.utils.cpp_extension import include_paths, library_paths
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-shared", "-fPIC", "-std=c++17", "-O2", str(src), "-o",
           str(SHIM.with_name(SHIM.name + f".{os.getpid()}.tmp")),
           f"-I{INCLUDE}", *[f"-I{p}" for p in include_paths(device_type="cuda")],
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-L{HERE}", "-lffa_b200", "-Wl,-rpath,$ORIGIN",
           *[f"-L{p}" for p in library_paths(device_type="cuda")],
           f"-L{_cuda_home()}/lib64", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda",
           "-ltorch", "-lcudart"]
    _run(cmd, verbose)
    SHIM.with_name(SHIM.name + f".{os.getpid()}.tmp").replace(SHIM)
    return SHIM


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> None:
    build_library(force, verbose, ptxas_info)
    build_shim(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
