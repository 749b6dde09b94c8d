"""Build recipe for the parity checkers (test infrastructure, not product).

Outputs:
  oracle/libffa_oracle.so
      our C restatement of the reference's conventional path (ffa_oracle.c).
  oracle/_ref/ffa_corrected_ctc_cpp<EXT_SUFFIX>
      the reference repository's own CPU comparator
      (benchmarks/patches/cpu_corrected.cpp), compiled in place from the
      reference tree with the flags its adapter uses
      (benchmarks/adapters/cpp.py:42).
  oracle/_ref/fast_forced_aligner_cuda.so
      the reference's CUDA extension (src/fast_forced_aligner/csrc/
      alignment.cu) compiled in place for sm_100a with the flags its loader
      passes (alignment.py:60, "-O3 --fmad=false").  Loaded with
      torch.ops.load_library, it registers the reference's own
      torch.ops.fast_forced_aligner_cuda.{align,emission_validity} ops, which the
      GPU parity tests and bench.py's reference lanes call.

Reference sources are read where they lie and never copied; every output
lands under oracle/ (the _ref/ folder is git-ignored but travels to the GPU
box with the rest of the tree).  The reference tree is absent on the GPU box:
there, only the prebuilt files are used.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
# The reference checkout: FFA_REFERENCE_ROOT, else a "reference" folder beside
# this repository's root.  Where neither exists (the GPU box), only the
# prebuilt checkers under oracle/_ref are used.
REFERENCE = Path(os.environ.get("FFA_REFERENCE_ROOT") or HERE.parent.parent / "reference")
ORACLE_SO = HERE / "libffa_oracle.so"
CORRECTED_SO = REF_OUT / ("ffa_corrected_ctc_cpp" + sysconfig.get_config_var("EXT_SUFFIX"))
REF_CUDA_SO = REF_OUT / "fast_forced_aligner_cuda.so"


def _stale(output: Path, *inputs: Path) -> bool:
    if not output.exists():
        return True
    mtime = output.stat().st_mtime
    return any(p.stat().st_mtime > mtime for p in inputs)


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True)


def build_oracle(force: bool = False) -> Path:
    src = HERE / "ffa_oracle.c"
    if force or _stale(ORACLE_SO, src, HERE / "ffa_oracle.h"):
        tmp = ORACLE_SO.with_suffix(f".{os.getpid()}.tmp")
        _run(["gcc", "-O2", "-std=gnu11", "-D_GNU_SOURCE", "-ffp-contract=off",
              "-fno-fast-math", "-fPIC", "-shared", "-pthread", str(src),
              "-o", str(tmp), "-lm"])
        tmp.replace(ORACLE_SO)
    return ORACLE_SO


def build_corrected(force: bool = False) -> Path | None:
    src = REFERENCE / "benchmarks" / "patches" / "cpu_corrected.cpp"
    if not src.is_file():
        return CORRECTED_SO if CORRECTED_SO.exists() else None
    REF_OUT.mkdir(exist_ok=True)
    if force or _stale(CORRECTED_SO, src):
        import pybind11
        tmp = CORRECTED_SO.with_name(CORRECTED_SO.name + f".{os.getpid()}.tmp")
        _run(["g++", "-O3", "-shared", "-std=c++17", "-fPIC", "-pthread",
              "-I" + sysconfig.get_paths()["include"], "-I" + pybind11.get_include(),
              str(src), "-o", str(tmp)])
        tmp.replace(CORRECTED_SO)
    return CORRECTED_SO


def build_reference_cuda(force: bool = False) -> Path | None:
    src = REFERENCE / "src" / "fast_forced_aligner" / "csrc" / "alignment.cu"
    if not src.is_file():
        return REF_CUDA_SO if REF_CUDA_SO.exists() else None
    REF_OUT.mkdir(exist_ok=True)
    if not (force or _stale(REF_CUDA_SO, src)):
        return REF_CUDA_SO
    import torch
    from torch.utils.cpp_extension import include_paths, library_paths
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    obj = REF_OUT / f"alignment.{os.getpid()}.o"
    tmp = REF_CUDA_SO.with_name(REF_CUDA_SO.name + f".{os.getpid()}.tmp")
    incs = [f"-I{p}" for p in include_paths(device_type="cuda")]
    try:
        _run([f"{cuda_home}/bin/nvcc", "-c", str(src), "-o", str(obj), *incs,
              "-O3", "--fmad=false", "-std=c++17",
              "-gencode", "arch=compute_100a,code=sm_100a",
              "-Xcompiler", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              "-DTORCH_EXTENSION_NAME=fast_forced_aligner_cuda",
              "-DTORCH_API_INCLUDE_EXTENSION_H",
              "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
              "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__",
              "--expt-relaxed-constexpr"])
        libs = [f"-L{p}" for p in library_paths(device_type="cuda")]
        _run(["g++", "-shared", str(obj), "-o", str(tmp), *libs,
              f"-L{cuda_home}/lib64", "-lc10", "-lc10_cuda", "-ltorch_cpu",
              "-ltorch_cuda", "-ltorch", "-lcudart"])
        tmp.replace(REF_CUDA_SO)
    finally:
        obj.unlink(missing_ok=True)
        tmp.unlink(missing_ok=True)
    return REF_CUDA_SO


def build_all(force: bool = False, reference_cuda: bool = True) -> None:
    build_oracle(force)
    if not REFERENCE.is_dir():
        print(f"oracle/build.py: no reference tree at {REFERENCE} (set FFA_REFERENCE_ROOT); "
              "using the prebuilt checkers under oracle/_ref, if any", file=sys.stderr)
    build_corrected(force)
    if reference_cuda:
        build_reference_cuda(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, reference_cuda="--no-ref-cuda" not in sys.argv)
