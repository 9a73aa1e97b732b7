"""Build the B200 kernels in place.

Produces, inside ``sm120_rmsnorm/``:
  * ``libsm120norm_b200.so`` -- the C-ABI library (include/sm120norm_b200.h):
    all CUDA kernels, compiled for sm_100a only, every non-ABI symbol hidden;
  * ``_C<ext suffix>``       -- the PyTorch binding (csrc/torch_binding.cpp),
    linked against the library through an ``$ORIGIN`` rpath.

Usage: ``python build.py [--force] [--verbose]`` (``--verbose`` prints
``ptxas -v`` register / spill / shared-memory reports).
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REPO = ROOT.parent
PACKAGE = ROOT / "sm120_rmsnorm"
CSRC = ROOT / "csrc"
INCLUDE = REPO / "include"
BUILD = ROOT / "_build"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["runtime.cu", "row_norm.cu", "head_norm_rope.cu", "head_cache.cu", "norm_quant.cu", "norm_fp4.cu", "qkv_gemm.cu"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    f"-I{INCLUDE}", f"-I{CSRC}",
]
LIBRARY = PACKAGE / "libsm120norm_b200.so"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd[:3])} ...")
    return proc.stdout + proc.stderr


def _torch_cudart_dirs() -> list[Path]:
    """Directories holding the libcudart.so.12 that PyTorch loads, if any."""
    try:
        import torch
    except ImportError:
        return []
    site = Path(torch.__file__).resolve().parent.parent
    return [d for d in [site / "nvidia" / "cuda_runtime" / "lib"] if (d / "libcudart.so.12").exists()]


def build_library(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    jobs = []
    for name in CUDA_SOURCES:
        src = CSRC / name
        obj = BUILD / (Path(name).stem + ".o")
        if force or _stale(obj, [src, *headers]):
            cmd = [NVCC, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)
    if jobs:
        with ThreadPoolExecutor(max_workers=len(jobs)) as pool:
            for out in pool.map(lambda c: _run(c, verbose), jobs):
                if verbose and out:
                    print(out)
    objects = [BUILD / (Path(n).stem + ".o") for n in CUDA_SOURCES]
    if force or jobs or _stale(LIBRARY, objects):
        tmp = BUILD / LIBRARY.name
        # The CUDA runtime is linked as a shared library so that, inside a
        # PyTorch process, this library and PyTorch share one runtime instance
        # (one current device, one set of streams). The rpath prefers the
        # runtime PyTorch ships with, then the toolkit's.
        rpaths = [str(p) for p in _torch_cudart_dirs()] + [str(CUDA_HOME / "lib64")]
        _run([NVCC, *ARCH, "-shared", "-cudart", "shared", *map(str, objects), "-o", str(tmp),
              "-Xlinker", "--exclude-libs,ALL", "-Xlinker", "-Bsymbolic",
              *[f"-Xlinker=-rpath,{r}" for r in rpaths]], verbose)
        os.replace(tmp, LIBRARY)
    return LIBRARY


def _torch_flags() -> tuple[list[str], list[str]]:
    import torch
    from torch.utils import cpp_extension

    includes = [*cpp_extension.include_paths(), sysconfig.get_paths()["include"],
                str(CUDA_HOME / "include"), str(INCLUDE)]
    flags = [f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
             "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    libdirs = cpp_extension.library_paths()
    link = [f"-L{d}" for d in libdirs] + [f"-Wl,-rpath,{d}" for d in libdirs]
    link += ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python"]
    return [f"-I{i}" for i in includes] + flags, link


def build_binding(force: bool = False, verbose: bool = False) -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    target = PACKAGE / f"_C{suffix}"
    src = CSRC / "torch_binding.cpp"
    if not force and not _stale(target, [src, LIBRARY, *INCLUDE.glob("*.h")]):
        return target
    compile_flags, link_flags = _torch_flags()
    BUILD.mkdir(exist_ok=True)
    tmp = BUILD / target.name
    cxx = shutil.which("g++") or "g++"
    _run([cxx, "-O2", "-std=c++17", "-fPIC", "-shared", *compile_flags, str(src), "-o", str(tmp),
          *link_flags, f"-L{PACKAGE}", "-l:libsm120norm_b200.so", "-Wl,-rpath,$ORIGIN"], verbose)
    os.replace(tmp, target)
    return target


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force, verbose)
    build_binding(force, verbose)


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    build(args.force, args.verbose)
    print(f"built {LIBRARY.name} and the _C extension in {PACKAGE}")
