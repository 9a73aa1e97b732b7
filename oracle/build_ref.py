"""Recipe: the reference project's own CUDA kernels, compiled for sm_100a.

TEST INFRASTRUCTURE. Compiles the reference's two source files
(csrc/rmsnorm_kernels.cu and csrc/bindings.cpp) where they lie, with the flags
of its setup.py (nvcc -O3 --use_fast_math -lineinfo, c++ -O3) but for
sm_100a, into ``oracle/_ref/sm120_reference_C*.so`` -- a PyTorch extension
module exposing the reference's seven pybind functions. Its TORCH_LIBRARY
namespace is renamed (``-Dsm120_norm=sm120_norm_reference``) so it can be
loaded next to this repository's extension. Nothing under the reference tree
is modified or copied; the build folder is ``oracle/_ref/build``.

Used only by the tests (a second checker) and by ``bench.py --impl reference``
(timing the reference's kernels on the same B200). The GPU host has no copy of
the reference, so the built module travels with the repository snapshot.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
MODULE = "sm120_reference_C"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))


def module_path() -> Path:
    return OUT / f"{MODULE}{sysconfig.get_config_var('EXT_SUFFIX') or '.so'}"


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"reference build step failed: {cmd[0]}")


def reference_root(reference: Path | str | None = None) -> Path | None:
    """The reference checkout to build from: `reference`, else the
    SM120N_REFERENCE_ROOT environment variable; None when neither is given."""
    if reference is None:
        reference = os.environ.get("SM120N_REFERENCE_ROOT")
    return Path(reference) if reference else None


def build(reference: Path, force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    kernels = reference / "csrc" / "rmsnorm_kernels.cu"
    bindings = reference / "csrc" / "bindings.cpp"
    target = module_path()
    if (not force and target.exists()
            and target.stat().st_mtime >= max(kernels.stat().st_mtime, bindings.stat().st_mtime)):
        return target
    build_dir = OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    includes = [*cpp_extension.include_paths(), sysconfig.get_paths()["include"],
                str(CUDA_HOME / "include")]
    defines = [f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
               f"-DTORCH_EXTENSION_NAME={MODULE}", "-DTORCH_API_INCLUDE_EXTENSION_H"]
    inc = [f"-I{i}" for i in includes]
    kernels_obj = build_dir / "rmsnorm_kernels.o"
    _run([str(CUDA_HOME / "bin" / "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a",
          "-O3", "--use_fast_math", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
          *cpp_extension.COMMON_NVCC_FLAGS, *defines, *inc, "-c", str(kernels),
          "-o", str(kernels_obj)])
    bindings_obj = build_dir / "bindings.o"
    _run(["g++", "-O3", "-std=c++17", "-fPIC", *defines, "-Dsm120_norm=sm120_norm_reference",
          *inc, "-c", str(bindings), "-o", str(bindings_obj)])
    libdirs = cpp_extension.library_paths()
    tmp = build_dir / target.name
    _run(["g++", "-shared", str(kernels_obj), str(bindings_obj), "-o", str(tmp),
          *[f"-L{d}" for d in libdirs], *[f"-Wl,-rpath,{d}" for d in libdirs],
          f"-L{CUDA_HOME / 'lib64'}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
          "-ltorch_cuda", "-ltorch_python", "-lcudart"])
    os.replace(tmp, target)
    for leftover in build_dir.iterdir():  # only the module travels
        leftover.unlink()
    build_dir.rmdir()
    return target


def build_if_present(reference: Path | str | None = None) -> Path | None:
    """Build when a reference checkout is given (argument or
    SM120N_REFERENCE_ROOT) and present; otherwise use whatever was built
    before, if anything."""
    root = reference_root(reference)
    if root is not None and (root / "csrc" / "rmsnorm_kernels.cu").exists():
        return build(root)
    return module_path() if module_path().exists() else None


def load():
    """Import the built module, or return None if it was never built."""
    if not module_path().exists():
        return None
    if str(OUT) not in sys.path:
        sys.path.insert(0, str(OUT))
    import importlib
    return importlib.import_module(MODULE)


if __name__ == "__main__":
    import argparse

    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", type=Path, default=None,
                        help="reference checkout (default: $SM120N_REFERENCE_ROOT)")
    parser.add_argument("--force", action="store_true")
    cli = parser.parse_args()
    root = reference_root(cli.reference)
    if root is None:
        parser.error("give --reference or set SM120N_REFERENCE_ROOT")
    print(build(root, force=cli.force))
