"""In-tree build of the sm_100a extension ``resihp._C``.

Compiles every ``resihp/csrc/*.cu`` and ``*.cpp`` with ``-gencode
arch=compute_100a,code=sm_100a`` only (an explicit arch flag keeps torch from adding
its own arch list) and leaves ``_C.so`` inside the package, so the built library
travels with the source tree and no JIT cache outside the repository is involved.

``--checked`` builds the same sources with ``-DRESIHP_BOUNDS_CHECK`` into
``_C_checked.so``: the kernels then test the addresses they compute (TMA coordinates,
TMEM column ranges, vector-copy alignment) and record ``kErrBounds`` instead of
issuing a bad access. ``RESIHP_CHECKED=1`` makes the loader use it.

    python -m resihp.ops.build [--checked]
"""

from __future__ import annotations

import glob
import os
import shutil
import sys

PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
NAME = "_C"
CHECKED_NAME = "_C_checked"
CHECKED_FLAGS = ["-DRESIHP_BOUNDS_CHECK"]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def library_path(checked: bool = False) -> str:
    return os.path.join(PKG, (CHECKED_NAME if checked else NAME) + ".so")


def cuda_flags(checked: bool = False) -> list[str]:
    return CUDA_FLAGS + (CHECKED_FLAGS if checked else []) + ["-I" + CSRC, "-Xcompiler", "-fPIC"]


def build(verbose: bool = False, checked: bool = False) -> str:
    from torch.utils import cpp_extension

    name = CHECKED_NAME if checked else NAME
    directory = BUILD + ("_checked" if checked else "")
    os.makedirs(directory, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    cpp_extension.load(
        name=name,
        sources=sources(),
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=cuda_flags(checked),
        extra_ldflags=["-lcuda"] if _has_libcuda() else [],
        build_directory=directory,
        verbose=verbose,
        with_cuda=True,
        is_python_module=True,
    )
    built = os.path.join(directory, name + ".so")
    shutil.copy2(built, library_path(checked))
    return library_path(checked)


def _has_libcuda() -> bool:
    return False  # the driver API is reached through cudaGetDriverEntryPoint


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, checked="--checked" in sys.argv)
    print(path)
