"""In-tree build of the sm_100a extension ``resihp._C``.

Compiles every ``resihp/csrc/*.cu`` and ``*.cpp`` with ``-gencode
arch=compute_100a,code=sm_100a`` only (an explicit arch flag keeps torch from adding
its own arch list) and leaves ``_C.so`` inside the package, so the built library
travels with the source tree and no JIT cache outside the repository is involved.

    python -m resihp.ops.build
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


def library_path() -> str:
    return os.path.join(PKG, NAME + ".so")


def build(verbose: bool = False) -> str:
    from torch.utils import cpp_extension

    os.makedirs(BUILD, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    cpp_extension.load(
        name=NAME,
        sources=sources(),
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=CUDA_FLAGS + ["-I" + CSRC, "-Xcompiler", "-fPIC"],
        extra_ldflags=["-lcuda"] if _has_libcuda() else [],
        build_directory=BUILD,
        verbose=verbose,
        with_cuda=True,
        is_python_module=True,
    )
    built = os.path.join(BUILD, NAME + ".so")
    shutil.copy2(built, library_path())
    return library_path()


def _has_libcuda() -> bool:
    return False  # the driver API is reached through cudaGetDriverEntryPoint


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
