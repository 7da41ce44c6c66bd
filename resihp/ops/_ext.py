"""Loader for the in-tree sm_100a extension ``resihp/_C.so``.

The bf16 CUDA path has no fallback: a missing or unloadable extension is an error
(``require()`` raises), never a silent switch to torch kernels. FP32 tensors (CPU, or
CUDA in a reference-semantics run) take the plain-torch FP32 path of each op, which is
what the CPU test tier and the reference-semantics runs use.
"""

from __future__ import annotations

import importlib.util
import os

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
#: ``RESIHP_CHECKED=1`` loads the bounds-checked build of the same kernels instead.
CHECKED = os.environ.get("RESIHP_CHECKED", "0") == "1"
_NAME = "_C_checked" if CHECKED else "_C"
_LIB = os.path.join(_PKG, _NAME + ".so")
_module = None
_error: Exception | None = None


def _load():
    global _module, _error
    if _module is not None or _error is not None:
        return _module
    try:
        import torch  # noqa: F401  (libtorch must be loaded before the extension)

        spec = importlib.util.spec_from_file_location("resihp." + _NAME, _LIB)
        if spec is None or not os.path.exists(_LIB):
            raise ImportError(f"extension not built: {_LIB} (run python -m resihp.ops.build"
                              f"{' --checked' if CHECKED else ''})")
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
        _module = module
    except Exception as exc:  # kept and re-raised by require()
        _error = exc
    return _module


# Kernels each extension entry point launches (for the benchmark's launch count).
KERNELS_PER_CALL = {
    "gemm": 1, "rmsnorm_fwd": 1, "rmsnorm_bwd": 2, "rope": 1, "swiglu_fwd": 1, "swiglu_bwd": 1,
    "adamw": 1, "embedding_fwd": 1, "embedding_bwd": 2, "xent_stats": 1, "xent_grad": 1,
    "attn_fwd": 1, "attn_bwd": 3, "ag_gemm": 1, "gemm_rs": 1, "dp_allreduce_adamw": 1, "reshard_gather": 1,
}


class _Counting:
    """Proxy over the extension module that counts kernel launches per entry point."""

    def __init__(self, module):
        self._module = module
        self.launches = 0
        self.enabled = False

    def __getattr__(self, name):
        fn = getattr(self._module, name)
        per = KERNELS_PER_CALL.get(name)
        if per is None:
            return fn

        def counted(*args, **kwargs):
            if self.enabled:
                self.launches += per
            return fn(*args, **kwargs)

        return counted


_counting = None


def launch_counter() -> "_Counting":
    """The counting proxy; set ``.enabled`` and read ``.launches``."""
    require()
    return _counting


def available() -> bool:
    return _load() is not None


def require():
    """The loaded extension module; raises if it cannot be loaded."""
    global _counting
    module = _load()
    if module is None:
        raise RuntimeError(f"resihp CUDA extension unavailable: {_error}")
    if _counting is None:
        _counting = _Counting(module)
    return _counting


def library_path() -> str:
    return _LIB
