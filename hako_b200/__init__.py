"""hako_b200 — B200 (sm_100a) decode path for the hako engine.

The compute lives in libhakm_cuda.so (hand-written CUDA behind a C ABI,
include/hakm_cuda.h). This package is its Python binding plus the seeded
synthetic workloads. The library loads on first use of `lib`, `HakmCtx` or
the helpers below and raises if it is not built: there is no fallback.
"""
import importlib

__all__ = ["HakmCtx", "HakmcError", "lib", "check", "last_error"]

_LAZY = {"HakmCtx": ".model", "HakmcError": "._lib", "lib": "._lib", "check": "._lib",
         "last_error": "._lib"}


def __getattr__(name):
    if name in _LAZY:
        mod = importlib.import_module(_LAZY[name], __name__)
        return getattr(mod, name)
    raise AttributeError(name)
