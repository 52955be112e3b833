"""hako_b200 — B200 (sm_100a) decode path for the hako engine.

The compute lives in libhakm_cuda.so (hand-written CUDA behind a C ABI,
include/hakm_cuda.h). This package is its Python binding plus the seeded
synthetic workloads; importing it fails loudly if the library is not built.
"""
from ._lib import HakmcError, check, last_error, lib  # noqa: F401
from .model import HakmCtx  # noqa: F401

__all__ = ["HakmCtx", "HakmcError", "lib", "check", "last_error"]
