"""ctypes binding of libhakm_cuda (include/hakm_cuda.h).

The library is the product: if it is missing this module raises at import
time rather than falling back to anything else.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(HERE, "_lib")
CUDA_LIB_PATH = os.path.join(LIB_DIR, "libhakm_cuda.so")

# Every symbol include/hakm_cuda.h declares: name -> (restype, argtypes)
_vp, _i, _f, _sz = C.c_void_p, C.c_int, C.c_float, C.c_size_t
SIGNATURES = {
    "hakmc_last_error": (C.c_char_p, []),
    "hakmc_version": (_i, []),
    "hakmc_create": (_vp, [_vp, _sz, _i, _i, _i]),
    "hakmc_destroy": (None, [_vp]),
    "hakmc_free": (None, [_vp]),
    "hakmc_prefill": (_i, [_vp, _vp, _i, _vp, _vp]),
    "hakmc_prefill_batched": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "hakmc_fill_kv_normal": (_i, [_vp, _i, _i, C.c_ulonglong]),
    "hakmc_tp_handle_bytes": (C.c_size_t, []),
    "hakmc_tp_export": (_i, [_vp, _vp]),
    "hakmc_tp_connect": (_i, [_vp, _i, _i, _vp]),
    "hakmc_tp_rank": (_i, [_vp]),
    "hakmc_tp_world": (_i, [_vp]),
    "hakmc_reset": (None, [_vp]),
    "hakmc_pos": (_i, [_vp]),
    "hakmc_set_pos": (_i, [_vp, _i]),
    "hakmc_vocab": (_i, [_vp]),
    "hakmc_dim": (_i, [_vp]),
    "hakmc_n_layers": (_i, [_vp]),
    "hakmc_forward": (_i, [_vp, _i, _vp, _vp]),
    "hakmc_generate": (_i, [_vp, _vp, _i, _i, _vp]),
    "hakmc_forward_batch": (_i, [_vp, _vp, _vp, _i, _vp, _vp]),
    "hakmc_decode": (_i, [_vp, _i, _vp]),
    "hakmc_time_phase": (_i, [_vp, _i, _i, _vp]),
    "hakmc_trace_phase": (_i, [_vp, _i, _i, _vp, _i]),
    "hakmc_trace_step": (_i, [_vp, _vp, _i]),
    "hakmc_set_layers": (_i, [_vp, _i]),
    "hakmc_hidden": (_i, [_vp, _i, _vp]),
    "hakmc_fill_kv": (_i, [_vp, _i, _vp, _vp, _i]),
    "hakmc_debug_read": (_i, [_vp, _i, _vp]),
    "hakmc_last_device_ms": (_f, [_vp]),
    "hakmc_quantize_q8_32": (_i, [_vp, _i, _vp, _vp, _vp]),
    "hakmc_gemv_q4k_q8": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _vp]),
    "hakmc_gemv_q4k_q8_batch_scratch": (_sz, [_i, _i, _i]),
    "hakmc_gemv_q4k_q8_batch": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "hakmc_gemm_q4k_q8_scratch": (_sz, [_i, _i, _i]),
    "hakmc_gemm_q4k_q8": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp, _sz, _vp]),
    "hakmc_gemv_q4k": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "hakmc_q4k_subsums": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "hakmc_q6k_pack": (_i, [_vp, _vp, _i, _i, _vp]),
    "hakmc_q6k_packed_bytes": (_sz, [_i, _i]),
    "hakmc_gemv_q6k": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp]),
    "hakmc_lmhead_argmax": (_i, [_vp, _vp, _vp, _vp, _vp, _f, _i, _i, _vp]),
    "hakmc_dequant": (_i, [_vp, _vp, _i, _i, _i, _vp]),
    "hakmc_rmsnorm": (_i, [_vp, _vp, _vp, _i, _f, _vp]),
    "hakmc_attention": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "hakmc_rope_neox": (_i, [_vp, _i, _i, _i, _f, _vp]),
    "hakmc_attention_noalloc": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "hakmc_attention_rows": (_i, [_vp, _vp, _vp, _vp, _i, _i, _vp, _i, _sz, _i, _i, _i, _vp]),
    "hakmc_gemm_q6k": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "hakmc_test_expf": (_i, [_vp, _vp, _i, _i, _vp]),
    "hakmc_sample": (_i, [_vp, _i, _f, _f, _i, _vp, _vp, _vp]),
    "hakmc_sample_last": (_i, [_vp, _f, _f, _i, _vp, _vp]),
    "hakmc_plan_rows": (_i, [_vp, _i, _i, _i, _vp]),
    "hakmc_plan_attn_units": (_i, [_i, _i, _i, _i, _vp, _i]),
}


class HakmcError(RuntimeError):
    """A libhakm_cuda call returned an error code."""


def _load() -> C.CDLL:
    if not os.path.exists(CUDA_LIB_PATH):
        raise ImportError(
            f"{CUDA_LIB_PATH} is missing: build it with `python -m hako_b200.build` "
            "(the CUDA path has no fallback)")
    lib = C.CDLL(CUDA_LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def last_error() -> str:
    return (lib.hakmc_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str = "") -> int:
    if rc < 0:
        raise HakmcError(f"{what or 'hakmc'} failed ({rc}): {last_error()}")
    return rc
