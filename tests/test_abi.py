"""The C ABI library loads, exports every symbol include/hakm_cuda.h declares,
and rejects malformed MLF2 images the way the reference loader does
(src/loader.c:26-44) — all without a GPU."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from hako_b200 import _lib, synth

HEADER = os.path.join(ROOT, "include", "hakm_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hakmc_\w+)\s*\(", src)))


def test_header_symbols_exported():
    names = declared_symbols()
    assert len(names) >= 25
    lib = C.CDLL(_lib.CUDA_LIB_PATH)
    for n in names:
        assert hasattr(lib, n), f"{n} declared but not exported"
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)


def test_library_is_sm100a_only():
    # the shipped library carries sm_100a SASS; nothing else is compiled in
    from hako_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version():
    assert _lib.lib.hakmc_version() == 100


def _create(img: np.ndarray):
    return _lib.lib.hakmc_create(C.c_void_p(img.ctypes.data), img.nbytes, 64, 1, 0)


def test_rejects_bad_magic():
    img = np.frombuffer(b"GGUF" + bytes(200), np.uint8).copy()
    assert not _create(img)
    assert "magic" in _lib.last_error()


def test_rejects_short_and_bad_version():
    assert not _create(np.zeros(16, np.uint8))
    assert "small" in _lib.last_error()
    img = np.zeros(256, np.uint8)
    img[:4] = np.frombuffer(b"MLF2", np.uint8)
    img[4] = 3
    assert not _create(img)
    assert "version" in _lib.last_error()


def test_rejects_corrupt_offsets():
    path = synth.cached_model(synth.PRESETS["tiny"])
    img = np.fromfile(path, np.uint8)
    bad = img.copy()
    bad[60:68] = np.frombuffer(np.uint64(1 << 40).tobytes(), np.uint8)  # tensors_off
    assert not _create(bad)
    assert "offsets" in _lib.last_error()
    trunc = img[: len(img) // 2].copy()  # tensor data past the end
    assert not _create(trunc)
    assert "past end" in _lib.last_error()


def test_kernel_entry_points_validate_shapes():
    lib = _lib.lib
    assert lib.hakmc_quantize_q8_32(None, 33, None, None, None) == -22
    assert lib.hakmc_gemv_q4k(None, None, None, None, 16, 300, None) == -22
    assert lib.hakmc_q6k_packed_bytes(10, 2048) == 10 * 8 * 210


def test_python_api_reports_errors(tmp_path):
    from hako_b200 import HakmCtx
    p = tmp_path / "bad.mlf2"
    p.write_bytes(b"NOPE" + bytes(300))
    with pytest.raises(RuntimeError, match="magic"):
        HakmCtx(str(p))


def test_batched_matmul_scratch_sizes():
    """Host-side planning of the batched matmuls (no GPU: 148 SMs assumed).
    dp4a path: one row chunk needs no partials; chunk-order launches keep one
    float per (chunk, activation, row). Tensor-core path: a row is never
    split along K, so it needs no scratch."""
    L = _lib.lib
    assert L.hakmc_gemv_q4k_q8_batch_scratch(4, 300, 1) == 0   # K not a multiple of 256
    assert L.hakmc_gemv_q4k_q8_batch_scratch(4, 256, 0) == 0   # empty batch
    # 2048 x 11008 at 16 activations: 6 chunks x 16 x 2048 partials (chunk order)
    assert L.hakmc_gemv_q4k_q8_batch_scratch(2048, 11008, 16) >= 6 * 16 * 2048 * 4
    # a single chunk per row and one tile per CTA: tickets only
    small = L.hakmc_gemv_q4k_q8_batch_scratch(2048, 2048, 4)
    assert 0 < small < 64 * 1024
    for shape in [(0, 256, 1), (18944, 3584, 64), (2048, 11008, 64), (5, 256, 3)]:
        assert L.hakmc_gemm_q4k_q8_scratch(*shape) == 0
