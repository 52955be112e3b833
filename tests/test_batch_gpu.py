"""Batched Q4_K x q8_32 matmuls against the reference's own Q4_K matmul
(src/nn.c:76-82 -> q4k_vec_dot, src/quant.c:150-232), applied to each
activation of the batch.

Bars: the tensor-core kernel (hakmc_gemm_q4k_q8, and hakmc_gemv_q4k_q8_batch
where it routes there) restates the reference's fp32 steps and order, so it
is bit-identical. The dp4a kernel behind hakmc_gemv_q4k_q8_batch's short
batches sums per-chunk partials: rel-L2 <= 1e-5 per activation (the q8 codes
and the per-32 integer sums are exact; only the fp32 summation order
differs), and bit-identical results across repeated calls (the partials are
summed in a fixed order whatever the grid)."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2
from hako_b200 import check, lib, synth

pytestmark = pytest.mark.gpu

TOL = 1e-5


def same(a, b):
    return np.array_equal(np.ascontiguousarray(a, np.float32).view(np.uint32),
                          np.ascontiguousarray(b, np.float32).view(np.uint32))


def P(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def run_batch(cuda, w, xq, xs, bias, rows, k, n, scratch=False):
    import torch
    wd = torch.from_numpy(w).to(cuda)
    xqd = torch.from_numpy(np.ascontiguousarray(xq)).to(cuda)
    xsd = torch.from_numpy(np.ascontiguousarray(xs)).to(cuda)
    bd = torch.from_numpy(bias).to(cuda) if bias is not None else None
    out = torch.full((n, rows), float("nan"), dtype=torch.float32, device=cuda)
    if scratch:
        nbytes = lib.hakmc_gemv_q4k_q8_batch_scratch(rows, k, n)
        sc = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
        for _ in range(2):  # a call leaves the scratch reusable
            check(lib.hakmc_gemv_q4k_q8_batch(P(out), P(wd), P(xqd), P(xsd), P(bd), rows, k, n, P(sc), nbytes, None))
    else:
        check(lib.hakmc_gemv_q4k_q8_batch(P(out), P(wd), P(xqd), P(xsd), P(bd), rows, k, n, None, 0, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


# config-1 shapes (rows x K) at batch 1/4/16/64, plus ragged cases: a row
# count that is not a multiple of the 32-row tile, a K whose last 8-block
# chunk is partial, and batches that are not powers of two or exceed one
# launch's 16 activations
CASES = [(256, 2048, 1), (2048, 2048, 4), (11008, 2048, 16), (2048, 11008, 16), (3584, 18944, 4),
         (18944, 3584, 1), (512, 3584, 64), (5, 256, 3), (33, 2304, 17), (100, 512, 7)]


@pytest.mark.parametrize("rows,k,n", CASES)
def test_gemv_q4k_batch_matches_reference(cuda, reference, rows, k, n):
    w = synth.random_q4k(rows, k, 7 * rows + k + n)
    xs_f = [synth.normal(k, 1000 + 13 * i + k) for i in range(n)]
    q = [reference.quantize_q8_32(x) for x in xs_f]
    xq = np.stack([a for a, _ in q])
    xs = np.stack([b for _, b in q])
    bias = synth.normal(rows, 79) if n % 2 else None
    out = run_batch(cuda, w, xq, xs, bias, rows, k, n, scratch=(rows % 2 == 0))
    # the routing of hakmc_gemv_q4k_q8_batch: above 16 activations (above 8
    # for 16M weights or more in 64 or more row tiles) the tensor cores
    exact = n > 16 or (n > 8 and rows * k >= 16 << 20 and (rows + 127) // 128 >= 64)
    for i in range(n):
        ref = reference.matmul(w, 12, xs_f[i], rows, k, bias=bias)
        if exact:
            assert same(out[i], ref), (i, rel_l2(out[i], ref))
        else:
            assert rel_l2(out[i], ref) < TOL, i


@pytest.mark.parametrize("rows,k,n", [(2048, 11008, 16), (3584, 18944, 4)])
def test_gemv_q4k_batch_deterministic(cuda, reference, rows, k, n):
    # chunk-order partials summed by the second kernel; tile order with
    # tiles shared by several CTAs (their pieces summed by the last one)
    w = synth.random_q4k(rows, k, 5)
    q = [reference.quantize_q8_32(synth.normal(k, 50 + i)) for i in range(n)]
    xq = np.stack([a for a, _ in q])
    xs = np.stack([b for _, b in q])
    a = run_batch(cuda, w, xq, xs, None, rows, k, n)
    b = run_batch(cuda, w, xq, xs, None, rows, k, n, scratch=True)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_gemv_q4k_batch_rejects_bad_shapes(cuda):
    import torch
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    p = C.c_void_p(buf.data_ptr())
    assert lib.hakmc_gemv_q4k_q8_batch(p, p, p, p, None, 4, 300, 1, None, 0, None) < 0  # K not a multiple of 256
    assert lib.hakmc_gemv_q4k_q8_batch(p, p, p, p, None, 4, 256, 0, None, 0, None) < 0  # empty batch
    assert lib.hakmc_gemv_q4k_q8_batch(p, C.c_void_p(buf.data_ptr() + 8), p, p, None, 4, 256, 1,
                                       None, 0, None) < 0  # unaligned w
    assert lib.hakmc_gemv_q4k_q8_batch(p, p, p, p, None, 64, 4096, 4, p, 16, None) < 0  # scratch too small


def run_tc(cuda, w, xq, xs, bias, rows, k, n):
    import torch
    wd = torch.from_numpy(w).to(cuda)
    xqd = torch.from_numpy(np.ascontiguousarray(xq)).to(cuda)
    xsd = torch.from_numpy(np.ascontiguousarray(xs)).to(cuda)
    bd = torch.from_numpy(bias).to(cuda) if bias is not None else None
    out = torch.full((n, rows), float("nan"), dtype=torch.float32, device=cuda)
    check(lib.hakmc_gemm_q4k_q8(P(out), P(wd), P(xqd), P(xsd), P(bd), rows, k, n, None, 0, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


# tensor-core path: activation tiles of 16 or 32; ragged rows (not a
# multiple of the 128-row tile), ragged batches, one super-block, long rows
# with few row tiles
TC_CASES = [(256, 2048, 16), (2048, 2048, 64), (11008, 2048, 64), (2048, 11008, 64), (3584, 18944, 16),
            (300, 512, 100), (5, 256, 1), (130, 2304, 130), (512, 3584, 256), (1000, 1024, 30), (18944, 3584, 4)]


@pytest.mark.parametrize("rows,k,n", TC_CASES)
def test_gemm_q4k_tensor_cores_match_reference(cuda, reference, rows, k, n):
    w = synth.random_q4k(rows, k, 11 * rows + k + n)
    xs_f = [synth.normal(k, 2000 + 17 * i + k) for i in range(n)]
    q = [reference.quantize_q8_32(x) for x in xs_f]
    xq = np.stack([a for a, _ in q])
    xs = np.stack([b for _, b in q])
    bias = synth.normal(rows, 81) if n % 2 == 0 else None
    out = run_tc(cuda, w, xq, xs, bias, rows, k, n)
    for i in range(n):
        ref = reference.matmul(w, 12, xs_f[i], rows, k, bias=bias)
        assert same(out[i], ref), (i, rel_l2(out[i], ref))


def test_gemm_q4k_tensor_cores_deterministic(cuda, reference):
    rows, k, n = 2048, 3584, 64
    w = synth.random_q4k(rows, k, 6)
    q = [reference.quantize_q8_32(synth.normal(k, 70 + i)) for i in range(n)]
    xq = np.stack([a for a, _ in q])
    xs = np.stack([b for _, b in q])
    a = run_tc(cuda, w, xq, xs, None, rows, k, n)
    b = run_tc(cuda, w, xq, xs, None, rows, k, n)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
