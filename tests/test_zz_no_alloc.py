"""hakmc_attention_noalloc: the attention entry point for callers that cannot
allocate device memory once running (a host whose device budget belongs to
another framework's pool, or a loop that must not take cudaMalloc's device
synchronisation). Its scratch is a fixed ~1 MiB array inside the library
instead of an allocation. Checked against hakmc_attention, which allocates its
scratch, on the same inputs, two calls in a row (the array keeps the previous
call's contents, so the second call proves the reset). Collected last so a
stop-at-first-failure run has already run every other test."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_l2
from hako_b200 import check, lib

pytestmark = pytest.mark.gpu

TOL = 1e-5  # the kernel tests' fp32 bar; both calls run the same kernel


def _run(fn, cuda, q, kc, vc, pos, H, KVH, hd):
    import torch
    out = torch.empty(H * hd, dtype=torch.float32, device=cuda)
    dq = torch.from_numpy(q).to(cuda)
    dk = torch.from_numpy(kc).to(cuda)
    dv = torch.from_numpy(vc).to(cuda)
    rc = fn(C.c_void_p(out.data_ptr()), C.c_void_p(dq.data_ptr()), C.c_void_p(dk.data_ptr()),
            C.c_void_p(dv.data_ptr()), pos, H, KVH, hd, None)
    check(rc, fn.__name__)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("H,KVH,hd,pos", [(16, 2, 128, 300), (28, 4, 128, 1000), (4, 2, 64, 0)])
def test_noalloc_matches_allocating_entry_point(cuda, H, KVH, hd, pos):
    rng = np.random.default_rng(pos + 7 * H)
    max_seq = pos + 1
    outs = []
    for call in range(2):
        q = rng.standard_normal(H * hd).astype(np.float32)
        kc = rng.standard_normal((max_seq, KVH * hd)).astype(np.float32)
        vc = rng.standard_normal((max_seq, KVH * hd)).astype(np.float32)
        ref = _run(lib.hakmc_attention, cuda, q, kc, vc, pos, H, KVH, hd)
        got = _run(lib.hakmc_attention_noalloc, cuda, q, kc, vc, pos, H, KVH, hd)
        assert rel_l2(got, ref) < TOL, (call, rel_l2(got, ref))
        outs.append(got)
    assert not np.array_equal(outs[0], outs[1])  # the second call computed new inputs


def test_noalloc_rejects_oversize(cuda):
    import torch
    H, KVH, hd, pos = 32, 8, 128, 8191  # 32 * 128 chunks * 130 floats > the fixed array
    buf = torch.zeros(1, dtype=torch.float32, device=cuda)
    p = C.c_void_p(buf.data_ptr())
    rc = lib.hakmc_attention_noalloc(p, p, p, p, pos, H, KVH, hd, None)
    assert rc == -34
    from hako_b200 import last_error
    assert "fixed array" in last_error()
