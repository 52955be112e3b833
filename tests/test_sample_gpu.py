"""On-device sampling for temperature > 0 (hakmc_sample, hakmc_sample_last)
against the reference's own compiled sample_token (src/sample.c:27-58, built
into oracle/_ref): the same seeded logits, temperature, top_k and top_p and
the same generator state must give the same token, the same advanced state
and the same probabilities (the reference turns its logits into them in
place), bit for bit."""
import ctypes as C

import numpy as np
import pytest

from hako_b200 import HakmCtx, check, lib, synth

pytestmark = pytest.mark.gpu


class Sampler(C.Structure):  # src/sample.h:6-11
    _fields_ = [("temp", C.c_float), ("top_p", C.c_float), ("top_k", C.c_int), ("rng", C.c_uint64)]


def ref_sample(reference, logits, temp, top_p, top_k, rng):
    L = reference.L
    L.sample_token.restype = C.c_int
    L.sample_token.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    s = Sampler(temp, top_p, top_k, rng)
    x = np.array(logits, np.float32, copy=True)
    tok = L.sample_token(C.byref(s), C.c_void_p(x.ctypes.data), x.size)
    return tok, s.rng, x


def dev_sample(cuda, logits, temp, top_p, top_k, rng):
    import torch
    d = torch.from_numpy(np.array(logits, np.float32, copy=True)).to(cuda)
    st = C.c_ulonglong(rng)
    tok = C.c_int(-1)
    check(lib.hakmc_sample(C.c_void_p(d.data_ptr()), d.numel(), temp, top_p, top_k, C.byref(st), C.byref(tok),
                           None), "hakmc_sample")
    return tok.value, st.value, d.cpu().numpy()


CASES = [(0.7, 0.9, 40), (1.0, 0.0, 0), (0.25, 1.0, 0), (1.3, 0.5, 0), (0.7, 0.0, 1), (0.9, 0.95, 1000),
         (0.6, 0.0, 5000), (1.0, 0.999, 0)]


@pytest.mark.parametrize("n", [9, 10, 13, 100, 1024, 4099, 151936])
def test_sample_matches_reference(cuda, reference, n):
    rng = np.random.default_rng(n)
    state = 0x9e3779b97f4a7c15
    for temp, top_p, top_k in CASES:
        for scale in (0.5, 3.0):
            logits = (rng.standard_normal(n) * scale).astype(np.float32)
            a = ref_sample(reference, logits, temp, top_p, top_k, state)
            b = dev_sample(cuda, logits, temp, top_p, top_k, state)
            assert b[0] == a[0], (n, temp, top_p, top_k, scale, a[0], b[0])
            assert b[1] == a[1]
            assert np.array_equal(b[2].view(np.uint32), a[2].view(np.uint32)), (n, temp, top_p, top_k)
            state = a[1]


def test_sample_ties_keep_index_order(cuda, reference):
    """Many equal probabilities: the candidate order among ties (glibc's
    stable merge sort) decides the pick."""
    rng = np.random.default_rng(3)
    n = 20000
    state = 12345
    for trial in range(12):
        logits = rng.integers(-3, 4, n).astype(np.float32) * 0.5
        for temp, top_p, top_k in ((1.0, 0.9, 0), (0.8, 0.0, 300), (1.2, 0.3, 5000)):
            a = ref_sample(reference, logits, temp, top_p, top_k, state)
            b = dev_sample(cuda, logits, temp, top_p, top_k, state)
            assert (b[0], b[1]) == (a[0], a[1]), (trial, temp, top_p, top_k)
            state = a[1]


def test_greedy_sample_is_argmax(cuda, reference):
    rng = np.random.default_rng(9)
    logits = rng.standard_normal(5000).astype(np.float32)
    logits[[17, 4000]] = logits.max() + 1.0  # tie: the first wins
    a = ref_sample(reference, logits, 0.0, 0.9, 40, 77)
    b = dev_sample(cuda, logits, 0.0, 0.9, 40, 77)
    assert b[0] == a[0] == 17 and b[1] == a[1] == 77


def test_sample_last_on_model_logits(cuda, reference):
    """Sampling the context's own last logits on the device (no logits copy)
    equals the reference's sample_token on the reference's logits, step by
    step, each pick fed back."""
    from oracle.oracle import RefModel
    path = synth.cached_model(synth.PRESETS["small"])
    ref = RefModel(path, 64)
    state_r = state_d = 42
    with HakmCtx(path, max_seq=64) as ctx:
        tok = 11
        for step in range(12):
            lr, _ = ref.forward(tok)
            ctx.forward(tok, want_logits=False)
            a = ref_sample(reference, lr, 0.8, 0.9, 40, state_r)
            st = C.c_ulonglong(state_d)
            t = C.c_int(-1)
            check(lib.hakmc_sample_last(ctx._h, 0.8, 0.9, 40, C.byref(st), C.byref(t)), "sample_last")
            assert (t.value, st.value) == (a[0], a[1]), step
            state_r, state_d = a[1], st.value
            tok = a[0]
    ref.close()
