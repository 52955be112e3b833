"""Pins the CPU oracle against the reference engine's own outputs (golden
vectors made by tests/golden/make_golden.py from oracle/_ref) and, when the
reference build is present, against it directly on fresh random inputs.

The oracle restates the reference's arithmetic as its own build performs it
(-O3 -ffast-math -march=x86-64-v3: lane orders, fused multiply-adds,
rsqrtss, glibc/libmvec exp), so every comparison here is bit for bit."""
import ctypes as C
import os

import numpy as np
import pytest

from conftest import first_divergence, golden_json, golden_npz, have_reference, rel_l2
from hako_b200 import synth


def test_q8_golden_bit_exact(oracle):
    g = golden_npz("q8.npz")
    n = len([k for k in g.files if k.startswith("xq")])
    assert n >= 6
    for i in range(n):
        xq, xs = oracle.quantize_q8_32(g[f"x{i}"])
        assert np.array_equal(xq, g[f"xq{i}"]), f"case {i}"
        assert np.array_equal(xs.view(np.uint32), g[f"xs{i}"].view(np.uint32)), f"case {i}"


def test_q8_edge_semantics(oracle):
    # all-zero block: scale 0, every code 0; .5 ties round to even
    g = golden_npz("q8.npz")
    xq, xs = oracle.quantize_q8_32(g["x4"])
    assert xq[0] == 127 and xq[1] == 0 and xq[2] == 2 and xq[3] == 2  # 0.5->0, 1.5->2, 2.5->2
    xq, xs = oracle.quantize_q8_32(np.zeros(64, np.float32))
    assert not xq.any() and not xs.any()


def test_q4k_integer_sums_pinned(oracle):
    g = golden_npz("q4k.npz")
    for t in range(g["pin_blocks"].shape[0]):
        iqx, ix = oracle.q4k_subsums(g["pin_blocks"][t], 1, 256, g["pin_xq"][t])
        assert np.array_equal(iqx, g["pin_iqx"][t])
        assert np.array_equal(ix, g["pin_ix"][t])


def test_q4k_dot_golden(oracle):
    g = golden_npz("q4k.npz")
    w, xq, xs = g["w"], g["xq"], g["xs"]
    rb = 8 * 144
    ours = np.array([oracle.L.orc_q4k_dot(w[r * rb:].ctypes.data, 2048, xq.ctypes.data, xs.ctypes.data)
                     for r in range(8)], np.float32)
    assert np.array_equal(ours.view(np.uint32), g["dots"].view(np.uint32))


def test_dequant_golden_bit_exact(oracle):
    g = golden_npz("dequant.npz")
    assert np.array_equal(oracle.dequant(g["w4"], 12, 4096), g["d4"])
    assert np.array_equal(oracle.dequant(g["w6"], 14, 4096), g["d6"])


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_ops_golden(oracle):
    g = golden_npz("ops.npz")
    assert np.array_equal(bits(oracle.rmsnorm(g["x"], g["w"], 1e-6)), bits(g["rms"]))
    for pos in (0, 1, 17, 511, 4095):
        assert np.array_equal(bits(oracle.rope(g["q"], 128, pos, 1e6)), bits(g[f"rope{pos}"])), pos


def test_libm_restatements_pinned(oracle):
    """glibc's scalar expf, libmvec's 8- and 4-wide expf and the host's
    rsqrtss, restated, against the host libraries on a strided sweep of all
    float bit patterns (the full sweep agrees too; it takes minutes)."""
    out = (C.c_longlong * 4)()
    oracle.L.orc_check_libm.restype = None
    oracle.L.orc_check_libm.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32, C.c_void_p]
    oracle.L.orc_check_libm(0, 0xFFFFFFFF, 4093, out)
    assert list(out) == [0, 0, 0, 0]
    # the softmax and silu ranges densely
    for lo, hi in ((0xBF800000, 0xC2B00000), (0x00000000, 0x3F800000)):
        oracle.L.orc_check_libm(lo, hi, 61, out)
        assert list(out) == [0, 0, 0, 0], hex(lo)


def test_synth_deterministic():
    fx = golden_json("tiny.json")
    path = synth.cached_model(synth.PRESETS["tiny"])
    assert os.path.getsize(path) == fx["bytes"]
    assert synth.file_sha256(path) == fx["sha256"]


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_oracle_model_stream(name):
    """The restated forward reproduces the reference's greedy stream and its
    logged logits exactly."""
    from oracle.oracle import OracleModel
    fx = golden_json(f"{name}.json")
    path = synth.cached_model(synth.PRESETS[name])
    m = OracleModel(path, 256)
    for i, rec in enumerate(fx["logits"]):
        lg = m.forward(fx["prompt"][i])
        assert lg[:8].tolist() == rec["first8"], i
        assert int(np.argmax(lg)) == rec["argmax"]
    m.reset()
    lg = None
    for t in fx["prompt"]:
        lg = m.forward(t)
    toks = []
    for _ in range(fx["n_gen"]):
        t = int(np.argmax(lg))
        toks.append(t)
        lg = m.forward(t)
    m.close()
    assert first_divergence(toks, fx["tokens"]) is None


@pytest.mark.skipif(not have_reference(), reason="reference build absent")
@pytest.mark.parametrize("name,steps", [("tiny", 40), ("small", 24)])
def test_oracle_forward_bit_exact(name, steps):
    """Logits and hidden state of every step identical to the reference's
    own hakm_forward, token fed back greedily."""
    from oracle.oracle import OracleModel, RefModel
    path = synth.cached_model(synth.PRESETS[name])
    om, rm = OracleModel(path, 256), RefModel(path, 256)
    tok = 7
    for step in range(steps):
        a = om.forward(tok)
        b, am = rm.forward(tok)
        assert np.array_equal(bits(a), bits(b)), step
        assert np.array_equal(bits(om.hidden()), bits(rm.hidden())), step
        tok = am
    om.close()


@pytest.mark.skipif(not have_reference(), reason="reference build absent")
def test_oracle_nn_ops_bit_exact(oracle, reference):
    """rmsnorm, softmax, silu and rope at every remainder of the 8-lane
    split, against the reference's compiled functions."""
    rng = np.random.default_rng(5)
    for n in list(range(1, 40)) + [256, 2048, 3584, 4097]:
        x = (rng.standard_normal(n) * rng.uniform(0.01, 10)).astype(np.float32)
        w = rng.uniform(0.5, 1.5, n).astype(np.float32)
        assert np.array_equal(bits(oracle.rmsnorm(x, w, 1e-6)), bits(reference.rmsnorm(x, w, 1e-6))), n
        a, b = x.copy(), x.copy()
        oracle.L.orc_softmax(a.ctypes.data, n)
        reference.L.softmax(b.ctypes.data, n)
        assert np.array_equal(bits(a), bits(b)), n
    oracle.L.orc_silu.restype, oracle.L.orc_silu.argtypes = C.c_float, [C.c_float]
    for v in (rng.standard_normal(2000) * 12).astype(np.float32):
        assert bits(oracle.L.orc_silu(float(v))) == bits(reference.L.silu_f(float(v)))
    for hd in (16, 64, 128, 8):
        for pos in (0, 3, 100, 4095, 32767):
            q = rng.standard_normal(hd * 2).astype(np.float32)
            assert np.array_equal(bits(oracle.rope(q, hd, pos, 1e6)), bits(reference.rope(q, hd, pos, 1e6)))


@pytest.mark.skipif(not have_reference(), reason="reference build absent")
def test_oracle_vs_reference_random(oracle, reference):
    rng = np.random.default_rng(99)
    for rows, k in [(16, 256), (64, 2048), (8, 11008), (4, 18944), (8, 3584)]:
        x = (rng.standard_normal(k) * rng.uniform(0.01, 10)).astype(np.float32)
        xq_o, xs_o = oracle.quantize_q8_32(x)
        xq_r, xs_r = reference.quantize_q8_32(x)
        assert np.array_equal(xq_o, xq_r) and np.array_equal(xs_o, xs_r)
        w4 = synth.random_q4k(rows, k, int(rng.integers(1 << 30)))
        w6 = synth.random_q6k(rows, k, int(rng.integers(1 << 30)))
        b = rng.standard_normal(rows).astype(np.float32)
        for w, t in ((w4, 12), (w6, 14)):
            assert np.array_equal(bits(oracle.matmul(w, t, x, rows, k, b)), bits(reference.matmul(w, t, x, rows, k, b)))
        assert np.array_equal(oracle.dequant(w4, 12, rows * k), reference.dequant(w4, 12, rows * k))
        assert np.array_equal(oracle.dequant(w6, 14, rows * k), reference.dequant(w6, 14, rows * k))


def test_synth_quantizers_roundtrip(oracle):
    """The synthetic RTN quantizers produce blocks that decode (with the
    restated dequant) close to their inputs."""
    import ctypes as C
    lib = synth.lib()
    x = synth.normal(256 * 16, 5, 0.02)
    b4 = np.zeros(16 * 144, np.uint8)
    b6 = np.zeros(16 * 210, np.uint8)
    for i in range(16):
        lib.synth_quantize_q4k_block(C.c_void_p(x[256 * i:].ctypes.data), C.c_void_p(b4[144 * i:].ctypes.data))
        lib.synth_quantize_q6k_block(C.c_void_p(x[256 * i:].ctypes.data), C.c_void_p(b6[210 * i:].ctypes.data))
    assert rel_l2(oracle.dequant(b4, 12, x.size), x) < 0.12
    assert rel_l2(oracle.dequant(b6, 14, x.size), x) < 0.03


def special_q8_blocks():
    """Blocks whose scale path leaves the normal range: 127/amax overflows
    (amax below 2^-121), infinities, NaN, FLT_MAX, subnormals."""
    rng = np.random.default_rng(11)
    blocks = []
    for amax in (1e-38, 3e-37, 4e-37, 1e-30, 3.4e38):
        b = rng.uniform(-1, 1, 32).astype(np.float32) * np.float32(amax)
        b[3] = np.float32(amax)
        blocks.append(b)
    b = rng.standard_normal(32).astype(np.float32); b[5] = np.inf; blocks.append(b)
    b = rng.standard_normal(32).astype(np.float32); b[7] = -np.inf; b[8] = np.inf; blocks.append(b)
    b = rng.standard_normal(32).astype(np.float32); b[9] = np.nan; blocks.append(b)
    b = np.full(32, np.nan, np.float32); blocks.append(b)
    b = np.full(32, 1e-45, np.float32); b[::2] = -1e-45; blocks.append(b)
    return np.concatenate(blocks).astype(np.float32)


def test_q8_special_values_match_reference(oracle, reference):
    x = special_q8_blocks()
    oq, os_ = oracle.quantize_q8_32(x)
    rq, rs = reference.quantize_q8_32(x)
    assert np.array_equal(oq, rq)
    assert np.array_equal(os_.view(np.uint32), rs.view(np.uint32))
