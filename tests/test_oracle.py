"""Pins the CPU oracle against the reference engine's own outputs (golden
vectors made by tests/golden/make_golden.py from oracle/_ref) and, when the
reference build is present, against it directly on fresh random inputs."""
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
    assert rel_l2(ours, g["dots"]) < 1e-6


def test_dequant_golden_bit_exact(oracle):
    g = golden_npz("dequant.npz")
    assert np.array_equal(oracle.dequant(g["w4"], 12, 4096), g["d4"])
    assert np.array_equal(oracle.dequant(g["w6"], 14, 4096), g["d6"])


def test_ops_golden(oracle):
    g = golden_npz("ops.npz")
    assert rel_l2(oracle.rmsnorm(g["x"], g["w"], 1e-6), g["rms"]) < 1e-6
    for pos in (0, 1, 17, 511, 4095):
        # the reference vectorizes powf/cosf/sinf through glibc's libmvec; the
        # restatement calls scalar libm: a few ulp of the angle pos*freq apart
        tol = 2e-6 + 1e-7 * pos
        assert np.abs(oracle.rope(g["q"], 128, pos, 1e6) - g[f"rope{pos}"]).max() < tol, pos


def test_synth_deterministic():
    fx = golden_json("tiny.json")
    path = synth.cached_model(synth.PRESETS["tiny"])
    assert os.path.getsize(path) == fx["bytes"]
    assert synth.file_sha256(path) == fx["sha256"]


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_oracle_model_stream(name):
    """The restated forward reproduces the reference's greedy stream up to
    the first step whose reference top1-top2 margin is inside the int8
    rounding-flip noise of two fp32 summation orders."""
    from oracle.oracle import OracleModel
    fx = golden_json(f"{name}.json")
    path = synth.cached_model(synth.PRESETS[name])
    m = OracleModel(path, 256)
    lg = None
    for t in fx["prompt"]:
        lg = m.forward(t)
    toks = []
    for _ in range(fx["n_gen"]):
        t = int(np.argmax(lg))
        toks.append(t)
        lg = m.forward(t)
    m.close()
    i = first_divergence(toks, fx["tokens"])
    assert i is None or fx["gaps"][i] < 2e-2, f"diverged at {i} with margin {fx['gaps'][i]}"


@pytest.mark.skipif(not have_reference(), reason="reference build absent")
def test_oracle_vs_reference_random(oracle, reference):
    rng = np.random.default_rng(99)
    for rows, k in [(16, 256), (64, 2048), (8, 11008)]:
        x = (rng.standard_normal(k) * rng.uniform(0.01, 10)).astype(np.float32)
        xq_o, xs_o = oracle.quantize_q8_32(x)
        xq_r, xs_r = reference.quantize_q8_32(x)
        assert np.array_equal(xq_o, xq_r) and np.array_equal(xs_o, xs_r)
        w4 = synth.random_q4k(rows, k, int(rng.integers(1 << 30)))
        w6 = synth.random_q6k(rows, k, int(rng.integers(1 << 30)))
        assert rel_l2(oracle.matmul(w4, 12, x, rows, k), reference.matmul(w4, 12, x, rows, k)) < 1e-5
        assert rel_l2(oracle.matmul(w6, 14, x, rows, k), reference.matmul(w6, 14, x, rows, k)) < 1e-5
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
