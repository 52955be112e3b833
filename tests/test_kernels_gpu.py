"""Kernel-level parity through the C ABI on the GPU.

Every kernel restates the reference build's roundings (gcc -O3 -ffast-math
for x86-64-v3: lane orders, fused multiply-adds, rsqrtss, glibc / libmvec
exp), so the bar is bit identity with the reference's compiled functions
(or, for attention, which the reference has no function for, with the
oracle's restatement that the whole-forward tests pin): the int8 quantizer,
Q4_K integer sub-block sums, dequantization, Q4_K and Q6_K matmuls with
bias (one vector, and many rows at once), the fused lm_head + first-index
greedy pick, rmsnorm, RoPE, attention (one vector, and prompt / decode rows),
and the device's exp routines against the host's libm / libmvec."""
import ctypes as C

import numpy as np
import pytest

from conftest import golden_npz, rel_l2
from hako_b200 import check, lib, synth

pytestmark = pytest.mark.gpu

TOL = 1e-5


def same(a, b):
    return np.array_equal(np.ascontiguousarray(a, np.float32).view(np.uint32),
                          np.ascontiguousarray(b, np.float32).view(np.uint32))


def P(t):
    return C.c_void_p(t.data_ptr())


_KEEP = []


@pytest.fixture(autouse=True)
def _keep_alive():
    """Device copies made inline (P(dev(...))) must outlive the launch: the
    caching allocator would otherwise hand their memory to the next copy."""
    yield
    sync()
    _KEEP.clear()


def dev(a, cuda):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    _KEEP.append(t)
    return t


def sync():
    import torch
    torch.cuda.synchronize()


def empty(shape, dtype, cuda):
    import torch
    return torch.empty(shape, dtype=dtype, device=cuda)


def packed_q6k(w, rows, k, cuda):
    """Upload verbatim Q6_K rows and re-lay them with hakmc_q6k_pack."""
    import torch
    src = dev(w, cuda)
    dst = torch.empty(lib.hakmc_q6k_packed_bytes(rows, k), dtype=torch.uint8, device=cuda)
    _KEEP.append(dst)
    check(lib.hakmc_q6k_pack(P(dst), P(src), rows, k, None))
    return dst


def test_quantize_golden_bit_exact(cuda):
    import torch
    g = golden_npz("q8.npz")
    for i in range(len([k for k in g.files if k.startswith("xq")])):
        x = g[f"x{i}"]
        xq = empty(x.size, torch.int8, cuda)
        xs = empty(x.size // 32, torch.float32, cuda)
        check(lib.hakmc_quantize_q8_32(P(dev(x, cuda)), x.size, P(xq), P(xs), None))
        sync()
        assert np.array_equal(xq.cpu().numpy(), g[f"xq{i}"]), i
        assert np.array_equal(xs.cpu().numpy().view(np.uint32), g[f"xs{i}"].view(np.uint32)), i


def test_quantize_random_bit_exact(cuda, reference):
    import torch
    rng = np.random.default_rng(5)
    for n in (32, 2048, 11008, 18944):
        x = (rng.standard_normal(n) * rng.uniform(1e-4, 1e3)).astype(np.float32)
        xq = empty(n, torch.int8, cuda)
        xs = empty(n // 32, torch.float32, cuda)
        check(lib.hakmc_quantize_q8_32(P(dev(x, cuda)), n, P(xq), P(xs), None))
        sync()
        rq, rs = reference.quantize_q8_32(x)
        assert np.array_equal(xq.cpu().numpy(), rq) and np.array_equal(xs.cpu().numpy(), rs)


def test_quantize_special_values_bit_exact(cuda, reference):
    import torch
    from test_oracle import special_q8_blocks
    x = special_q8_blocks()
    xq = empty(x.size, torch.int8, cuda)
    xs = empty(x.size // 32, torch.float32, cuda)
    check(lib.hakmc_quantize_q8_32(P(dev(x, cuda)), x.size, P(xq), P(xs), None))
    sync()
    rq, rs = reference.quantize_q8_32(x)
    assert np.array_equal(xq.cpu().numpy(), rq)
    assert np.array_equal(xs.cpu().numpy().view(np.uint32), rs.view(np.uint32))


def test_q4k_integer_sums_pinned(cuda):
    import torch
    g = golden_npz("q4k.npz")
    for t in range(g["pin_blocks"].shape[0]):
        iqx = empty(8, torch.int32, cuda)
        ix = empty(8, torch.int32, cuda)
        check(lib.hakmc_q4k_subsums(P(iqx), P(ix), P(dev(g["pin_blocks"][t], cuda)),
                                    P(dev(g["pin_xq"][t], cuda)), 1, 256, None))
        sync()
        assert np.array_equal(iqx.cpu().numpy(), g["pin_iqx"][t])
        assert np.array_equal(ix.cpu().numpy(), g["pin_ix"][t])


@pytest.mark.parametrize("rows,k", [(256, 2048), (2048, 2048), (11008, 2048), (2048, 11008),
                                    (3584, 3584), (512, 3584), (18944, 3584), (3584, 18944)])
def test_q4k_subsums_bit_exact(cuda, oracle, rows, k):
    import torch
    w = synth.random_q4k(rows, k, rows + k)
    x = synth.normal(k, k)
    xq, xs = oracle.quantize_q8_32(x)
    sub = min(rows, 64)
    iqx = empty(sub * k // 32, torch.int32, cuda)
    ix = torch.empty_like(iqx)
    check(lib.hakmc_q4k_subsums(P(iqx), P(ix), P(dev(w, cuda)), P(dev(xq, cuda)), sub, k, None))
    sync()
    oi, ox = oracle.q4k_subsums(w, sub, k, xq)
    assert np.array_equal(iqx.cpu().numpy(), oi) and np.array_equal(ix.cpu().numpy(), ox)


@pytest.mark.parametrize("rows,k", [(256, 2048), (2048, 2048), (11008, 2048), (2048, 11008),
                                    (512, 3584), (18944, 3584), (3584, 18944), (4, 256), (3, 512)])
def test_gemv_q4k_matches_reference(cuda, reference, rows, k):
    import torch
    w = synth.random_q4k(rows, k, 3 * rows + k)
    x = synth.normal(k, k + 1)
    out = empty(rows, torch.float32, cuda)
    check(lib.hakmc_gemv_q4k(P(out), P(dev(w, cuda)), P(dev(x, cuda)), None, rows, k, None))
    sync()
    assert same(out.cpu().numpy(), reference.matmul(w, 12, x, rows, k))
    # pre-quantized activation entry point, with bias
    xq, xs = reference.quantize_q8_32(x)
    b = synth.normal(rows, 77)
    check(lib.hakmc_gemv_q4k_q8(P(out), P(dev(w, cuda)), P(dev(xq, cuda)), P(dev(xs, cuda)),
                                P(dev(b, cuda)), rows, k, None))
    sync()
    assert same(out.cpu().numpy(), reference.matmul(w, 12, x, rows, k, bias=b))


def test_gemv_q4k_golden_dots(cuda):
    import torch
    g = golden_npz("q4k.npz")
    out = empty(8, torch.float32, cuda)
    check(lib.hakmc_gemv_q4k_q8(P(out), P(dev(g["w"], cuda)), P(dev(g["xq"], cuda)), P(dev(g["xs"], cuda)),
                                None, 8, 2048, None))
    sync()
    assert same(out.cpu().numpy(), g["dots"])


@pytest.mark.parametrize("rows,k", [(256, 2048), (2048, 2048), (2048, 11008), (512, 3584),
                                    (3584, 18944), (151936, 2048), (5, 256)])
def test_gemv_q6k_matches_reference(cuda, reference, rows, k):
    import torch
    w = synth.random_q6k(rows, k, 5 * rows + k)
    x = synth.normal(k, k + 2)
    packed = packed_q6k(w, rows, k, cuda)
    out = empty(rows, torch.float32, cuda)
    b = synth.normal(rows, 78)
    check(lib.hakmc_gemv_q6k(P(out), P(packed), P(dev(x, cuda)), P(dev(b, cuda)), rows, k, None))
    sync()
    assert same(out.cpu().numpy(), reference.matmul(w, 14, x, rows, k, bias=b))


def test_dequant_bit_exact(cuda):
    import torch
    g = golden_npz("dequant.npz")
    for key, t, ref in (("w4", 12, "d4"), ("w6", 14, "d6")):
        out = empty(4096, torch.float32, cuda)
        check(lib.hakmc_dequant(P(out), P(dev(g[key], cuda)), t, 4, 1024, None))
        sync()
        assert np.array_equal(out.cpu().numpy(), g[ref])


@pytest.mark.parametrize("vocab,k", [(151936, 2048), (152064, 3584), (1000, 256)])
def test_lmhead_argmax(cuda, reference, vocab, k):
    import torch
    w = synth.random_q6k(vocab, k, vocab)
    x = synth.normal(k, 3)
    nw = (1 + 0.1 * synth.normal(k, 4)).astype(np.float32)
    packed = packed_q6k(w, vocab, k, cuda)
    lg = empty(vocab, torch.float32, cuda)
    am = torch.zeros(1, dtype=torch.int32, device=cuda)
    check(lib.hakmc_lmhead_argmax(P(lg), P(am), P(packed), P(dev(x, cuda)), P(dev(nw, cuda)), 1e-6,
                                  vocab, k, None))
    sync()
    ref = reference.matmul(w, 14, reference.rmsnorm(x, nw, 1e-6), vocab, k)
    assert same(lg.cpu().numpy(), ref)
    assert int(am.item()) == int(np.argmax(ref))


def test_lmhead_argmax_ties_pick_first(cuda):
    """Duplicate rows give equal logits: the lowest index wins, as with the
    reference's strict '>' scan (src/sample.c:30)."""
    import torch
    k, vocab = 256, 4096
    w = synth.random_q6k(vocab, k, 9)
    row = w[:210].copy()
    for r in (17, 1000, 4000):  # three copies of the same row
        w[r * 210:(r + 1) * 210] = row
    # make that row the clear maximum: large positive d, positive scales
    x = np.ones(k, np.float32)
    for r in (0, 17, 1000, 4000):
        w[r * 210 + 192:r * 210 + 208] = 31
        w[r * 210:r * 210 + 192] = 0xFF  # q = 63 -> +31
        w[r * 210 + 208:r * 210 + 210] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
    packed = packed_q6k(w, vocab, k, cuda)
    am = torch.zeros(1, dtype=torch.int32, device=cuda)
    check(lib.hakmc_lmhead_argmax(None, P(am), P(packed), P(dev(x, cuda)), None, 1e-6, vocab, k, None))
    sync()
    assert int(am.item()) == 0


def test_rmsnorm(cuda):
    import torch
    g = golden_npz("ops.npz")
    y = empty(2048, torch.float32, cuda)
    check(lib.hakmc_rmsnorm(P(y), P(dev(g["x"], cuda)), P(dev(g["w"], cuda)), 2048, 1e-6, None))
    sync()
    assert same(y.cpu().numpy(), g["rms"])


@pytest.mark.parametrize("n", [8, 256, 2048, 3584, 11008])
def test_rmsnorm_random_bit_exact(cuda, reference, n):
    import torch
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * rng.uniform(1e-3, 1e2)).astype(np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    y = empty(n, torch.float32, cuda)
    check(lib.hakmc_rmsnorm(P(y), P(dev(x, cuda)), P(dev(w, cuda)), n, 1e-6, None))
    sync()
    assert same(y.cpu().numpy(), reference.rmsnorm(x, w, 1e-6))


@pytest.mark.parametrize("pos", [0, 1, 17, 511, 4095])
def test_rope(cuda, pos):
    g = golden_npz("ops.npz")
    q = dev(g["q"], cuda)
    check(lib.hakmc_rope_neox(P(q), 16, 128, pos, 1e6, None))
    sync()
    assert same(q.cpu().numpy(), g[f"rope{pos}"])


@pytest.mark.parametrize("hd,pos", [(64, 3), (64, 30000), (128, 100000)])
def test_rope_random_bit_exact(cuda, reference, hd, pos):
    q = synth.normal(4 * hd, hd + pos)
    d = dev(q, cuda)
    check(lib.hakmc_rope_neox(P(d), 4, hd, pos, 1e6, None))
    sync()
    assert same(d.cpu().numpy(), reference.rope(q, hd, pos, 1e6))


@pytest.mark.parametrize("H,KVH,hd,pos", [(16, 2, 128, 0), (16, 2, 128, 6), (16, 2, 128, 11), (16, 2, 128, 63),
                                          (16, 2, 128, 255), (16, 2, 128, 256), (28, 4, 128, 1000),
                                          (28, 4, 128, 4095), (4, 2, 64, 300), (4, 2, 64, 2)])
def test_attention(cuda, oracle, H, KVH, hd, pos):
    """Against the oracle's restatement of src/model.c:124-142 (pinned to the
    reference by the whole-forward oracle tests): positions below 8, at 4..7
    past a multiple of 8, and long caches."""
    import torch
    rng = np.random.default_rng(pos + H)
    max_seq = pos + 1
    q = (rng.standard_normal(H * hd) * 2).astype(np.float32)
    kc = rng.standard_normal((max_seq, KVH * hd)).astype(np.float32)
    vc = rng.standard_normal((max_seq, KVH * hd)).astype(np.float32)
    out = empty(H * hd, torch.float32, cuda)
    check(lib.hakmc_attention(P(out), P(dev(q, cuda)), P(dev(kc, cuda)), P(dev(vc, cuda)), pos, H, KVH, hd, None))
    sync()
    assert same(out.cpu().numpy(), oracle.attention(q, kc, vc, pos, H, KVH, hd))


@pytest.mark.parametrize("H,KVH,hd,pos0,rows", [(16, 2, 128, 0, 40), (28, 4, 128, 300, 17), (8, 2, 64, 5, 3),
                                                (4, 2, 64, 0, 1)])
def test_attention_rows_prompt(cuda, oracle, H, KVH, hd, pos0, rows):
    """hakmc_attention_rows over a prompt chunk (row r at position pos0 + r
    of one cache): every row equals the oracle's attention at its position."""
    import torch
    rng = np.random.default_rng(pos0 + rows)
    n = pos0 + rows
    q = rng.standard_normal((rows, H * hd)).astype(np.float32)
    kc = rng.standard_normal((n, KVH * hd)).astype(np.float32)
    vc = rng.standard_normal((n, KVH * hd)).astype(np.float32)
    out = empty((rows, H * hd), torch.float32, cuda)
    check(lib.hakmc_attention_rows(P(out), P(dev(q, cuda)), P(dev(kc, cuda)), P(dev(vc, cuda)), rows, pos0, None,
                                   n - 1, 0, H, KVH, hd, None))
    sync()
    got = out.cpu().numpy()
    for r in range(rows):
        assert same(got[r], oracle.attention(q[r], kc, vc, pos0 + r, H, KVH, hd)), r


@pytest.mark.parametrize("H,KVH,hd,cap", [(28, 4, 128, 1100), (16, 2, 128, 9000), (8, 2, 64, 300)])
def test_attention_rows_decode(cuda, oracle, H, KVH, hd, cap):
    """Decode rows: row r reads its own cache slot up to its own position
    (ragged positions, around multiples of 8 and of the 8-wide exp split).
    Up to ~6,000 positions a CTA serves all query heads of a kv head; the
    9,000-position case takes the one-head-per-CTA kernel."""
    import torch
    pos = sorted({min(p, cap - 1) for p in (0, 3, 7, 8, 12, 255, 256, 1000, 1027, cap - 1)})
    rows = len(pos)
    rng = np.random.default_rng(11)
    q = rng.standard_normal((rows, H * hd)).astype(np.float32)
    kc = rng.standard_normal((rows, cap, KVH * hd)).astype(np.float32)
    vc = rng.standard_normal((rows, cap, KVH * hd)).astype(np.float32)
    out = empty((rows, H * hd), torch.float32, cuda)
    rp = dev(np.array(pos, np.int32), cuda)
    check(lib.hakmc_attention_rows(P(out), P(dev(q, cuda)), P(dev(kc, cuda)), P(dev(vc, cuda)), rows, 0, P(rp),
                                   max(pos), cap * KVH * hd, H, KVH, hd, None))
    sync()
    got = out.cpu().numpy()
    for r in range(rows):
        assert same(got[r], oracle.attention(q[r], kc[r], vc[r], pos[r], H, KVH, hd)), r


def test_attention_rows_rejects_long_rows(cuda):
    import torch
    buf = empty(1 << 10, torch.float32, cuda)
    assert lib.hakmc_attention_rows(P(buf), P(buf), P(buf), P(buf), 1, 0, None, 60000, 0, 16, 2, 128, None) < 0
    assert lib.hakmc_attention_rows(P(buf), P(buf), P(buf), P(buf), 1, 0, None, 10, 0, 16, 3, 128, None) < 0


@pytest.mark.parametrize("rows,k,n", [(256, 2048, 9), (2048, 11008, 64), (3584, 18944, 17), (512, 3584, 1),
                                      (151936, 2048, 4), (5, 256, 33), (100, 2304, 40)])
def test_gemm_q6k_matches_reference(cuda, reference, rows, k, n):
    """hakmc_gemm_q6k: every output row of every activation equals the
    reference's Q6_K matmul (src/nn.c:84-95 as built) bit for bit; with
    accumulate, out + that value (one IEEE add)."""
    import torch
    w = synth.random_q6k(rows, k, 3 * rows + k + n)
    packed = packed_q6k(w, rows, k, cuda)
    x = np.stack([synth.normal(k, 300 + i) for i in range(n)])
    b = synth.normal(rows, 79) if n % 2 else None
    base = np.random.default_rng(n).standard_normal((n, rows)).astype(np.float32)
    out = dev(base, cuda)
    acc = n % 3 == 0
    check(lib.hakmc_gemm_q6k(P(out), P(packed), P(dev(x, cuda)), P(dev(b, cuda)) if b is not None else None, rows, k,
                             n, int(acc), None))
    sync()
    got = out.cpu().numpy()
    for i in range(n):
        want = reference.matmul(w, 14, x[i], rows, k, bias=b)
        if acc:
            want = (base[i] + want).astype(np.float32)
        assert same(got[i], want), i


def test_device_exp_matches_host_libm(cuda, oracle):
    """The device's glibc scalar expf and libmvec 8- / 4-wide expf against the
    oracle's restatements (which tests/test_oracle.py pins against the host
    libraries): a strided sweep of every float bit pattern plus the dense
    softmax range [-88, 0]."""
    import torch
    u = np.concatenate([np.arange(0, 1 << 32, 1021, dtype=np.uint64),
                        np.arange(0xBF800000, 0xC2B00000, 97, dtype=np.uint64),
                        np.arange(0x00000000, 0x3F800000, 97, dtype=np.uint64)]).astype(np.uint32)
    x = u.view(np.float32)
    x = x[~np.isnan(x)]
    dx = dev(x, cuda)
    out = empty(x.size, torch.float32, cuda)
    for variant, fn in ((0, oracle.L.orc_expf), (1, oracle.L.orc_expf_v8), (2, oracle.L.orc_expf_v4)):
        check(lib.hakmc_test_expf(P(out), P(dx), x.size, variant, None))
        sync()
        got = out.cpu().numpy()
        idx = np.random.default_rng(variant).choice(x.size, 200000, replace=False)
        want = np.array([fn(float(v)) for v in x[idx]], np.float32)
        assert same(got[idx], want), variant
