"""Whole-model parity on the GPU against the reference engine's own compiled
forward pass (oracle/_ref) and the golden streams it produced.

Every path restates the reference build's roundings and orders, so every
test holds to bit identity: the single-sequence decode path (the persistent
step kernel behind hakmc_forward / hakmc_prefill / hakmc_generate /
hakmc_decode, and the per-phase kernels behind HAKMC_STEP=0) and the
row-batched passes (hakmc_prefill_batched, hakmc_forward_batch with eight or
more rows) give logits, hidden states, K/V and greedy streams equal to the
reference's bit for bit."""
import os

import numpy as np
import pytest

from conftest import first_divergence, golden_json, rel_l2
from hako_b200 import HakmCtx, HakmcError, synth

pytestmark = pytest.mark.gpu

def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def same(a, b):
    return np.array_equal(bits(a), bits(b))


@pytest.fixture(scope="module")
def tiny_path():
    return synth.cached_model(synth.PRESETS["tiny"])


@pytest.fixture(scope="module")
def small_path():
    return synth.cached_model(synth.PRESETS["small"])


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_greedy_stream_matches_golden(cuda, name):
    fx = golden_json(f"{name}.json")
    path = synth.cached_model(synth.PRESETS[name])
    assert synth.file_sha256(path) == fx["sha256"]
    with HakmCtx(path, max_seq=256) as ctx:
        toks = ctx.generate(fx["prompt"], fx["n_gen"])
        assert toks == fx["tokens"]
        # generate is deterministic and reset restarts the sequence
        ctx.reset()
        assert ctx.generate(fx["prompt"], fx["n_gen"]) == toks
        # the per-token API gives the same stream as the device-side loop
        ctx.reset()
        am = None
        for i, t in enumerate(fx["prompt"]):
            lg, am = ctx.forward(t, want_logits=True)
            if i < len(fx.get("logits", [])):
                assert lg[:8].tolist() == fx["logits"][i]["first8"], i
        step = []
        for _ in range(fx["n_gen"]):
            step.append(am)
            _, am = ctx.forward(am, want_logits=False)
        assert step == toks


@pytest.mark.parametrize("name,steps", [("tiny", 24), ("small", 24), ("mid", 16)])
def test_logits_match_reference(cuda, reference, name, steps):
    """Every step's logits and greedy pick equal the reference's, bit for
    bit, the pick fed back."""
    from oracle.oracle import RefModel
    path = synth.cached_model(synth.PRESETS[name])
    ref = RefModel(path, 256)
    with HakmCtx(path, max_seq=256) as ctx:
        tok = 5
        for i in range(steps):
            a, am_r = ref.forward(tok)
            b, am_g = ctx.forward(tok)
            assert same(b, a), (i, rel_l2(b, a))
            assert am_g == am_r
            tok = am_r
    ref.close()


def test_per_phase_path_matches_reference(cuda, reference, small_path, monkeypatch):
    """HAKMC_STEP=0: one kernel per phase (CUDA graph per step) instead of
    the persistent step kernel; same bits."""
    from oracle.oracle import RefModel
    monkeypatch.setenv("HAKMC_STEP", "0")
    ref = RefModel(small_path, 64)
    with HakmCtx(small_path, max_seq=64) as ctx:
        tok = 9
        for i in range(12):
            a, am_r = ref.forward(tok)
            b, am_g = ctx.forward(tok)
            assert same(b, a), (i, rel_l2(b, a))
            assert am_g == am_r
            tok = am_r
    ref.close()


def test_layer_outputs(cuda, reference, small_path):
    """Residual streams after n = 0..L layers (0: the embedding row, deq_row
    src/nn.c:55-59), over 8 positions: identical to the reference's."""
    from oracle.oracle import RefModel
    toks = [11, 4000, 256, 259, 1, 2, 3, 77]
    cfg = synth.PRESETS["small"]
    for n in range(0, cfg.n_layers + 1):
        ref = RefModel(small_path, 64)
        ref.set_layers(n)
        with HakmCtx(small_path, max_seq=64) as ctx:
            ctx.set_layers(n)
            for t in toks:
                ref.forward(t, want_logits=False)
                ctx.forward(t, want_logits=False)
                assert same(ctx.hidden(), ref.hidden()), (n, t, rel_l2(ctx.hidden(), ref.hidden()))
        ref.close()


@pytest.mark.parametrize("name", ["3b", "7b"])
def test_embedding_rows_bit_exact(cuda, reference, name):
    """Q6_K token_embd rows (deq_row, src/nn.c:55-59) of both vocab sizes,
    first, last and random ids: identical to the reference's."""
    from oracle.oracle import RefModel
    cfg = synth.PRESETS[name]
    path = synth.cached_model(cfg)
    rng = np.random.default_rng(17)
    ids = [0, 1, cfg.vocab - 1, cfg.vocab // 2] + rng.integers(0, cfg.vocab, 4).tolist()
    ref = RefModel(path, 16)
    ref.set_layers(0)
    with HakmCtx(path, max_seq=16) as ctx:
        ctx.set_layers(0)
        for t in ids:
            ref.reset()
            ctx.reset()
            ref.forward(int(t), want_logits=False)
            ctx.forward(int(t), want_logits=False)
            assert same(ctx.hidden(), ref.hidden()), t
    ref.close()


def test_long_context_attention(cuda, reference, small_path):
    """700 positions (eleven V tiles of the attention kernel): the last
    step's logits identical to the reference's."""
    from oracle.oracle import RefModel
    cfg = synth.PRESETS["small"]
    n = 700  # ffn 1536 > 700: inside the reference's scores-buffer limit
    assert n < cfg.ffn_dim
    toks = [(7 * i + 3) % 4000 for i in range(n)]
    ref = RefModel(small_path, 1024)
    with HakmCtx(small_path, max_seq=1024) as ctx:
        for t in toks[:-1]:
            ref.forward(t, want_logits=False)
            ctx.forward(t, want_logits=False)
        a, _ = ref.forward(toks[-1])
        b, _ = ctx.forward(toks[-1])
    ref.close()
    assert same(b, a), rel_l2(b, a)


def test_position_limits(cuda, tiny_path):
    with HakmCtx(tiny_path, max_seq=4) as ctx:
        for t in (1, 2, 3, 4):
            ctx.forward(t, want_logits=False)
        assert ctx.pos == 4
        with pytest.raises(HakmcError):
            ctx.forward(5, want_logits=False)
        with pytest.raises(HakmcError):
            ctx.generate([1], 2)
        ctx.reset()
        assert ctx.pos == 0
        ctx.forward(1, want_logits=False)
        with pytest.raises(HakmcError):
            ctx.forward(10 ** 6, want_logits=False)  # token out of range


def test_fill_kv_matches_prefill(cuda, reference, small_path):
    """A cache pre-filled with the reference's own K/V (hakm_ctx.k_cache /
    v_cache / pos, src/model.h:20-21), then one decode step, matches the
    reference's step on that cache bit for bit."""
    from oracle.oracle import RefModel
    cfg = synth.PRESETS["small"]
    toks = [11, 4000, 256, 259, 1, 2, 3, 77, 500]
    ref = RefModel(small_path, 64)
    for t in toks[:-1]:
        ref.forward(t, want_logits=False)
    k, v = ref.read_kv(cfg.n_layers, cfg.kv_dim, len(toks) - 1)
    a, am_r = ref.forward(toks[-1])
    ref.close()
    with HakmCtx(small_path, max_seq=64) as ctx:
        ctx.fill_kv(k, v, seq=0)
        assert ctx.pos == len(toks) - 1
        b, am_g = ctx.forward(toks[-1])
        assert ctx.pos == len(toks)
    assert same(b, a)
    assert am_g == am_r


@pytest.mark.parametrize("name,max_seq", [("3b", 128), ("7b", 256)])
def test_big_model_stream(cuda, name, max_seq):
    """Config 0 (3B: 16 seeded prompt ids, 64 greedy tokens) and config 3
    (7B: 32 ids, 128 tokens): the whole stream equals the golden stream of
    the reference build."""
    fx = golden_json(f"{name}.json")
    path = synth.cached_model(synth.PRESETS[name])
    assert os.path.getsize(path) == fx["bytes"]
    assert synth.file_sha256(path) == fx["sha256"]
    with HakmCtx(path, max_seq=max_seq) as ctx:
        toks = ctx.generate(fx["prompt"], fx["n_gen"])
    assert first_divergence(toks, fx["tokens"]) is None, (first_divergence(toks, fx["tokens"]), toks[:8])


def test_prefill_matches_per_token_feed(cuda, reference, small_path):
    """hakmc_prefill (one launch, lm_head only on the last id) leaves the same
    state as feeding the ids one hakm_forward at a time, and as the
    reference's feed loop: same last logits (bit for bit), same
    continuation."""
    from oracle.oracle import RefModel
    prompt = [11, 4000, 256, 259, 1, 2, 3, 77, 9, 123]
    with HakmCtx(small_path, max_seq=64) as a, HakmCtx(small_path, max_seq=64) as b:
        la, ama = a.prefill(prompt)
        lb = amb = None
        for t in prompt:
            lb, amb = b.forward(t)
        assert a.pos == b.pos == len(prompt)
        assert ama == amb
        assert same(la, lb)
        assert a.generate([ama], 8) == b.generate([amb], 8)
    ref = RefModel(small_path, 64)
    lr = None
    for t in prompt:
        lr, _ = ref.forward(t)
    ref.close()
    assert same(la, lr)


@pytest.mark.parametrize("preset,n,chunk", [("small", 40, 0), ("small", 40, 7), ("mid", 300, 128)])
def test_prefill_batched_matches_per_position_prefill(cuda, reference, preset, n, chunk):
    """hakmc_prefill_batched (positions batched through each layer: tensor-core
    Q4_K matmuls, Q6_K lane chains, attention of each row over the cache)
    leaves the state hakmc_prefill leaves, bit for bit: the last logits, the
    KV cache (the next step's logits), the position; and its logits are the
    reference's feed loop's. Chunks of 7 rows cross chunk boundaries inside
    the prompt; the mid model has head_dim 128 and a 300-position prompt."""
    from oracle.oracle import RefModel
    path = synth.cached_model(synth.PRESETS[preset])
    prompt = [(37 * i + 11) % 4000 for i in range(n)]
    with HakmCtx(path, max_seq=512) as a, HakmCtx(path, max_seq=512) as b:
        la, ama = a.prefill_batched(prompt, chunk_rows=chunk)
        lb, amb = b.prefill(prompt)
        assert a.pos == b.pos == n
        assert same(la, lb), rel_l2(la, lb)
        assert ama == amb == int(np.argmax(la))
        na, nma = a.forward(amb)
        nb, nmb = b.forward(amb)
        assert same(na, nb), rel_l2(na, nb)
        assert nma == nmb
    ref = RefModel(path, 512)
    lr = None
    for i, t in enumerate(prompt):
        lr, _ = ref.forward(t, want_logits=i == n - 1)
    ref.close()
    assert same(la, lr), rel_l2(la, lr)


@pytest.mark.parametrize("layers", [1, 2])
def test_prefill_batched_hidden_states(cuda, small_path, layers):
    """The residual stream of the last position after 1 and 2 layers equals
    the per-position path's (and so the reference's, test_layer_outputs)."""
    prompt = [(91 * i + 5) % 4000 for i in range(33)]
    with HakmCtx(small_path, max_seq=64) as a, HakmCtx(small_path, max_seq=64) as b:
        a.set_layers(layers)
        b.set_layers(layers)
        a.prefill_batched(prompt, chunk_rows=16)
        b.prefill(prompt)
        assert same(a.hidden(), b.hidden()), rel_l2(a.hidden(), b.hidden())


def test_prefill_batched_rejects_bad_input(cuda, small_path):
    with HakmCtx(small_path, max_seq=8) as ctx:
        with pytest.raises(HakmcError):
            ctx.prefill_batched([1] * 9)
        with pytest.raises(HakmcError):
            ctx.prefill_batched([1, 10 ** 7])
        assert ctx.pos == 0
        ctx.prefill_batched([1, 2, 3])
        assert ctx.pos == 3


def test_prefill_rejects_bad_input(cuda, small_path):
    with HakmCtx(small_path, max_seq=8) as ctx:
        with pytest.raises(HakmcError):
            ctx.prefill([1] * 9)
        with pytest.raises(HakmcError):
            ctx.prefill([1, 10 ** 7])
        assert ctx.pos == 0


@pytest.mark.parametrize("layers", [None, 1])
def test_forward_batch_rows_equal_single_sequence_contexts(cuda, small_path, layers):
    """hakmc_forward_batch: row i is hakm_forward on a context holding
    sequence i's cache (slot i), bit for bit, although the rows go through
    each layer together (weights read once for all of them). Nine sequences
    (a batch that takes the batched pass) with different prompts, fed and
    then decoded greedily in lockstep; three of them start later, idle rows
    write a spare position."""
    prompts = [[11, 22, 33, 44], [500, 600, 700, 800], [3000, 17, 42, 9], [7, 8, 9, 10], [1234, 99, 5, 66],
               [1, 2, 3, 4], [4095, 4094, 100, 200], [31, 62, 93, 124], [2048, 1024, 512, 256]]
    n_seq, n_gen, start = 9, 6, [0, 0, 2, 0, 1, 0, 3, 0, 0]
    batch = HakmCtx(small_path, max_seq=64, max_batch=n_seq)
    singles = [HakmCtx(small_path, max_seq=64) for _ in prompts]
    if layers:
        for x in [batch] + singles:
            x.set_layers(layers)
    try:
        nxt = [None] * n_seq
        feed = [list(p) for p in prompts]
        pos = [0] * n_seq
        for rnd in range(len(prompts[0]) + n_gen + 2):
            toks, poss, rows = [], [], []
            for i in range(n_seq):
                active = rnd >= start[i] and pos[i] < len(prompts[i]) + n_gen
                tok = (feed[i].pop(0) if feed[i] else nxt[i]) if active else 1
                toks.append(tok)
                poss.append(pos[i] if active else 63)  # idle rows write position 63 only
                rows.append(active)
            logits, am = batch.forward_batch(toks, poss, want_logits=True)
            for i in range(n_seq):
                assert am[i] == int(np.argmax(logits[i])), (rnd, i)
                if not rows[i]:
                    continue
                ref_logits, ref_am = singles[i].forward(toks[i])
                assert same(logits[i], ref_logits), (rnd, i, rel_l2(logits[i], ref_logits))
                assert int(am[i]) == ref_am, (rnd, i)
                nxt[i] = int(am[i])
                pos[i] += 1
        assert batch.pos == 0  # the single-sequence state is left alone
    finally:
        batch.close()
        for s in singles:
            s.close()


def test_forward_batch_long_caches(cuda, small_path):
    """Batched decode over long caches: nine sequences whose caches hold 700
    seeded N(0,1) positions (each its own seed), one step each at positions
    700..708, against single-sequence contexts filled with the same values."""
    n_seq = 9
    pos = [700 + i for i in range(n_seq)]
    toks = [(131 * i + 7) % 4000 for i in range(n_seq)]
    with HakmCtx(small_path, max_seq=1024, max_batch=n_seq) as batch:
        for i in range(n_seq):
            batch.fill_kv_normal(pos[i], seq=i, seed=50 + i)
        logits, am = batch.forward_batch(toks, pos, want_logits=True)
    for i in range(n_seq):
        with HakmCtx(small_path, max_seq=1024) as one:
            one.fill_kv_normal(pos[i], seq=0, seed=50 + i)
            assert one.pos == pos[i]
            ref, ref_am = one.forward(toks[i])
        assert same(logits[i], ref), (i, rel_l2(logits[i], ref))
        assert int(am[i]) == ref_am, i


@pytest.mark.parametrize("preset,n_seq,n_pos", [("small", 9, 700), ("small", 64, 1400), ("3b", 9, 4096)])
def test_forward_batch_vs_reference(cuda, reference, preset, n_seq, n_pos):
    """hakmc_forward_batch against the reference's own hakm_forward: every
    row's sequence has a cache of n_pos seeded N(0, 1) positions (each row
    its own seed, the same values written into the reference's
    hakm_ctx.k_cache / v_cache, src/model.h:21-22), then one decode step per
    row at positions n_pos + i % 4: logits and picks bit for bit. (The
    reference keeps its attention scores in gate_buf, so positions stay below
    ffn_dim: 1536 on the small model, 11008 on 3B.)"""
    from oracle.oracle import RefModel
    cfg = synth.PRESETS[preset]
    path = synth.cached_model(cfg)
    assert n_pos + 4 < cfg.ffn_dim
    max_seq = n_pos + n_seq + 8
    toks = [(131 * i + 7) % cfg.vocab for i in range(n_seq)]
    pos = [n_pos + i % 4 for i in range(n_seq)]
    refs = []
    with HakmCtx(path, max_seq=max_seq, max_batch=n_seq) as batch:
        for i in range(n_seq):
            rng = np.random.default_rng(1000 + i)
            k = rng.standard_normal((cfg.n_layers, pos[i], cfg.kv_dim)).astype(np.float32)
            v = rng.standard_normal((cfg.n_layers, pos[i], cfg.kv_dim)).astype(np.float32)
            batch.fill_kv(k, v, seq=i)
            ref = RefModel(path, max_seq)
            ref.write_kv(k, v)
            refs.append(ref)
        logits, am = batch.forward_batch(toks, pos, want_logits=True)
    for i in range(n_seq):
        lr, amr = refs[i].forward(toks[i])
        refs[i].close()
        assert same(logits[i], lr), (i, rel_l2(logits[i], lr))
        assert int(am[i]) == amr == int(np.argmax(logits[i])), i


def test_forward_batch_repeated_calls(cuda, small_path):
    """Two hundred consecutive batched steps of twelve sequences (the cached
    graph replayed, positions past several attention tiles): every call
    succeeds, picks are the logits' argmax, and a replay of the same calls
    on a fresh context gives the same bits (deterministic)."""
    n_seq, n_steps = 12, 200

    def run():
        out = []
        with HakmCtx(small_path, max_seq=256, max_batch=n_seq) as ctx:
            toks = [(37 * i + 3) % 4000 for i in range(n_seq)]
            for p in range(n_steps):
                logits, am = ctx.forward_batch(toks, [p] * n_seq, want_logits=(p % 50 == 49))
                if logits is not None:
                    assert all(int(am[i]) == int(np.argmax(logits[i])) for i in range(n_seq))
                    out.append(logits.copy())
                toks = [int(a) for a in am]
        return out, toks

    a, ta = run()
    b, tb = run()
    assert ta == tb
    for x, y in zip(a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))


def test_forward_batch_small_batches_are_forward(cuda, small_path):
    """Batches below the batched pass's size take the step kernel per
    sequence, as hakm_forward: bit for bit (three sequences, then one)."""
    with HakmCtx(small_path, max_seq=64, max_batch=3) as a:
        singles = [HakmCtx(small_path, max_seq=64) for _ in range(3)]
        try:
            for p in range(5):
                toks = [11 * (p + 1) + 7 * i for i in range(3)]
                la, ama = a.forward_batch(toks, [p] * 3, want_logits=True)
                for i in range(3):
                    lb, amb = singles[i].forward(toks[i])
                    assert np.array_equal(la[i].view(np.uint32), lb.view(np.uint32)), (p, i)
                    assert ama[i] == amb
            la, ama = a.forward_batch([5], [5], want_logits=True)  # slot 0 alone
            lb, amb = singles[0].forward(5)
            assert np.array_equal(la[0].view(np.uint32), lb.view(np.uint32))
            assert ama[0] == amb
        finally:
            for x in singles:
                x.close()


def test_forward_batch_rejects_bad_input(cuda, tiny_path):
    ctx = HakmCtx(tiny_path, max_seq=16, max_batch=2)
    try:
        with pytest.raises(HakmcError):
            ctx.forward_batch([1, 2], [0, 16])  # position beyond max_seq
        with pytest.raises(HakmcError):
            ctx.forward_batch([1, 2, 3], [0, 0, 0])  # more sequences than max_batch
        with pytest.raises(HakmcError):
            ctx.forward_batch([1, -5], [0, 0])  # token out of range
    finally:
        ctx.close()
