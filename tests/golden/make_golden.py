"""Generate the golden vectors under tests/golden/ from the reference engine's
OWN compiled sources (oracle/_ref/libhakm_ref.so, built by `make -C oracle ref`
from mithraeums/hako's src/ with its Makefile:8 flags).

    python tests/golden/make_golden.py [--big]

Fixtures (all small; synthetic models are regenerated from their seeded
configs and pinned by sha256):
  q8.npz        quantize_row_q8_32 on random and edge-case vectors
  q4k.npz       q4k_vec_dot on random rows; integer sub-block sums pinned
                through crafted rows (d = 1, dmin = 0, one scale = 1)
  dequant.npz   dequant_q4_K / dequant_q6_K outputs
  ops.npz       rmsnorm, rope_neox
  tiny.json     tiny model: file hash, logits checksums, greedy stream
  3b.json       (--big) config 0: file hash, 16-id prompt, 64 greedy ids and
                the top1-top2 logit gap of every step
  7b.json       (--big) config 3: 32-id prompt, 128 greedy ids and gaps
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from hako_b200 import synth  # noqa: E402
from oracle.oracle import Reference, RefModel  # noqa: E402

F16_ONE = 0x3C00


def q8_cases():
    rng = np.random.default_rng(1234)
    cases = [rng.standard_normal(4096).astype(np.float32),
             (rng.standard_normal(2048) * 1e-3).astype(np.float32),
             (rng.standard_normal(2048) * 50).astype(np.float32)]
    z = np.zeros(256, np.float32)
    z[40:72] = rng.standard_normal(32)  # zero blocks around a live block
    cases.append(z)
    # exact .5 ties after scaling: amax 127 -> scale fl(1/127)*127, values k+0.5
    t = np.zeros(64, np.float32)
    t[0] = 127.0
    t[1:32] = np.arange(31, dtype=np.float32) + 0.5
    t[32] = -127.0
    t[33:64] = -(np.arange(31, dtype=np.float32) + 0.5)
    cases.append(t)
    # subnormal magnitudes (scale underflow / reciprocal overflow paths)
    s = np.full(64, 1e-39, np.float32)
    s[32:] = np.float32(3e-38)
    s[1] = -2e-39
    cases.append(s)
    return cases


def main(big: bool) -> None:
    R = Reference()
    # ---------------------------------------------------------------- q8
    out = {}
    for i, x in enumerate(q8_cases()):
        xq, xs = R.quantize_q8_32(x)
        out[f"x{i}"], out[f"xq{i}"], out[f"xs{i}"] = x, xq, xs
    np.savez_compressed(os.path.join(HERE, "q8.npz"), **out)

    # ---------------------------------------------------------------- q4k
    K = 2048
    w = synth.random_q4k(8, K, 42)
    x = synth.normal(K, 43)
    xq, xs = R.quantize_q8_32(x)
    dots = np.array([R.q4k_vec_dot(w[r * 8 * 144:(r + 1) * 8 * 144], K, xq, xs) for r in range(8)], np.float32)
    # integer pins: one block, d = 1 (or dmin = 1), one 6-bit scale (or min) = 1
    rng = np.random.default_rng(7)
    pin_blocks, pin_xq, pin_iqx, pin_ix = [], [], [], []
    for trial in range(16):
        blk = np.zeros(144, np.uint8)
        blk[16:] = rng.integers(0, 256, 128, dtype=np.uint8)
        xqv = rng.integers(-127, 128, 256).astype(np.int8)
        ones = np.ones(8, np.float32)
        iq, ixs = [], []
        for j in range(8):
            for which in ("s", "m"):
                b = blk.copy()
                sc = np.zeros(12, np.uint8)
                if j < 4:
                    sc[j if which == "s" else j + 4] = 1
                else:
                    sc[j + 4] = 1 if which == "s" else 0x10
                b[4:16] = sc
                d_u16 = F16_ONE if which == "s" else 0
                m_u16 = F16_ONE if which == "m" else 0
                b[0:2] = np.frombuffer(np.uint16(d_u16).tobytes(), np.uint8)
                b[2:4] = np.frombuffer(np.uint16(m_u16).tobytes(), np.uint8)
                v = R.q4k_vec_dot(b, 256, xqv, ones)
                (iq if which == "s" else ixs).append(int(round(v)) if which == "s" else -int(round(v)))
        pin_blocks.append(blk); pin_xq.append(xqv); pin_iqx.append(iq); pin_ix.append(ixs)
    np.savez_compressed(os.path.join(HERE, "q4k.npz"), w=w, x=x, xq=xq, xs=xs, dots=dots,
                        pin_blocks=np.stack(pin_blocks), pin_xq=np.stack(pin_xq),
                        pin_iqx=np.array(pin_iqx, np.int32), pin_ix=np.array(pin_ix, np.int32))

    # ---------------------------------------------------------------- dequant
    w4 = synth.random_q4k(4, 1024, 5)
    w6 = synth.random_q6k(4, 1024, 6)
    np.savez_compressed(os.path.join(HERE, "dequant.npz"), w4=w4, w6=w6,
                        d4=R.dequant(w4, 12, 4 * 1024), d6=R.dequant(w6, 14, 4 * 1024))

    # ---------------------------------------------------------------- ops
    xr = synth.normal(2048, 50)
    wr = (1.0 + 0.1 * synth.normal(2048, 51)).astype(np.float32)
    q = synth.normal(16 * 128, 52)
    ops = dict(x=xr, w=wr, rms=R.rmsnorm(xr, wr, 1e-6), q=q)
    for pos in (0, 1, 17, 511, 4095):
        ops[f"rope{pos}"] = R.rope(q, 128, pos, 1.0e6)
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **ops)

    # ---------------------------------------------------------------- models
    def model_fixture(name, prompt, n_gen, max_seq, logits_steps=0):
        cfg = synth.PRESETS[name]
        path = synth.cached_model(cfg)
        m = RefModel(path, max_seq)
        fx = {"config": name, "bytes": os.path.getsize(path), "sha256": synth.file_sha256(path),
              "prompt": [int(t) for t in prompt], "n_gen": n_gen}
        if logits_steps:
            sums = []
            for t in prompt[:logits_steps]:
                lg, am = m.forward(int(t))
                sums.append({"argmax": am, "sum": float(lg.astype(np.float64).sum()),
                             "l2": float(np.linalg.norm(lg.astype(np.float64))), "first8": lg[:8].tolist()})
            fx["logits"] = sums
            m.reset()
        toks, gaps = m.greedy(prompt, n_gen)
        fx["tokens"] = [int(t) for t in toks]
        fx["gaps"] = [float(g) for g in gaps]
        m.close()
        with open(os.path.join(HERE, f"{name}.json"), "w") as f:
            json.dump(fx, f, indent=1)
        print(name, "min gap", min(fx["gaps"]), fx["tokens"][:8])

    model_fixture("tiny", [5, 17, 300, 999, 2, 7, 64, 1000], 32, 256, logits_steps=8)
    model_fixture("small", [11, 4000, 256, 259, 1, 2, 3, 77], 32, 256, logits_steps=4)
    if big:
        rng = np.random.default_rng(0)
        model_fixture("3b", rng.integers(0, 151643, 16).tolist(), 64, 128)
        rng = np.random.default_rng(3)
        model_fixture("7b", rng.integers(0, 151643, 32).tolist(), 128, 256)


if __name__ == "__main__":
    main(big="--big" in sys.argv)
