"""Host side of tensor-parallel setup, on CPU: the handle all-gather over a
world-size-2 gloo group delivers every rank's bytes to every rank in rank
order (what hakmc_tp_connect needs)."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "tp", os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "hako_b200", "tp.py"))
    tp = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(tp)
    mine = bytes([rank]) * (100 + rank)  # ranks' handles need not even share a length here
    got = tp.all_gather_bytes(mine)
    q.put((rank, got))
    dist.destroy_process_group()


def test_handle_all_gather_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    expect = [bytes([0]) * 100, bytes([1]) * 101]
    assert res[0] == expect and res[1] == expect


def _plan(seg_rows, grid, cta):
    import ctypes as C
    import numpy as np
    from hako_b200 import lib
    rows = np.array(seg_rows, np.int32)
    out = np.zeros(2 * len(seg_rows), np.int32)
    rc = lib.hakmc_plan_rows(C.c_void_p(rows.ctypes.data), len(seg_rows), grid, cta, C.c_void_p(out.ctypes.data))
    assert rc == 0
    return out.reshape(-1, 2)


# the step program's GEMV phases as row segments (hakm_runtime.cu make_phase):
# qkv = [q and k rows in RoPE-pair order, v rows], wo, ffn gate/up
# interleaved, ffn down, lm_head
def _phases(cfg):
    D, KV, F, V = cfg.d_model, cfg.kv_dim, cfg.ffn_dim, cfg.vocab
    return {"qkv": [D + KV, KV], "wo": [D], "ffn": [2 * F], "down": [D], "lm_head": [V]}


@pytest.mark.parametrize("name", ["3b", "7b"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_row_partition_covers_every_row_once(name, world):
    """Rows of every phase split over the CTAs of all ranks (148 per GPU):
    each row computed exactly once, in 4-row groups (RoPE and SwiGLU row
    pairs never split across CTAs or GPUs), whole rows (K is never split, so
    each row's q8_32 blocks and Q6_K lane chains stay on one GPU) — including
    the 7B ffn (18944 = 74 super-blocks, uneven over 4 and 8 GPUs)."""
    import numpy as np
    from hako_b200 import synth
    cfg = synth.PRESETS[name]
    sms = 148
    grid = sms * world
    for ph, segs in _phases(cfg).items():
        seen = [np.zeros(n, np.int32) for n in segs]
        per_rank = np.zeros((world, len(segs)), np.int64)
        for cta in range(grid):
            rg = _plan(segs, grid, cta)
            for s, (a, b) in enumerate(rg):
                assert 0 <= a <= b <= segs[s], (ph, cta, s, a, b)
                if b > a:
                    assert a % 4 == 0 and (b % 4 == 0 or b == segs[s]), (ph, cta, a, b)
                    seen[s][a:b] += 1
                    per_rank[cta // sms, s] += b - a
        for s in range(len(segs)):
            assert (seen[s] == 1).all(), (ph, s, int((seen[s] != 1).sum()))
        # balanced: no rank gets more than one 4-row group per CTA above its share
        for s in range(len(segs)):
            assert per_rank[:, s].max() - per_rank[:, s].min() <= 4 * sms, (ph, s, per_rank[:, s])


@pytest.mark.parametrize("H,hd", [(16, 128), (28, 128), (8, 64)])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_attention_units_dealt_once(H, hd, world):
    """Attention units (query head, 32 dimensions) dealt round-robin to the
    ranks: every unit on exactly one rank (28 heads x 4 slices over 8 GPUs
    included)."""
    import ctypes as C
    import numpy as np
    from hako_b200 import lib
    n_units = H * hd // 32
    seen = np.zeros(n_units, np.int32)
    buf = np.zeros(n_units, np.int32)
    for r in range(world):
        n = lib.hakmc_plan_attn_units(H, hd, r, world, C.c_void_p(buf.ctypes.data), n_units)
        assert 0 <= n <= n_units
        seen[buf[:n]] += 1
    assert (seen == 1).all()
