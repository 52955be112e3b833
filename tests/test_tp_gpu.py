"""Tensor parallelism on 2 GPUs, one process per GPU (CUDA IPC): the step
kernel splits every phase's rows over both GPUs' CTAs and all-gathers each
output by peer stores. Row sharding leaves every float sum as on one GPU,
so tokens and logits must be bit-identical to a single-GPU context's; and
each rank keeps only its own rows of the split matrices.
Skipped on a box with fewer than 2 GPUs."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROMPT = [11, 4000, 256, 259, 1, 2, 3, 77, 9, 123, 4095, 17]


def _rank(rank, world, preset, n_gen, conn):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from hako_b200 import HakmCtx, synth
    path = synth.cached_model(synth.PRESETS[preset])
    out = {}
    if rank == 0:  # the single-GPU answer first, on GPU 0
        with HakmCtx(path, max_seq=128, device=0) as one:
            out["single_logits"], _ = one.prefill(PROMPT)
            out["single"] = one.generate([int(np.argmax(out["single_logits"]))], n_gen)
    import torch
    ctx = HakmCtx(path, max_seq=128, device=rank)
    conn.send(ctx.tp_export())
    handles = conn.recv()
    free0 = torch.cuda.mem_get_info(rank)[0]
    ctx.tp_connect(rank, handles)
    out["freed"] = torch.cuda.mem_get_info(rank)[0] - free0  # the rows of other ranks, dropped
    out["logits"], am = ctx.prefill(PROMPT)
    out["tp"] = ctx.generate([am], n_gen)
    out["pos"] = ctx.pos
    ctx.close()
    conn.send(out)


@pytest.mark.parametrize("preset", ["small", "3b"])
def test_tp2_bit_identical_to_one_gpu(cuda, preset):
    import torch
    import multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from hako_b200 import synth
    synth.cached_model(synth.PRESETS[preset])  # made once, before the ranks look for it
    ctx = mp.get_context("spawn")
    world, n_gen = 2, 24
    pipes = [ctx.Pipe() for _ in range(world)]
    procs = [ctx.Process(target=_rank, args=(r, world, preset, n_gen, pipes[r][1])) for r in range(world)]
    for p in procs:
        p.start()
    try:
        handles = [pipes[r][0].recv() if pipes[r][0].poll(300) else None for r in range(world)]
        assert all(h is not None for h in handles)
        for r in range(world):
            pipes[r][0].send(handles)
        res = [pipes[r][0].recv() if pipes[r][0].poll(600) else None for r in range(world)]
        assert all(x is not None for x in res)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    cfg = synth.PRESETS[preset]
    # the bytes of the matrices the step program splits: a decode step's
    # weights less the tied lm_head (the embedding, which stays whole)
    split = cfg.weight_bytes_per_token() - cfg.vocab * cfg.d_model // 256 * 210
    for r in range(world):
        assert res[r]["tp"] == res[0]["single"], r
        assert np.array_equal(res[r]["logits"], res[0]["single_logits"]), r
        assert res[r]["pos"] == len(PROMPT) + n_gen
        if preset == "3b":  # each rank keeps about half of the split weights
            assert res[r]["freed"] > 0.4 * split, (r, res[r]["freed"], split)


@pytest.mark.parametrize("sampling", [("-t", "0"), ("-t", "0.8", "-k", "40", "-p", "0.9", "-s", "1234")])
def test_dropin_cli_tensor_parallel(cuda, sampling):
    """The reference CLI over the drop-in with HAKMC_GPUS=2: one context
    tensor parallel over two GPUs (two threads making the same calls), the
    deferred prompt and the device pick as on one GPU; the printed bytes
    equal the unmodified reference CLI's."""
    import torch
    from oracle.oracle import DROPIN_CLI, REF_CLI
    from test_dropin_gpu import _run
    from hako_b200 import synth
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if not (os.path.exists(REF_CLI) and os.path.exists(DROPIN_CLI)):
        pytest.skip("oracle/_ref CLIs not built (make -C oracle ref dropin)")
    path = synth.cached_model(synth.PRESETS["small"])
    prompt = "once upon a time there was a"
    ours = _run(DROPIN_CLI, path, 40, prompt, {"HAKMC_GPUS": "2"}, sampling=sampling)
    assert ours == _run(REF_CLI, path, 40, prompt, sampling=sampling)
