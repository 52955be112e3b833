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
