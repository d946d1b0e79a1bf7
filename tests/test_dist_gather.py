"""Multi-process (world size 2, gloo, CPU) test of the data-parallel plumbing used by
bench.py --gpus N: per-rank codes of different lengths gathered to rank 0, and the max-over-
ranks timing reduction."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from qwentts_turbo_b200.dist import gather_codes, max_over_ranks
        n = 3 + 2 * rank
        codes = torch.arange(n * 16, dtype=torch.int32).reshape(n, 16) + 1000 * rank
        got = gather_codes(codes)
        t = max_over_ranks(1.5 + rank)
        if rank == 0:
            out_q.put(([g.tolist() for g in got], t))
        else:
            out_q.put((got, t))
    finally:
        dist.destroy_process_group()


def test_gather_codes_and_max_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    root = [r for r in res if r[0] is not None]
    assert len(root) == 1
    gathered, t = root[0]
    assert [len(g) for g in gathered] == [3, 5]
    assert gathered[1][0][0] == 1000
    assert all(r[1] == 2.5 for r in res)
