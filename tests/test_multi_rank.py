"""Multi-rank host logic on CPU ranks (gloo, world size 2): the row sharding and the final output gather that bench.py
runs over NCCL, one process per GPU.  Rows are independent, so each rank owns its own seeded batch and the only
collective is the gather."""
import os
import socket
from datetime import timedelta

import torch

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from duo import serve
        ids = serve.rank_prompts(rank, 6, 5, 1000, seed=3)
        vec = serve.rank_vectors(rank, 6, 8, 2.0, seed=3)
        toks = ids[:, :2] + 10 * rank  # stand-in for the rank's generated tokens
        q.put((rank, ids, vec, serve.gather_rows(toks, WORLD)))
    finally:
        dist.destroy_process_group()


def test_two_ranks_shard_and_gather():
    import torch.multiprocessing as mp
    from duo import serve
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(WORLD):
        rank, ids, vec, allt = q.get(timeout=120)
        got[rank] = (ids, vec, allt)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # a rank's inputs depend only on its rank (not on the number of ranks); ranks get different prompts
    for r in range(WORLD):
        assert torch.equal(got[r][0], serve.rank_prompts(r, 6, 5, 1000, seed=3))
        assert torch.equal(got[r][1], serve.rank_vectors(r, 6, 8, 2.0, seed=3))
        assert bool((got[r][1][3:] == 0).all()) and bool((got[r][1][:3] != 0).any())
    assert not torch.equal(got[0][0], got[1][0])
    # every rank ends with all ranks' outputs, in rank order
    expect = torch.stack([got[r][0][:, :2] + 10 * r for r in range(WORLD)])
    for r in range(WORLD):
        assert torch.equal(got[r][2], expect)
    assert serve.rank_rows(1, 6) == 6
