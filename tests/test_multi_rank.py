"""Multi-rank host logic on CPU ranks (gloo, world size 2 and 4): the fixed-batch sharding and the final gather that
bench.py runs over NCCL, one process per GPU.  One batch (prompts, vectors, push-test candidates) is drawn once and
split into contiguous blocks of whole units -- prompt rows for serving, (candidate, context) triples for the push
test -- and every rank ends with all ranks' outputs in global row order."""
import os
import socket
from datetime import timedelta

import pytest
import torch


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from duo import probe, serve
        # serving: 16 prompt rows of one batch, 16 / world per rank
        rows, decode = 16, 3
        r0, r1 = serve.shard(rank, world, rows)
        ids = serve.batch_prompts(rows, 5, 1000, seed=3)[r0:r1]
        vec = serve.batch_vectors(rows, 8, 2.0, seed=3)[r0:r1]
        toks = (ids[:, :decode] * 0 + torch.arange(r0, r1, dtype=torch.int32)[:, None] * 100 +
                torch.arange(decode, dtype=torch.int32))  # stand-in for the rank's generated tokens [rows, decode]
        all_toks = serve.gather_rows(toks, world)
        # push test: 4 candidates x 2 contexts = 8 triples = 24 rows, whole triples per rank
        cands, ctxs, targets, weights = serve.probe_batch(4, 2, 6, 5, layers=24, inter=3584, vocab=1000, seed=3)
        t0, t1 = serve.triple_block(rank, world, len(cands), len(ctxs))
        units = [1.0] * len(cands)
        ids_all, pushes, base = probe.build_batch(cands, ctxs, units)
        my_rows = list(range(3 * t0, 3 * t1))
        my_base = [base[r] - 3 * t0 if base[r] >= 0 else -1 for r in my_rows]
        stats = torch.tensor([[float(r), float(my_base[i])] + [0.0] * 4 for i, r in enumerate(my_rows)])
        all_stats = serve.gather_rows(stats, world)
        q.put((rank, ids, vec, all_toks, my_base, all_stats, (r0, r1), (t0, t1)))
    finally:
        dist.destroy_process_group()


def test_shard_covers_every_unit_once():
    from duo import serve
    for units in (1, 7, 72, 216, 256):
        for world in (1, 2, 3, 4, 8):
            blocks = [serve.shard(r, world, units) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == units
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in blocks]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [2, 4])
def test_ranks_shard_one_batch_and_gather(world):
    import torch.multiprocessing as mp
    from duo import serve
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        item = q.get(timeout=180)
        got[item[0]] = item[1:]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    full_ids = serve.batch_prompts(16, 5, 1000, seed=3)
    full_vec = serve.batch_vectors(16, 8, 2.0, seed=3)
    # the ranks' blocks tile the one batch (not a batch per rank)
    assert torch.equal(torch.cat([got[r][0] for r in range(world)]), full_ids)
    assert torch.equal(torch.cat([got[r][1] for r in range(world)]), full_vec)
    assert bool((full_vec[8:] == 0).all()) and bool((full_vec[:8] != 0).any())
    # every rank ends with every row's tokens in global row order
    expect = torch.arange(16, dtype=torch.int32)[:, None] * 100 + torch.arange(3, dtype=torch.int32)
    for r in range(world):
        assert torch.equal(got[r][2], expect)
    # push test: whole triples per rank, each pushed row's base on the same rank, stats gathered in global row order
    for r in range(world):
        my_base = got[r][3]
        assert len(my_base) % 3 == 0
        for i, b in enumerate(my_base):
            assert (b == -1) if i % 3 == 1 else (0 <= b < len(my_base) and b == 3 * (i // 3) + 1)
        assert torch.equal(got[r][4][:, 0], torch.arange(24, dtype=torch.float32))
