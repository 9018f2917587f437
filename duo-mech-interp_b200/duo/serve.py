"""Multi-GPU plumbing for one fixed batch of independent rows (prompts / steering rows), one process per GPU.

Rows never exchange data in the engine's forward (the reference's only parallelism is rows inside one forward,
engine/model.js:404-466), so one batch is split into contiguous blocks of whole units across the ranks and the only
collective is a final gather of each rank's outputs:
  * serving (throughput config): a unit is one prompt row; 256 rows split 256 / N per rank;
  * push test (analysis.js:480-537): a unit is a (candidate, context) triple of rows (+dose, 0, -dose), so every
    pushed row has its unpushed base row on the same rank; 72 triples = 216 rows split 72 / N per rank.
The batch itself (prompts, vectors, candidates, targets) is drawn from generators seeded once for the whole batch, so
every rank sees the same global batch and the result does not depend on the number of ranks.
"""
import torch


def shard(rank, world, units):
    """Contiguous block [start, stop) of `units` for `rank` (the first units % world ranks take one more)."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    base, extra = divmod(units, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def batch_prompts(rows, prompt, vocab, seed=0):
    """[rows, prompt] int32 random token ids of the whole batch."""
    g = torch.Generator().manual_seed(seed * 1000003 + 17)
    return torch.randint(0, vocab, (rows, prompt), generator=g, dtype=torch.int32)


def batch_vectors(rows, hidden, scale, seed=0, carrying=None):
    """[rows, hidden] steering vectors N(0, 1) * scale for the first `carrying` rows of the batch (default half), zero
    after."""
    g = torch.Generator().manual_seed((seed + 1) * 1000003 + 29)
    v = torch.randn(rows, hidden, generator=g) * scale
    v[(rows // 2 if carrying is None else carrying):] = 0
    return v


def probe_batch(n_cands, n_ctx, ctx_len, n_targets, layers, inter, vocab, seed=0):
    """The push test's batch: candidates [(layer, neuron)], contexts [n_ctx lists of ctx_len ids], target ids and
    weights.  Row order is (candidate, context, strength) -- duo.probe.triple_rows."""
    g = torch.Generator().manual_seed(seed * 1000003 + 41)
    cands = [(int(torch.randint(0, layers, (1,), generator=g)), int(torch.randint(0, inter, (1,), generator=g)))
             for _ in range(n_cands)]
    contexts = [torch.randint(0, vocab, (ctx_len,), generator=g).tolist() for _ in range(n_ctx)]
    targets = torch.randint(0, vocab, (n_targets,), generator=g).tolist()
    weights = (torch.rand(n_targets, generator=g) + 0.05).tolist()
    return cands, contexts, targets, weights


def triple_block(rank, world, n_cands, n_ctx):
    """This rank's (candidate, context) triples of a push test as candidate-major unit indices [start, stop), and its
    global rows [3 start, 3 stop)."""
    start, stop = shard(rank, world, n_cands * n_ctx)
    return start, stop


def gather_rows(x, world, group=None):
    """All ranks' equal-sized [rows, ...] blocks concatenated in rank order: [world * rows, ...] (one all_gather into
    a single tensor; works on NCCL and gloo process groups)."""
    if world == 1:
        return x
    import torch.distributed as dist
    out = torch.empty((world * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out
