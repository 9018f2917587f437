"""Multi-GPU serving plumbing for batches of independent rows (prompts / steering rows).

Rows never exchange data in the engine's forward, so the batch is sharded across ranks (one process per GPU) and the
only collective is a final gather of each rank's outputs (the reference's independent steering rows and prompts,
engine/analysis.js:480-537, are likewise independent).  Every rank serves `rows` rows of its own: rank r owns global
rows [r rows, (r + 1) rows) of a batch of world * rows, and its prompts and steering vectors are drawn from
generators seeded by (seed, r), so a rank's inputs do not depend on how many ranks there are.
"""
import torch


def rank_rows(rank, rows_per_rank):
    """Global index of the first row of `rank`'s batch."""
    return rank * rows_per_rank


def rank_prompts(rank, rows, prompt, vocab, seed=0):
    """[rows, prompt] int32 random token ids of `rank`'s batch."""
    g = torch.Generator().manual_seed(seed * 1000003 + rank)
    return torch.randint(0, vocab, (rows, prompt), generator=g, dtype=torch.int32)


def rank_vectors(rank, rows, hidden, scale, seed=0, carrying=None):
    """[rows, hidden] steering vectors N(0, 1) * scale for the first `carrying` rows (default half), zero after."""
    g = torch.Generator().manual_seed((seed + 1) * 1000003 + rank)
    v = torch.randn(rows, hidden, generator=g) * scale
    v[(rows // 2 if carrying is None else carrying):] = 0
    return v


def gather_rows(x, world, group=None):
    """All ranks' [rows, ...] outputs, stacked in rank order: [world, rows, ...] (one all_gather; works on NCCL and
    gloo process groups)."""
    if world == 1:
        return x.unsqueeze(0)
    import torch.distributed as dist
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.stack(parts)
