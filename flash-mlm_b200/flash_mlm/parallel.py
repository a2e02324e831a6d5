"""Multi-GPU sharding of the flash-mlm forward path (one process per GPU).

The attention has no exchange step: every (sequence, head) pair is
independent.  A job is therefore split across ranks with no collective on the
data path:

* by heads: rank r owns a contiguous block of heads [h0, h1) of every
  sequence (blocks as even as the head count allows) and keeps the matching
  contiguous row block [h0*Tctx, h1*Tctx) of the head-major KV cache (its KV
  shard); a job with causal_query_seq_attn (every sequence also reads the keys
  of all earlier ones) is always split this way;
* by sequences, balanced by attention cost (query rows x key rows, longest
  first), when asked or when the heads do not divide evenly; MLA (a single
  latent KV head) always shards by sequences.

``gather_packed_output`` reassembles the packed output on every rank with one
all-gather (NCCL over NVLink on GPUs, gloo on CPU) when a caller needs the full
result in one place; it is not part of the hot path.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class ShardPlan:
    rank: int
    world_size: int
    mode: str                      # "heads" or "batch"
    heads: tuple[int, int]         # [h0, h1)
    batches: list[int] = field(default_factory=list)  # sequences owned (batch mode) or all


def _costs(lengths, context_lengths, causal):
    costs, prefix = [], 0
    for b, L in enumerate(lengths):
        prefix += L
        kv = (prefix if causal else L) + (context_lengths[b] if context_lengths is not None else 0)
        costs.append(L * kv)
    return costs


def plan_shards(lengths: list[int], num_heads: int, world_size: int, *, context_lengths: list[int] | None = None,
                causal: bool = False, is_mla: bool = False, mode: str = "auto") -> list[ShardPlan]:
    """Deterministic plan for every rank (each rank can compute it locally).

    ``mode``: "heads" splits the heads into contiguous blocks as evenly as
    possible (block sizes differ by at most one); "batch" splits the
    sequences, balanced by cost (longest processing time first); "auto" uses
    heads when they divide evenly and batch otherwise.  MLA (one latent KV
    head shared by all query heads) is always split by sequences.  With
    ``causal_query_seq_attn`` a sequence also reads the keys of every earlier
    sequence, so a causal job is always split by heads.
    """
    if world_size < 1:
        raise ValueError("world_size must be >= 1")
    if mode not in ("auto", "heads", "batch"):
        raise ValueError("mode must be 'auto', 'heads' or 'batch'")
    B = len(lengths)
    if is_mla:
        if causal and world_size > 1:
            raise ValueError("MLA with causal_query_seq_attn cannot be split across ranks")
        mode = "batch"
    elif causal:
        mode = "heads"
    elif mode == "auto":
        mode = "heads" if num_heads % world_size == 0 else "batch"
    if mode == "heads":
        if num_heads < world_size:
            raise ValueError("a heads split needs at least one head per rank")
        bounds = [r * num_heads // world_size for r in range(world_size + 1)]
        return [ShardPlan(r, world_size, "heads", (bounds[r], bounds[r + 1]), list(range(B)))
                for r in range(world_size)]
    costs = _costs(lengths, context_lengths, causal)
    order = sorted(range(B), key=lambda b: (-costs[b], b))
    load = [0] * world_size
    owned: list[list[int]] = [[] for _ in range(world_size)]
    for b in order:  # longest processing time first
        r = min(range(world_size), key=lambda i: (load[i], i))
        owned[r].append(b)
        load[r] += costs[b]
    return [ShardPlan(r, world_size, "batch", (0, num_heads), sorted(owned[r])) for r in range(world_size)]


def shard_qkv(x: torch.Tensor, plan: ShardPlan) -> torch.Tensor:
    """This rank's slice of a padded [B, H, N, D] tensor (a view for head shards)."""
    if plan.mode == "heads":
        return x[:, plan.heads[0]:plan.heads[1]]
    return x[plan.batches]


def shard_lengths(lengths: torch.Tensor, plan: ShardPlan) -> torch.Tensor:
    if plan.mode == "heads":
        return lengths
    return lengths[torch.as_tensor(plan.batches, dtype=torch.long, device=lengths.device)]


def shard_head_major_cache(cache: torch.Tensor, plan: ShardPlan, total_context_len: int) -> torch.Tensor:
    """Rows of a head-major [H*Tctx, D] cache this rank keeps (heads mode); the whole cache otherwise."""
    if plan.mode != "heads":
        return cache
    return cache[plan.heads[0] * total_context_len:plan.heads[1] * total_context_len]


def gather_packed_output(local: torch.Tensor, plans: list[ShardPlan], lengths: list[int], num_heads: int,
                         group=None) -> torch.Tensor:
    """All-gather per-rank packed outputs into the full packed [H * T, D] layout.

    ``local`` is this rank's packed output ([h_local * T, D] for head shards,
    [H * T_local, D] over its own sequences for batch shards).
    """
    import torch.distributed as dist

    world = len(plans)
    D = local.shape[1]
    T = sum(lengths)
    if plans[0].mode == "heads":
        rows = [(p.heads[1] - p.heads[0]) * T for p in plans]
    else:
        rows = [num_heads * sum(lengths[b] for b in p.batches) for p in plans]
    size = max(rows)
    buf = torch.zeros((size, D), dtype=local.dtype, device=local.device)
    buf[:local.shape[0]] = local
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    if plans[0].mode == "heads":
        return torch.cat([parts[r][:rows[r]] for r in range(world)], dim=0)
    out = torch.empty((num_heads * T, D), dtype=local.dtype, device=local.device)
    starts = [0]
    for L in lengths:
        starts.append(starts[-1] + L)
    for r, p in enumerate(plans):
        t_local = sum(lengths[b] for b in p.batches)
        piece = parts[r][:rows[r]].view(num_heads, t_local, D) if t_local else None
        off = 0
        for b in p.batches:
            L = lengths[b]
            if L:
                out.view(num_heads, T, D)[:, starts[b]:starts[b] + L] = piece[:, off:off + L]
            off += L
    return out
