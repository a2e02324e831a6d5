"""Multi-rank sharding plumbing on CPU (gloo, world_size 2).

Each rank computes its shard with the CPU oracle (standing in for the GPU
kernel, which these CPU tests cannot launch), the packed outputs are
all-gathered, and the result must equal the unsharded computation exactly.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from flash_mlm.parallel import gather_packed_output, plan_shards, shard_head_major_cache, shard_lengths, shard_qkv


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, q, k, v, kc, vc, lengths, tcl, ctx_l, ret):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        H = q.shape[1]
        plans = plan_shards(lengths, H, world, context_lengths=ctx_l, is_mla=(mode == "batch"))
        p = plans[rank]
        lq = shard_lengths(torch.tensor(lengths), p).tolist()
        cu = np.concatenate([[0], np.cumsum(lq)]).astype(np.int64)
        qs, ks, vs = (shard_qkv(x, p).numpy() for x in (q, k, v))
        if p.mode == "heads":
            kcs = shard_head_major_cache(kc, p, tcl).numpy()
            vcs = shard_head_major_cache(vc, p, tcl).numpy()
            cu_kv = np.concatenate([[0], np.cumsum(ctx_l)])
            local = oracle.attention_packed(qs, ks, vs, cu, 0.125, k_cache=kcs, v_cache=vcs, cu_kv=cu_kv,
                                            context_batch_size=len(lengths), total_context_len=tcl)
        else:
            # MLA-style single latent head: context rows are per sequence; each rank keeps its sequences' rows
            starts = np.concatenate([[0], np.cumsum(ctx_l)])
            rows = [np.arange(starts[b], starts[b + 1]) for b in p.batches]
            kcs = kc.numpy()[np.concatenate(rows)] if rows else kc.numpy()[:0]
            cu_kv = np.concatenate([[0], np.cumsum([ctx_l[b] for b in p.batches])])
            local = oracle.attention_packed(qs, ks, ks, cu, 0.125, k_cache=kcs, v_cache=kcs, cu_kv=cu_kv,
                                            context_batch_size=len(p.batches), total_context_len=int(cu_kv[-1]),
                                            is_mla=True)
        full = gather_packed_output(torch.from_numpy(local), plans, lengths, H)
        if rank == 0:
            ret.put(full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["heads", "batch"])
def test_sharded_attention_reassembles_exactly(mode):
    g = torch.Generator().manual_seed(5)
    lengths = [40, 7, 0, 33, 18]
    B, H, N, D = len(lengths), 4, 40, 16
    q, k, v = (torch.randn((B, H, N, D), generator=g) for _ in range(3))
    ctx_l = [5, 0, 3, 9, 2]
    tcl = sum(ctx_l)
    if mode == "heads":
        kc, vc = torch.randn((H * tcl, D), generator=g), torch.randn((H * tcl, D), generator=g)
    else:
        kc = torch.randn((tcl, D), generator=g)
        vc = kc
    world = 2
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q, k, v, kc, vc, lengths, tcl, ctx_l, ret))
             for r in range(world)]
    for p in procs:
        p.start()
    full = ret.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    cu = np.concatenate([[0], np.cumsum(lengths)])
    cu_kv = np.concatenate([[0], np.cumsum(ctx_l)])
    if mode == "heads":
        ref = oracle.attention_packed(q.numpy(), k.numpy(), v.numpy(), cu, 0.125, k_cache=kc.numpy(),
                                      v_cache=vc.numpy(), cu_kv=cu_kv, context_batch_size=B, total_context_len=tcl)
    else:
        ref = oracle.attention_packed(q.numpy(), k.numpy(), k.numpy(), cu, 0.125, k_cache=kc.numpy(),
                                      v_cache=kc.numpy(), cu_kv=cu_kv, context_batch_size=B, total_context_len=tcl,
                                      is_mla=True)
    np.testing.assert_array_equal(full, ref)


def test_plan_balances_by_cost_and_is_deterministic():
    lengths = [512, 64, 300, 300, 80, 511, 1, 200]
    plans = plan_shards(lengths, 12, 8, context_lengths=[1000] * 8)
    assert all(p.mode == "batch" for p in plans)
    owned = sorted(b for p in plans for b in p.batches)
    assert owned == list(range(8))
    plans_h = plan_shards(lengths, 16, 4)
    assert [p.heads for p in plans_h] == [(0, 4), (4, 8), (8, 12), (12, 16)]
    assert plan_shards(lengths, 12, 8, context_lengths=[1000] * 8) == plans


def test_plan_modes_uneven_heads_and_causal_rules():
    lengths = [30, 10, 50, 20, 40]
    # heads split as evenly as the count allows (12 heads over 8 ranks: 1 or 2 each, contiguous)
    plans = plan_shards(lengths, 12, 8, mode="heads")
    sizes = [p.heads[1] - p.heads[0] for p in plans]
    assert sorted(set(sizes)) == [1, 2] and sum(sizes) == 12
    assert all(plans[r].heads[1] == plans[r + 1].heads[0] for r in range(7))
    assert all(p.batches == list(range(5)) for p in plans)
    # a causal job reads earlier sequences' keys: always split by heads, even when asked for batch
    assert all(p.mode == "heads" for p in plan_shards(lengths, 12, 4, causal=True, mode="batch"))
    # auto: heads when they divide, sequences otherwise; MLA always by sequences
    assert plan_shards(lengths, 16, 4)[0].mode == "heads"
    assert plan_shards(lengths, 12, 8)[0].mode == "batch"
    mla = plan_shards(lengths, 16, 2, is_mla=True, context_lengths=[5] * 5)
    assert {p.mode for p in mla} == {"batch"} and sorted(b for p in mla for b in p.batches) == list(range(5))
    with pytest.raises(ValueError, match="MLA with causal"):
        plan_shards(lengths, 16, 2, is_mla=True, causal=True)
    with pytest.raises(ValueError, match="at least one head per rank"):
        plan_shards(lengths, 4, 8, mode="heads")
    with pytest.raises(ValueError, match="mode must be"):
        plan_shards(lengths, 4, 2, mode="rows")


def test_bench_shards_cover_the_job():
    """bench.py's per-rank workloads: weak scaling grows the job N times, strong splits it; the
    ranks' shards cover every (sequence, head) of the job exactly once."""
    import argparse

    import bench

    args = argparse.Namespace(ctx=4096, batch=32)
    one = bench.Workload("2", args)
    strong = [bench.Workload("2", args, rank=r, world=4, scaling="strong") for r in range(4)]
    assert sum(w.H * w.T for w in strong) == one.H * one.T  # every (token, head) once
    assert sum(w.flops() for w in strong) == pytest.approx(one.flops())
    weak = [bench.Workload("2", args, rank=r, world=4, scaling="weak") for r in range(4)]
    assert sum(w.B for w in weak) == 4 * one.B and weak[0].B_job == 4 * one.B
    assert sorted(b for w in weak for b in w.plan.batches) == list(range(4 * one.B))
    causal = [bench.Workload("3", args, rank=r, world=2, scaling="weak") for r in range(2)]
    assert all(w.plan.mode == "heads" and w.H == 12 and w.B == 64 for w in causal)
