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
