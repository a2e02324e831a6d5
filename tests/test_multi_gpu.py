"""Sharded attention on two GPUs: the CUDA kernel on each rank's shard, NCCL all-gather.

Each rank runs flash_attn_mlm_compressed on its shard (heads with the matching
rows of the head-major KV cache, or whole sequences for MLA), the packed
outputs are gathered with NCCL, and rank 0 compares the result with the
unsharded call on its own GPU.  Every (sequence, head) item is computed the
same way in both runs, so the results must be bit-identical.  Skipped unless
two GPUs are visible.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(mode):
    g = torch.Generator().manual_seed(4242)
    B, N = 6, 192
    H, D = (8, 64) if mode == "heads" else (4, 512)
    dt = torch.bfloat16
    lengths = torch.randint(16, N + 1, (B,), generator=g, dtype=torch.int32)
    ctx = torch.randint(0, 300, (B,), generator=g, dtype=torch.int32)
    q = torch.randn((B, H, N, D), generator=g).to(dt)
    k = torch.randn((B, H, N, D), generator=g).to(dt)
    v = torch.randn((B, H, N, D), generator=g).to(dt)
    tcl = int(ctx.sum())
    kc = torch.randn((tcl if mode == "batch" else H * tcl, D), generator=g).to(dt)
    vc = torch.randn(tuple(kc.shape), generator=g).to(dt)
    return lengths, ctx, q, k, v, kc, vc


def _run(fm, q, k, v, kc, vc, lengths, ctx, is_mla, dev):
    H, N, D = q.shape[1], q.shape[2], q.shape[3]
    cu_kv = torch.zeros(len(ctx) + 1, dtype=torch.int32)
    cu_kv[1:] = ctx.cumsum(0)
    cache = fm.InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(dev), v_cache=None if is_mla else vc.to(dev),
                           total_context_len=int(cu_kv[-1]), cu_seqlens_kv=cu_kv.to(dev),
                           context_batch_size=len(ctx), is_mla=is_mla, num_heads=H, head_dim=D)
    meta = fm.build_pack_metadata(lengths.to(dev), N, 64)
    kk = k[:, :1].expand_as(k) if is_mla else k
    return fm.flash_attn_mlm_compressed(q.to(dev), kk.to(dev), (kk if is_mla else v).to(dev), num_heads=H,
                                        q_meta=meta, scale=D ** -0.5, inference_cache=cache, layer_id=0,
                                        block_n=64, is_mla=is_mla)


def _worker(rank, world, port, mode, ret):
    import sys

    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "flash-mlm_b200"))
    import torch.distributed as dist

    import flash_mlm as fm
    from flash_mlm.parallel import gather_packed_output, plan_shards, shard_head_major_cache, shard_qkv

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        lengths, ctx, q, k, v, kc, vc = _inputs(mode)
        is_mla = mode == "batch"
        H = q.shape[1]
        plans = plan_shards(lengths.tolist(), H, world, context_lengths=ctx.tolist(), is_mla=is_mla)
        p = plans[rank]
        if p.mode == "heads":
            tcl = int(ctx.sum())
            local = _run(fm, shard_qkv(q, p), shard_qkv(k, p), shard_qkv(v, p), shard_head_major_cache(kc, p, tcl),
                         shard_head_major_cache(vc, p, tcl), lengths, ctx, False, dev)
        else:
            starts = torch.cat([torch.zeros(1, dtype=torch.long), ctx.long().cumsum(0)])
            rows = torch.cat([torch.arange(int(starts[b]), int(starts[b + 1])) for b in p.batches])
            local = _run(fm, shard_qkv(q, p), shard_qkv(k, p), shard_qkv(v, p), kc[rows], vc[rows],
                         lengths[p.batches], ctx[p.batches], True, dev)
        full = gather_packed_output(local, plans, lengths.tolist(), H)
        fm.check_device_errors(dev)
        if rank == 0:
            ref = _run(fm, q, k, v, kc, vc, lengths, ctx, is_mla, dev)
            ret.put((bool(torch.equal(full, ref)), float((full.float() - ref.float()).abs().max())))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["heads", "batch"])
def test_two_gpu_sharded_attention_matches_single_gpu(mode):
    ctx = mp.get_context("spawn")
    ret = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, mode, ret)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
    codes = [pr.exitcode for pr in procs]
    assert codes == [0, 0], f"rank exit codes {codes}"
    equal, maxdiff = ret.get(timeout=10)
    assert equal, f"sharded result differs from the single-GPU call (max |diff| {maxdiff})"
