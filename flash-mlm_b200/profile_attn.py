"""Profiling driver for Nsight Compute: runs one BASELINE-shaped workload for a
few warm-up and measured iterations and nothing else (no timing loops, no
clock sampling), so `ncu -k regex:attn_fwd -s <warmup launches> -c <n>` can
capture the attention kernel on exactly that input.

    python flash-mlm_b200/profile_attn.py --config 2 --warmup 2 --iters 1

Configs: 1 dense [2,8,128,64] f16; 2 packed B=32 H=16 N=512
D=64 bf16 + shared 1024 context; 4 MLA B=16 H=128 D=512 + 4096 context per
sequence; 3 packed causal B=64 H=12 N=256 D=64 f16 +
per-sequence context U[256,2048]; 5a packed B=8 H=16 N=512 D=128 bf16 +
per-sequence context --ctx; 5b packed B=--batch H=16 N=512 D=128 bf16, no context.
`--op pack` / `--op unpack` / `--op append` run the copy kernels on config
2's shapes instead (pack_and_pad_main_tensors_for_mlm_compressed of q/k/v,
unpack_from_kernel of a packed [H*T, D] output, and InferenceCache
append_kv_cache of the batch's K/V into a reserved cache).
Equivalent of the reference's src/profile/profile_mlm_ncu.py.
"""

from __future__ import annotations

import argparse
import math
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))

import torch  # noqa: E402

import flash_mlm  # noqa: E402


def _lengths(g, B, lo, hi):
    return torch.randint(lo, hi + 1, (B,), generator=g, dtype=torch.int32)


def build(config: str, ctx: int, batch: int, device):
    """Returns a zero-argument callable that performs one step of the config."""
    g = torch.Generator().manual_seed(0)
    if config == "1":
        q, k, v = (torch.randn((2, 8, 128, 64), generator=g).to(torch.float16).to(device) for _ in range(3))
        return lambda: flash_mlm.flash_attn_mlm(q, k, v, scale=0.125)
    if config == "4":
        B, H, N, D = 16, 128, 256, 512
        lengths = _lengths(g, B, 128, 256)
        q = (torch.randn((B, H, N, D), generator=g) * 0.5).to(torch.bfloat16).to(device)
        k = (torch.randn((B, 1, N, D), generator=g) * 0.5).to(torch.bfloat16).to(device).expand(B, H, N, D)
        ctx = 4096
        cu_kv = torch.arange(B + 1, dtype=torch.int32) * ctx
        kc = (torch.randn((B * ctx, D), generator=g) * 0.5).to(torch.bfloat16).to(device)
        cache = flash_mlm.InferenceCache()
        cache.prefill_kv_cache(0, k_cache=kc, total_context_len=B * ctx, cu_seqlens_kv=cu_kv.to(device),
                               context_batch_size=B, is_mla=True, num_heads=H, head_dim=D)
        meta = flash_mlm.build_pack_metadata(lengths.to(device), N, 64)
        return lambda: flash_mlm.flash_attn_mlm_compressed(q, k, k, num_heads=H, q_meta=meta, scale=D ** -0.5,
                                                           inference_cache=cache, layer_id=0, block_n=64,
                                                           is_mla=True)
    if config == "2":
        B, H, N, D, C, lo, hi, dt = 32, 16, 512, 64, 1024, 64, 512, torch.bfloat16
    elif config == "3":
        B, H, N, D, C, lo, hi, dt = 64, 12, 256, 64, None, 32, 256, torch.float16
    elif config == "5a":
        B, H, N, D, C, lo, hi, dt = 8, 16, 512, 128, ctx, 256, 512, torch.bfloat16
    elif config == "5b":
        B, H, N, D, C, lo, hi, dt = batch, 16, 512, 128, 0, 256, 512, torch.bfloat16
    else:
        raise SystemExit(f"unknown config {config}")
    lengths = _lengths(g, B, lo, hi)
    q, k, v = (torch.randn((B, H, N, D), generator=g).to(dt).to(device) for _ in range(3))
    cache = flash_mlm.InferenceCache()
    causal = config == "3"
    if config == "3":
        ctx_l = _lengths(g, B, 256, 2048)
        cu_kv = torch.zeros(B + 1, dtype=torch.int32)
        cu_kv[1:] = ctx_l.cumsum(0)
        tcl = int(cu_kv[-1])
        kc = torch.randn((H * tcl, D), generator=g).to(dt).to(device)
        vc = torch.randn((H * tcl, D), generator=g).to(dt).to(device)
        cache.prefill_kv_cache(0, k_cache=kc, v_cache=vc, total_context_len=tcl, cu_seqlens_kv=cu_kv.to(device),
                               context_batch_size=B, is_mla=False, num_heads=H, head_dim=D)
    elif C:
        per_seq = config == "5a"
        nctx = B if per_seq else 1
        cu_kv = torch.arange(nctx + 1, dtype=torch.int32) * C
        kc = torch.randn((H * C * nctx, D), generator=g).to(dt).to(device)
        vc = torch.randn((H * C * nctx, D), generator=g).to(dt).to(device)
        cache.prefill_kv_cache(0, k_cache=kc, v_cache=vc, total_context_len=C * nctx, cu_seqlens_kv=cu_kv.to(device),
                               context_batch_size=nctx, is_mla=False, num_heads=H, head_dim=D)
    meta = flash_mlm.build_pack_metadata(lengths.to(device), N, 64)
    scale = 1.0 / math.sqrt(D)
    return lambda: flash_mlm.flash_attn_mlm_compressed(q, k, v, num_heads=H, q_meta=meta, scale=scale,
                                                       inference_cache=cache, layer_id=0, block_n=64,
                                                       causal_query_seq_attn=causal)


def build_pack_op(op: str, device):
    """Config 2 shapes (B=32, H=16, N=512, D=64, bf16, lengths U[64,512])."""
    from flash_mlm.host import host_utils

    g = torch.Generator().manual_seed(0)
    B, H, N, D = 32, 16, 512, 64
    lengths = _lengths(g, B, 64, 512)
    meta = flash_mlm.build_pack_metadata(lengths.to(device), N, 64)
    if op == "append":
        # append the batch's K/V as 32 new entries of a reserved cache, emptied before each call
        k, v = (torch.randn((B, H, N, D), generator=g).to(torch.bfloat16).to(device) for _ in range(2))
        cache = flash_mlm.InferenceCache()
        cache.reserve_kv_cache(0, capacity=meta.total_tokens, max_entries=B, is_mla=False, num_heads=H, head_dim=D,
                               dtype=torch.bfloat16, device=device)

        def step():
            cache.reset_kv_cache(0)
            cache.append_kv_cache(0, k, v, meta)
        return step
    if op == "pack":
        q, k, v = (torch.randn((B, H, N, D), generator=g).to(torch.bfloat16).to(device) for _ in range(3))
        return lambda: host_utils.pack_and_pad_main_tensors_for_mlm_compressed(q, k, v, q_meta=meta, num_heads=H,
                                                                              is_mla=False, block_m=64, block_n=64)
    packed = torch.randn((H * meta.total_tokens, D), generator=g).to(torch.bfloat16).to(device)
    return lambda: flash_mlm.unpack_from_kernel(packed, meta, H)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="attn", choices=["attn", "pack", "unpack", "append"])
    ap.add_argument("--config", default="2")
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--iters", type=int, default=1)
    args = ap.parse_args()
    device = torch.device("cuda", 0)
    step = build(args.config, args.ctx, args.batch, device) if args.op == "attn" else build_pack_op(args.op, device)
    for _ in range(args.warmup + args.iters):
        step()
    torch.cuda.synchronize()
    flash_mlm.check_device_errors(device)
    print("profile_attn: done")


if __name__ == "__main__":
    main()
