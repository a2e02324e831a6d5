"""The allocation-free packed entry point against the regular one.

fmlm_attn_packed_fwd_noalloc serves callers that cannot allocate device
memory (graph capture, locked allocators, plugin hosts that only pass in
pre-allocated buffers): it keeps the tile schedule in a library-owned device
array instead of a caller workspace.  This test calls it through the C ABI
twice in a row, on two different workloads, and checks each result against
the regular entry point (which uses a caller workspace) within the attention
tolerance of the other GPU tests.  It sits in its own file so that pytest
collects it last.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 8e-3}


def _case(seed, lengths, H, N, D, ctx_len, dtype):
    import flash_mlm

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(seed)
    B = len(lengths)
    q, k, v = (torch.randn((B, H, N, D), generator=g).to(dtype).to(dev) for _ in range(3))
    cache = flash_mlm.InferenceCache()
    if ctx_len:
        kc = torch.randn((H * ctx_len, D), generator=g).to(dtype).to(dev)
        vc = torch.randn((H * ctx_len, D), generator=g).to(dtype).to(dev)
        cache.prefill_kv_cache(0, k_cache=kc, v_cache=vc, total_context_len=ctx_len,
                               cu_seqlens_kv=torch.tensor([0, ctx_len], dtype=torch.int32, device=dev),
                               context_batch_size=1, is_mla=False, num_heads=H, head_dim=D)
    meta = flash_mlm.build_pack_metadata(torch.tensor(lengths, dtype=torch.int32, device=dev), N, 64)
    return q, k, v, cache, meta


def _regular_then_args(q, k, v, cache, meta, H, D):
    """Run the regular entry point (public API) and return its output and argument block."""
    import flash_mlm
    from flash_mlm import _lib
    from flash_mlm.host import host as host_mod

    host_mod.record_packed_launches(True)
    try:
        ref = flash_mlm.flash_attn_mlm_compressed(q, k, v, num_heads=H, q_meta=meta, scale=1.0 / D ** 0.5,
                                                  inference_cache=cache, layer_id=0, block_n=64)
        args = _lib.PackedArgs.from_buffer_copy(host_mod.last_packed_launch[0])
    finally:
        host_mod.record_packed_launches(False)
    return ref, args


def test_noalloc_entry_matches_workspace_entry_on_two_calls_in_a_row():
    import flash_mlm
    from flash_mlm import _lib

    L = _lib.lib()
    dev = torch.device("cuda", 0)
    stream = _lib.stream_ptr(dev)
    cases = [
        ((3, [160, 37, 99], 4, 160, 64, 90, torch.bfloat16)),
        ((4, [300, 1, 129, 257, 64], 2, 300, 128, 0, torch.float16)),
    ]
    keep = []
    for seed, lengths, H, N, D, ctx_len, dtype in cases:
        q, k, v, cache, meta = _case(seed, lengths, H, N, D, ctx_len, dtype)
        ref, args = _regular_then_args(q, k, v, cache, meta, H, D)
        out = torch.full_like(ref, float("nan"))
        args.out = out.data_ptr()
        args.workspace = None
        args.workspace_bytes = 0
        _lib.check(L.fmlm_attn_packed_fwd_noalloc(ctypes.byref(args), stream), "fmlm_attn_packed_fwd_noalloc")
        torch.cuda.synchronize(dev)
        flash_mlm.check_device_errors(dev)
        err = (out.float() - ref.float()).abs().max().item()
        assert torch.isfinite(out.float()).all()
        assert err <= TOL[dtype], f"no-alloc vs workspace entry point: max abs diff {err:.3e}"
        # Both entry points run the same kernel on the same tile schedule.
        assert torch.equal(out, ref)
        keep.append((q, k, v, cache, meta, ref, out))


def test_noalloc_entry_rejects_problems_beyond_its_scratch():
    from flash_mlm import _lib

    L = _lib.lib()
    args = _lib.PackedArgs()
    args.dtype, args.head_dim, args.num_heads, args.batch = 1, 64, 1, 30000
    args.total_q_len = 30000 * 512
    rc = L.fmlm_attn_packed_fwd_noalloc(ctypes.byref(args), None)
    assert rc == -1
    assert "built-in scratch" in L.fmlm_last_error().decode()
