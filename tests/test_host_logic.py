"""Host-side logic on CPU: cache bookkeeping, cache-context resolution,
validation messages (mirroring src/flash_mlm/host/test_host_utils.py and the
error cases of test_host.py), and the C-ABI library surface."""

import re
from pathlib import Path

import pytest
import torch

from flash_mlm.host.cache import InferenceCache, PackingCache
from flash_mlm.host.host_utils import (
    _compute_total_q_len_padded,
    _maybe_get_cache_context,
    validate_cache_request,
    validate_head_dim_supported,
)

ROOT = Path(__file__).resolve().parent.parent
CPU = torch.device("cpu")


def test_packing_cache_reuses_allocation_for_smaller_rows():
    cache = PackingCache()
    first = cache.get_2d("q", rows=8, cols=4, dtype=torch.float32, device=CPU)
    second = cache.get_2d("q", rows=6, cols=4, dtype=torch.float32, device=CPU)
    assert first.untyped_storage().data_ptr() == second.untyped_storage().data_ptr()
    assert second.shape == (6, 4)
    third = cache.get_2d("q", rows=16, cols=4, dtype=torch.float32, device=CPU)
    assert third.shape == (16, 4)
    with pytest.raises(ValueError, match="rows must be >= 0"):
        cache.get_2d("q", rows=-1, cols=4, dtype=torch.float32, device=CPU)
    with pytest.raises(ValueError, match="cols must be >= 1"):
        cache.get_2d("q", rows=1, cols=0, dtype=torch.float32, device=CPU)


def _mla_cache():
    cache = InferenceCache()
    cu = torch.tensor([0, 2, 5, 7], dtype=torch.int32)
    k = torch.arange(7 * 4, dtype=torch.float32).view(7, 4)
    cache.prefill_kv_cache(0, k_cache=k, v_cache=None, total_context_len=7, cu_seqlens_kv=cu,
                           context_batch_size=3, is_mla=True, num_heads=2, head_dim=4)
    return cache, k, cu


def test_cache_context_multi_batch_compressed():
    cache, k, cu = _mla_cache()
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id=0, batch_size=5, num_heads=2, head_dim=4,
                                   is_mla=True, context_batch_size=3, device=CPU, dtype=torch.float32,
                                   compressed=True)
    assert ctx.context_batch_size == 3 and ctx.total_context_len == 7 and ctx.k_cache is k
    torch.testing.assert_close(ctx.cu_seqlens_kv, cu)


def test_cache_context_shared_compressed():
    cache, k, _ = _mla_cache()
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id=0, batch_size=5, num_heads=2, head_dim=4,
                                   is_mla=True, context_batch_size=1, device=CPU, dtype=torch.float32,
                                   compressed=True)
    assert ctx.context_batch_size == 1 and ctx.k_cache is k
    torch.testing.assert_close(ctx.cu_seqlens_kv, torch.tensor([0, 7], dtype=torch.int32))


def test_cache_context_shared_dense():
    cache = InferenceCache()
    k = torch.arange(12 * 4, dtype=torch.float32).view(12, 4)
    v = k + 1000
    cache.prefill_kv_cache(0, k_cache=k, v_cache=v, total_context_len=6, context_batch_size=3, is_mla=False,
                           num_heads=2, head_dim=4)
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id=0, batch_size=5, num_heads=2, head_dim=4,
                                   is_mla=False, context_batch_size=1, device=CPU, dtype=torch.float32,
                                   compressed=False)
    assert ctx.context_batch_size == 1 and ctx.context_len == 6 and ctx.k_cache is k and ctx.v_cache is v
    assert ctx.cu_seqlens_kv is None


def test_cache_context_miss_and_mismatch_give_empty_context():
    ctx = _maybe_get_cache_context(inference_cache=None, layer_id=None, batch_size=4, num_heads=2, head_dim=8,
                                   is_mla=False, context_batch_size=None, device=CPU, dtype=torch.float16,
                                   compressed=True)
    assert ctx.total_context_len == 0 and ctx.context_batch_size == 4
    assert ctx.cu_seqlens_kv.tolist() == [0, 0, 0, 0, 0]
    cache, _, _ = _mla_cache()
    # wrong head_dim -> the entry does not match -> empty context, like the reference
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id=0, batch_size=2, num_heads=2, head_dim=8,
                                   is_mla=True, context_batch_size=None, device=CPU, dtype=torch.float32,
                                   compressed=True)
    assert ctx.total_context_len == 0
    with pytest.raises(ValueError, match=r"context_batch_size \(2\) must match cached entry context_batch_size \(3\)"):
        _maybe_get_cache_context(inference_cache=cache, layer_id=0, batch_size=2, num_heads=2, head_dim=4,
                                 is_mla=True, context_batch_size=2, device=CPU, dtype=torch.float32,
                                 compressed=True)


def test_cache_context_uniform_synthesis_and_dense_rule():
    cache = InferenceCache()
    k = torch.zeros(2 * 9, 4)
    cache.prefill_kv_cache("L", k_cache=k, v_cache=k.clone(), context_batch_size=3, is_mla=False, num_heads=2,
                           head_dim=4)
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id="L", batch_size=3, num_heads=2, head_dim=4,
                                   is_mla=False, context_batch_size=None, device=CPU, dtype=torch.float32,
                                   compressed=True)
    assert ctx.cu_seqlens_kv.tolist() == [0, 3, 6, 9]
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id="L", batch_size=3, num_heads=2, head_dim=4,
                                   is_mla=False, context_batch_size=None, device=CPU, dtype=torch.float32,
                                   compressed=False)
    assert ctx.context_len == 3
    # buffers handed to prefill_kv_cache are read as the reference reads them (dense: [C][H][ctx])
    assert ctx.layout == "batch_major" and ctx.k_cache is k
    # an entry a packed prefill wrote is head-major and serves the dense path in place:
    # [H][3 * 3] rows, entry c at rows 3c of each head
    cache._store_packed_prefill("P", k_cache=k, v_cache=k.clone(), total_context_len=9,
                                cu_seqlens_kv=torch.tensor([0, 3, 6, 9], dtype=torch.int32), context_batch_size=3,
                                is_mla=False, num_heads=2, head_dim=4)
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id="P", batch_size=3, num_heads=2, head_dim=4,
                                   is_mla=False, context_batch_size=None, device=CPU, dtype=torch.float32,
                                   compressed=False)
    assert ctx.layout == "heads_major" and ctx.context_len == 3 and ctx.total_context_len == 9


def test_cache_layouts_seen_by_each_path():
    """Dense prefill entries are batch-major; head-major entries with uneven entries cannot serve the dense path."""
    cache = InferenceCache()
    k = torch.zeros(3 * 2 * 4, 8)
    cache._store_dense_prefill(1, k_cache=k, v_cache=k.clone(), context_batch_size=3, is_mla=False, num_heads=2,
                               head_dim=8)
    e = cache.get_kv_cache(1, is_mla=False, num_heads=2, head_dim=8, dtype=torch.float32, device=CPU)
    assert e.layout == "batch_major" and e.total_context_len == 12
    ctx = _maybe_get_cache_context(inference_cache=cache, layer_id=1, batch_size=3, num_heads=2, head_dim=8,
                                   is_mla=False, context_batch_size=None, device=CPU, dtype=torch.float32,
                                   compressed=False)
    assert ctx.layout == "batch_major" and ctx.context_len == 4
    # MLA and single-head caches have one layout: no conversion is ever needed
    cache._store_dense_prefill(2, k_cache=torch.zeros(6, 8), v_cache=None, context_batch_size=3, is_mla=True,
                               num_heads=4, head_dim=8)
    e2 = cache.get_kv_cache(2, is_mla=True, num_heads=4, head_dim=8, dtype=torch.float32, device=CPU)
    assert cache.as_heads_major(e2) is e2
    # uneven head-major entries: the dense path refuses them (reference message)
    cache._store_packed_prefill(3, k_cache=torch.zeros(2 * 8, 8), v_cache=torch.zeros(2 * 8, 8),
                                total_context_len=8, cu_seqlens_kv=torch.tensor([0, 2, 8], dtype=torch.int32),
                                context_batch_size=2, is_mla=False, num_heads=2, head_dim=8)
    with pytest.raises(ValueError, match="requires uniform per-batch context lengths"):
        _maybe_get_cache_context(inference_cache=cache, layer_id=3, batch_size=2, num_heads=2, head_dim=8,
                                 is_mla=False, context_batch_size=None, device=CPU, dtype=torch.float32,
                                 compressed=False)


def test_reserved_cache_bookkeeping_and_limits():
    from flash_mlm.host.cache import PackMetadata

    cache = InferenceCache()
    cache.reserve_kv_cache(0, capacity=10, max_entries=2, is_mla=False, num_heads=2, head_dim=8,
                           dtype=torch.float16, device=CPU)
    r = cache.reserved(0)
    assert r.k.shape == (20, 8) and r.v.shape == (20, 8) and r.cu.tolist() == [0, 0, 0]
    with pytest.raises(ValueError, match="No cached KV context"):
        cache.get_kv_cache(0, is_mla=False, num_heads=2, head_dim=8, dtype=torch.float16, device=CPU)

    def meta(lengths, N):
        cu = [0]
        for x in lengths:
            cu.append(cu[-1] + x)
        t = torch.tensor(cu, dtype=torch.int32)
        m = PackMetadata(B=len(lengths), N=N, lengths=torch.tensor(lengths, dtype=torch.int32), cu_seqlens=t,
                         token_indices=torch.zeros(0, dtype=torch.int64), total_tokens=cu[-1], batch_ids_block_n=4,
                         batch_ids_q=torch.zeros(0, dtype=torch.int32), q_tile_starts_q=torch.zeros(0, dtype=torch.int32))
        m._cu_host = cu
        return m

    k = torch.zeros(3, 2, 6, 8, dtype=torch.float16)
    with pytest.raises(ValueError, match="exceeds max_entries=2"):
        cache.append_kv_cache(0, k, k, meta([1, 1, 1], 6))
    with pytest.raises(ValueError, match="exceeds capacity=10"):
        cache.append_kv_cache(0, k[:2], k[:2], meta([6, 5], 6))
    with pytest.raises(ValueError, match="No reserved KV cache"):
        cache.append_kv_cache(9, k, k, meta([1, 1, 1], 6))
    cache.clear_layer(0)
    assert cache.reserved(0) is None


def test_inference_cache_validation_messages():
    c = InferenceCache()
    k = torch.zeros(6, 4)
    with pytest.raises(ValueError, match="context_batch_size must be >= 1"):
        c.prefill_kv_cache(0, k_cache=k, v_cache=k, context_batch_size=0, is_mla=False, num_heads=2, head_dim=4)
    with pytest.raises(ValueError, match="non-MLA cache requires v_cache"):
        c.prefill_kv_cache(0, k_cache=k, context_batch_size=1, is_mla=False, num_heads=2, head_dim=4)
    with pytest.raises(ValueError, match="k_cache second dim must match head_dim"):
        c.prefill_kv_cache(0, k_cache=k, v_cache=k, context_batch_size=1, is_mla=False, num_heads=2, head_dim=8)
    with pytest.raises(ValueError, match="non-MLA k_cache rows must be divisible by num_heads"):
        c.prefill_kv_cache(0, k_cache=torch.zeros(5, 4), v_cache=torch.zeros(5, 4), context_batch_size=1,
                           is_mla=False, num_heads=2, head_dim=4)
    with pytest.raises(ValueError, match="total_context_len must be divisible by context_batch_size"):
        c.prefill_kv_cache(0, k_cache=k, v_cache=k, context_batch_size=2, is_mla=False, num_heads=2, head_dim=4)
    with pytest.raises(ValueError, match="context_batch_size is incompatible with cu_seqlens_kv length"):
        c.prefill_kv_cache(0, k_cache=k, v_cache=k, total_context_len=3, cu_seqlens_kv=torch.tensor([0, 3]),
                           context_batch_size=2, is_mla=False, num_heads=2, head_dim=4)
    c.prefill_kv_cache(1, k_cache=k, v_cache=k, context_batch_size=1, is_mla=False, num_heads=2, head_dim=4)
    with pytest.raises(ValueError, match="No cached KV context for layer_id=9"):
        c.get_kv_cache(9, is_mla=False, num_heads=2, head_dim=4, dtype=torch.float32, device=CPU)
    with pytest.raises(ValueError, match="Cached num_heads does not match request"):
        c.get_kv_cache(1, is_mla=False, num_heads=3, head_dim=4, dtype=torch.float32, device=CPU)
    with pytest.raises(ValueError, match=r"Cached KV mode \(is_mla\) does not match request"):
        c.get_kv_cache(1, is_mla=True, num_heads=2, head_dim=4, dtype=torch.float32, device=CPU)
    c.clear_layer(1)
    with pytest.raises(ValueError, match="No cached KV context"):
        c.get_kv_cache(1, is_mla=False, num_heads=2, head_dim=4, dtype=torch.float32, device=CPU)


def test_request_validators():
    with pytest.raises(ValueError, match="prefill=True requires inference_cache"):
        validate_cache_request(prefill=True, inference_cache=None, layer_id=None)
    with pytest.raises(ValueError, match="must be provided together or both omitted"):
        validate_cache_request(prefill=False, inference_cache=InferenceCache(), layer_id=None)
    with pytest.raises(ValueError, match="HEAD_DIM must be one of"):
        validate_head_dim_supported(48)
    assert _compute_total_q_len_padded(6, [0, 4, 6], 4, 4) == 8
    assert _compute_total_q_len_padded(6, [0, 4, 6], 32, 32) == 36


def test_public_api_errors_before_any_device_work():
    import flash_mlm

    q = torch.zeros(2, 2, 16, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match="prefill=True requires inference_cache"):
        flash_mlm.flash_attn_mlm(q, q, q, scale=0.5, prefill=True)
    with pytest.raises(ValueError, match="q, k, v must have the same shape"):
        flash_mlm.flash_attn_mlm(q, q[:, :1], q, scale=0.5)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        flash_mlm.build_pack_metadata(torch.tensor([3, 4], dtype=torch.int32), 4, 2)
    with pytest.raises(ValueError, match="All tensors must be CUDA tensors"):
        flash_mlm.flash_attn_mlm(q, q, q, scale=0.5)


def test_library_loads_and_exports_every_declared_symbol():
    from flash_mlm import _lib

    L = _lib.lib()
    header = (ROOT / "include" / "flash_mlm.h").read_text()
    declared = re.findall(r"FMLM_API\s+[\w\s\*]+?\b(fmlm_\w+)\s*\(", header)
    assert len(declared) >= 10
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/flash_mlm.h but not exported"
    assert L.fmlm_version() >= 100
    assert L.fmlm_packed_workspace_bytes(32, 9000, 64) % 16 == 0


def test_c_abi_rejects_bad_arguments_without_a_gpu():
    import ctypes

    from flash_mlm import _lib

    L = _lib.lib()
    assert L.fmlm_attn_packed_fwd(None, None) == -1
    a = _lib.PackedArgs()
    a.dtype, a.head_dim, a.num_heads, a.batch = 1, 48, 2, 2
    a.out = 16
    assert L.fmlm_attn_packed_fwd(ctypes.byref(a), None) == -2
    assert "HEAD_DIM" in L.fmlm_last_error().decode()
    assert L.fmlm_build_pack_metadata(None, 2, 4, 0, None, None, None, None, None, None) == -1
    # negative or oversized packed sizes are rejected before any device work
    b = _lib.PackedArgs()
    b.dtype, b.head_dim, b.num_heads, b.batch = 1, 64, 2, 2
    b.out, b.error_word, b.cu_seqlens_q = 16, 16, 16
    b.q_layout = b.kv_layout = _lib.FMLM_LAYOUT_PACKED
    b.total_q_len = -5
    assert L.fmlm_attn_packed_fwd(ctypes.byref(b), None) == -1
    assert "total_q_len must be >= 0" in L.fmlm_last_error().decode()
    assert L.fmlm_attn_packed_fwd_noalloc(ctypes.byref(b), None) == -1
    b.total_q_len = 65536 * 128
    assert L.fmlm_attn_packed_fwd(ctypes.byref(b), None) == -1
    assert "65536 * 128" in L.fmlm_last_error().decode()


def test_schedule_workspace_memo_rules():
    """A schedule is reused only for the same offsets tensors at the same version and scalars."""
    from flash_mlm.host.cache import PackingCache

    pc = PackingCache()
    dev = torch.device("cpu")
    cu = torch.tensor([0, 5, 9], dtype=torch.int32)
    ws1, hit1 = pc.schedule_workspace((cu,), ("k", 1), 64, dev)
    ws2, hit2 = pc.schedule_workspace((cu,), ("k", 1), 64, dev)
    assert not hit1 and hit2 and ws2 is ws1
    # different scalars, an equal-valued but different tensor, or an in-place change: rebuild
    assert not pc.schedule_workspace((cu,), ("k", 2), 64, dev)[1]
    assert not pc.schedule_workspace((cu.clone(),), ("k", 1), 64, dev)[1]
    cu.add_(0)
    assert not pc.schedule_workspace((cu,), ("k", 1), 64, dev)[1]
    assert pc.schedule_workspace((cu,), ("k", 1), 64, dev)[1]
    # a larger workspace requirement does not reuse a smaller buffer
    assert not pc.schedule_workspace((cu,), ("k", 1), 4096, dev)[1]
    # bounded, least recently used dropped
    keep = [torch.zeros(2, dtype=torch.int32) for _ in range(PackingCache._MAX_SCHEDULES + 2)]
    for t in keep:
        pc.schedule_workspace((t,), ("k",), 64, dev)
    assert pc._store.size("schedule") == PackingCache._MAX_SCHEDULES
    assert not pc.schedule_workspace((keep[0],), ("k",), 64, dev)[1]
    pc.clear()
    assert pc._store.size("schedule") == 0
