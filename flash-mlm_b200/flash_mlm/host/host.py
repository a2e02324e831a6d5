"""Host launchers of the flash-mlm forward path on B200.

``flash_attn_mlm``, ``flash_attn_mlm_compressed`` and
``flash_attn_mlm_precompressed`` keep the reference signatures, validation
order, error messages, cache semantics and return layouts
(src/flash_mlm/host/host.py:47-789).  Each launches the hand-written sm_100a
kernels of libflashmlm.so through the C ABI (include/flash_mlm.h):

* the compressed path reads q (and, when it can, k/v) straight from the
  padded [B, H, N, D] inputs and writes the trimmed packed output, so the
  reference's pack -> pad -> attention -> trim chain becomes one attention
  launch (plus a K/V pack when a prefill has to store packed K/V or when
  ``causal_query_seq_attn`` attends a packed prefix);
* query tiles are scheduled on the device from ``cu_seqlens`` (longest key
  range first) instead of from host tile maps.

``block_m``, ``block_n`` and ``auto_tune_tiles`` are accepted for API
compatibility: ``block_n`` is still checked against the metadata and
``block_m``/``block_n`` still decide the padded length of the K/V stored by a
prefill call; the kernels use their own fixed sm_100a tiling.
"""

from __future__ import annotations

import ctypes
import math

import torch

from flash_mlm import _lib
from flash_mlm.host.cache import BATCH_MAJOR, InferenceCache, PackMetadata, host_cu_seqlens
from flash_mlm.host.host_utils import (
    _compute_total_q_len_padded,
    _maybe_get_cache_context,
    _pack_flatten_for_kernel_into,
    make_contiguous,
    require_cuda_tensors,
    validate_cache_request,
    validate_cu_seqlens_rank1_min2,
    validate_head_dim_supported,
    validate_packed_cache_shapes,
    validate_qkv_same_shape_rank4,
)

def _validate_head_dim(d: int, is_mla: bool) -> None:
    """The reference whitelist {16, 32, 64, 128, 256} (host_utils.py:337-339), extended
    with 512 for MLA: the latent width of weight-absorbed MLA, which the B200
    kernel supports by splitting O into two 256-column halves."""
    if is_mla and d == 512:
        return
    validate_head_dim_supported(d)


# Largest reference autotune BLOCK_M (mlm_kernel.py:16); decides prefill padding under auto_tune_tiles.
_AUTO_TUNE_PAD_BLOCK_M = 128


def _cache_view(x: torch.Tensor | None, heads: int, rows: int, batch: int, total: int = 0) -> _lib.View4:
    """Flat rank-2 cache [batch * heads * rows, D] as a [batch][heads][rows] view."""
    if x is None or rows == 0 or x.numel() == 0:
        return _lib.view4(None)
    d = x.shape[1]
    rs = x.stride(0)
    return _lib.view4(x, rows=rows, heads=heads, batch=batch, row_stride=rs, head_stride=rows * rs,
                      batch_stride=heads * rows * rs)


def _heads_major_cache_view(x: torch.Tensor | None, heads: int, rows: int, batch: int, total: int) -> _lib.View4:
    """Head-major cache [heads * total, D] whose entry c sits at rows [c * rows, (c + 1) * rows)
    of each head, as a [batch][heads][rows] view (no copy)."""
    if x is None or rows == 0 or x.numel() == 0:
        return _lib.view4(None)
    rs = x.stride(0)
    return _lib.view4(x, rows=rows, heads=heads, batch=batch, row_stride=rs, head_stride=total * rs,
                      batch_stride=rows * rs)


def _workspace(device: torch.device, nbytes: int, cache: InferenceCache | None) -> torch.Tensor:
    rows = (nbytes + 15) // 16
    if cache is not None:
        return cache.packing.get_2d("fmlm:schedule", rows, 4, dtype=torch.int32, device=device)
    return torch.empty((rows, 4), dtype=torch.int32, device=device)


def flash_attn_mlm(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float,
    inference_cache: InferenceCache | None = None,
    layer_id: int | str | None = None,
    is_mla: bool = False,
    context_batch_size: int | None = None,
    block_m: int = 64,
    block_n: int = 32,
    auto_tune_tiles: bool = False,
    prefill: bool = False,
) -> torch.Tensor:
    """Dense (non-packed) MLM attention.

    q, k, v: [B, H, N, D].  Cached context (from ``inference_cache``) is a flat
    rank-2 tensor: MLA [total_context_tokens, D], otherwise
    [H * total_context_tokens, D].  Every query attends to its context (shared
    when ``context_batch_size == 1``) followed by all N tokens of its own
    (batch, head) sequence.  With ``prefill=True`` the context is skipped and
    this call's K/V become the layer's cached context.

    Returns [B, H, N, D] in q's dtype.
    """
    b, h, n, d = validate_qkv_same_shape_rank4(q, k, v, error_prefix="q/k/v")
    validate_cache_request(prefill=prefill, inference_cache=inference_cache, layer_id=layer_id)
    use_layer_cache = inference_cache is not None
    ctx = _maybe_get_cache_context(inference_cache=inference_cache, layer_id=layer_id, batch_size=b, is_mla=is_mla,
                                   num_heads=h, head_dim=d, context_batch_size=context_batch_size, dtype=q.dtype,
                                   device=q.device, compressed=False)
    k_cache, v_cache = ctx.k_cache, ctx.v_cache
    context_batch_size = ctx.context_batch_size
    context_len = ctx.context_len
    require_cuda_tensors(q, k, v, k_cache, v_cache)
    if context_batch_size is None or context_batch_size < 1:
        raise ValueError("context_batch_size must be >= 1")
    _validate_head_dim(d, is_mla)
    q, k, v, k_cache, v_cache = make_contiguous(q, k, v, k_cache, v_cache)
    out = torch.empty_like(q)

    has_ctx = (not prefill) and context_len > 0
    ctx_heads = 1 if is_mla else h
    args = _lib.DenseArgs()
    args.dtype = _lib.dtype_code(q.dtype)
    args.head_dim = d
    args.batch, args.num_heads, args.seq_len = b, h, n
    args.is_mla = int(is_mla)
    args.prefill = int(prefill)
    args.context_batch_size = context_batch_size
    args.context_len = context_len if has_ctx else 0
    args.scale = float(scale)
    args.q, args.k, args.v = _lib.view_bhnd(q), _lib.view_bhnd(k), _lib.view_bhnd(v)
    if has_ctx:
        view = _cache_view if ctx.layout == BATCH_MAJOR else _heads_major_cache_view
        total = int(ctx.total_context_len)
        args.k_cache = view(k_cache, ctx_heads, context_len, context_batch_size, total)
        args.v_cache = view(k_cache if is_mla else v_cache, ctx_heads, context_len, context_batch_size, total)
    args.out = out.data_ptr()
    args.error_word = _lib.error_word(q.device).data_ptr()
    if out.numel():
        with torch.cuda.device(q.device):
            _lib.check(_lib.lib().fmlm_attn_dense_fwd(ctypes.byref(args), _lib.stream_ptr(q.device)), "flash_attn_mlm")

    if prefill and use_layer_cache:
        # Dense prefill stores flattened K/V with uniform per-batch context len n (host.py:206-223).
        if is_mla:
            k_prefill = k[:, 0, :, :].contiguous().view(b * n, d)
            v_prefill = k_prefill
        else:
            k_prefill = k.contiguous().view(b * h * n, d)
            v_prefill = v.contiguous().view(b * h * n, d)
        inference_cache._store_dense_prefill(layer_id, k_cache=k_prefill, v_cache=v_prefill,
                                             context_batch_size=int(b), is_mla=is_mla, num_heads=h, head_dim=d)
    return out


def _packed_launch(*, q_view, k_view, v_view, q_layout, kv_layout, seq_len, total_q_len, num_heads, batch, d,
                   dtype, is_mla, prefill, causal, ctx, scale, cu_seqlens_q, out, out_rows_per_head, cache, device,
                   context_index=None, owners=(), out_padded=False):
    total_context_len = int(ctx.total_context_len)
    has_ctx = (not prefill) and total_context_len > 0
    ctx_heads = 1 if is_mla else num_heads
    args = _lib.PackedArgs()
    args.dtype = _lib.dtype_code(dtype)
    args.head_dim = d
    args.num_heads = num_heads
    args.batch = batch
    args.is_mla = int(is_mla)
    args.prefill = int(prefill)
    args.causal_query_seq_attn = int(causal)
    args.context_batch_size = int(ctx.context_batch_size)
    args.scale = float(scale)
    args.q_layout, args.kv_layout = q_layout, kv_layout
    args.seq_len = seq_len
    args.total_q_len = total_q_len
    args.q, args.k, args.v = q_view, k_view, v_view
    kc = vc = None
    if has_ctx:
        kc = ctx.k_cache.contiguous()
        vc = kc if is_mla else ctx.v_cache.contiguous()
        args.k_cache = _cache_view(kc, ctx_heads, total_context_len, 1)
        args.v_cache = _cache_view(vc, ctx_heads, total_context_len, 1)
        args.cu_seqlens_kv = ctx.cu_seqlens_kv.contiguous().data_ptr()
        if context_index is not None:
            args.context_index = context_index.data_ptr()
    args.cu_seqlens_q = cu_seqlens_q.data_ptr()
    args.out = out.data_ptr()
    args.out_rows_per_head = out_rows_per_head
    args.out_padded = int(out_padded)
    L = _lib.lib()
    nbytes = L.fmlm_packed_workspace_bytes(batch, total_q_len, d)
    if cache is not None:
        # A repeated call with the same offsets tensors reuses its device tile
        # schedule instead of rebuilding it.
        key_tensors = (cu_seqlens_q, ctx.cu_seqlens_kv) if has_ctx else (cu_seqlens_q,)
        if has_ctx and context_index is not None:
            key_tensors = key_tensors + (context_index,)
        key_scalars = (device.type, device.index, d, batch, num_heads, total_q_len, int(has_ctx), int(causal),
                       context_index is not None,
                       int(ctx.context_batch_size) if has_ctx else 0, bool(out_padded))
        ws, cached = cache.packing.schedule_workspace(key_tensors, key_scalars, nbytes, device)
        args.reuse_schedule = int(cached)
    else:
        ws = _workspace(device, nbytes, None)
    args.workspace = ws.data_ptr()
    args.workspace_bytes = ws.numel() * 4
    args.error_word = _lib.error_word(device).data_ptr()
    with torch.cuda.device(device):
        _lib.check(L.fmlm_attn_packed_fwd(ctypes.byref(args), _lib.stream_ptr(device)), "flash_attn_mlm_compressed")
    if _record_launches:
        global last_packed_launch
        keep = (tuple(owners), cu_seqlens_q, out, kc, vc, ctx.cu_seqlens_kv, context_index)
        last_packed_launch = (_lib.PackedArgs.from_buffer_copy(args), ws, keep)
    return (ws,)


# Profilers and benchmarks can ask for the argument block of the most recent
# packed launch (record_packed_launches(True)) to re-issue exactly that kernel
# launch through the C ABI with reuse_schedule=1, e.g. to time the attention
# kernel alone.  The record holds the workspace and every tensor whose address
# the argument block carries, so those pointers stay valid while it is kept.
# Off by default: production calls keep nothing alive.
_record_launches = False
last_packed_launch = None


def record_packed_launches(on: bool = True) -> None:
    """Keep (or stop keeping, and drop) the last packed launch's arguments and buffers."""
    global _record_launches, last_packed_launch
    _record_launches = bool(on)
    if not on:
        last_packed_launch = None


def flash_attn_mlm_compressed(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    num_heads: int,
    q_meta: PackMetadata,
    scale: float,
    inference_cache: InferenceCache | None = None,
    layer_id: int | str | None = None,
    is_mla: bool = False,
    context_batch_size: int | None = None,
    block_m: int = 64,
    block_n: int = 32,
    auto_tune_tiles: bool = False,
    prefill: bool = False,
    causal_query_seq_attn: bool = False,
    context_index: torch.Tensor | None = None,
    out_layout: str = "packed",
) -> torch.Tensor:
    """Packed variable-length MLM attention.

    q, k, v: padded [B, H, N, D]; only the first ``q_meta.lengths[b]`` tokens
    of sequence b are valid.  Each valid query attends to its context segment
    (``cu_seqlens_kv`` of the cached entry; shared when the context batch size
    is 1) followed by its own tokens, or, with ``causal_query_seq_attn``, by
    the tokens of all sequences up to and including its own.  MLA uses
    ``k[:, 0]`` as both key and value.  With ``prefill=True`` the context is
    skipped and this call's packed, padded K/V become the layer's context
    (``cu_seqlens_kv`` = ``q_meta.cu_seqlens``).

    ``context_index`` (optional, int32 [B] on q's device) maps query sequence
    b to context entry ``context_index[b]`` of the cached layer (index-mapped
    context batching, listed as planned in the reference README): any number
    of query sequences may share any entry.  It needs a cached context, is not
    combined with ``prefill`` or an explicit ``context_batch_size``, and costs
    one device read to range-check the indices.

    ``out_layout`` (beyond the reference): "packed" returns the packed output
    [H * total_tokens, D] in q's dtype; "padded" returns [B, H, N, D] with
    zero rows past each sequence -- what ``unpack_from_kernel`` would make of
    the packed output, bit for bit -- written directly by the attention
    kernel's epilogue (no separate unpack pass).
    """
    b, h, n, d = validate_qkv_same_shape_rank4(q, k, v, error_prefix="q/k/v")
    if h != num_heads:
        raise ValueError("q/k/v head dimension must match num_heads")
    validate_cache_request(prefill=prefill, inference_cache=inference_cache, layer_id=layer_id)
    if q_meta.B != b or q_meta.N != n:
        raise ValueError("q_meta shape metadata does not match q/k/v padded shape")
    total_tokens = q_meta.total_tokens
    if q_meta.batch_ids_block_n != block_n:
        raise ValueError("q_meta was built with different block_n")
    cu_seqlens_q = q_meta.cu_seqlens
    if out_layout not in ("packed", "padded"):
        raise ValueError('out_layout must be "packed" or "padded"')
    out_padded = out_layout == "padded"
    if context_index is not None:
        if prefill:
            raise ValueError("context_index cannot be combined with prefill=True")
        if inference_cache is None:
            raise ValueError("context_index requires inference_cache and layer_id")
        if context_batch_size is not None:
            raise ValueError("context_index selects context entries itself; leave context_batch_size unset")
        if (not isinstance(context_index, torch.Tensor) or context_index.dtype != torch.int32
                or tuple(context_index.shape) != (b,)):
            raise ValueError("context_index must be an int32 tensor of shape [B]")
        if context_index.device != q.device:
            raise ValueError("context_index must be on q's device")

    use_layer_cache = inference_cache is not None
    ctx = _maybe_get_cache_context(inference_cache=inference_cache, layer_id=layer_id, batch_size=b, is_mla=is_mla,
                                   num_heads=num_heads, head_dim=d, context_batch_size=context_batch_size,
                                   dtype=q.dtype, device=q.device, compressed=True)
    require_cuda_tensors(q, k, v, ctx.k_cache, ctx.v_cache, ctx.cu_seqlens_kv)
    if not cu_seqlens_q.is_cuda or not q_meta.batch_ids_q.is_cuda:
        raise ValueError("batch_ids_q and cu_seqlens_q must be CUDA tensors")
    if num_heads < 1:
        raise ValueError("num_heads must be >= 1")
    validate_packed_cache_shapes(ctx.k_cache, ctx.v_cache, num_heads=num_heads,
                                 total_context_len=int(ctx.total_context_len), head_dim=d, is_mla=is_mla)
    _validate_head_dim(d, is_mla)
    validate_cu_seqlens_rank1_min2(cu_seqlens_q, ctx.cu_seqlens_kv)
    if ctx.context_batch_size < 1:
        raise ValueError("context_batch_size must be >= 1")
    if ctx.context_batch_size + 1 > ctx.cu_seqlens_kv.numel():
        raise ValueError("context_batch_size is incompatible with cu_seqlens_kv length")
    if context_index is not None and int(ctx.total_context_len) > 0:
        lo, hi = (int(x) for x in torch.stack(torch.aminmax(context_index)).tolist())
        if lo < 0 or hi >= ctx.context_batch_size:
            raise ValueError(f"context_index values must lie in [0, {ctx.context_batch_size})")
        context_index = context_index.contiguous()

    cu_seqlens_q = cu_seqlens_q.contiguous()
    k_main = k[:, :1] if is_mla else k
    if q.stride(-1) != 1:
        q = q.contiguous()
    if k_main.stride(-1) != 1:
        k_main = k_main.contiguous()
    if not is_mla and v.stride(-1) != 1:
        v = v.contiguous()

    if out_padded:
        out = torch.empty((b, num_heads, n, d), dtype=q.dtype, device=q.device)
    else:
        out = torch.empty((num_heads * total_tokens, d), dtype=q.dtype, device=q.device)
    if total_tokens == 0:
        if out_padded:
            out.zero_()
        if prefill and use_layer_cache:
            _store_prefill(k, v, q_meta, num_heads, is_mla, block_m, block_n, auto_tune_tiles, inference_cache,
                           layer_id, d)
        return out

    need_packed_kv = prefill or causal_query_seq_attn
    if need_packed_kv:
        pad_block_m = _AUTO_TUNE_PAD_BLOCK_M if auto_tune_tiles else block_m
        if prefill and use_layer_cache:
            k_pk, v_pk, total_padded = _store_prefill(k, v, q_meta, num_heads, is_mla, block_m, block_n,
                                                      auto_tune_tiles, inference_cache, layer_id, d)
        else:
            total_padded = _compute_total_q_len_padded(total_tokens, host_cu_seqlens(q_meta), pad_block_m, block_n)
            k_pk, v_pk = _pack_main_kv(k, v, q_meta, num_heads, is_mla, total_padded,
                                       inference_cache.packing if inference_cache is not None else None, "k", "v")
        kv_heads = 1 if is_mla else num_heads
        k_view = _lib.view_packed(k_pk, kv_heads)
        v_view = _lib.view_packed(v_pk, kv_heads)
        k_view_src, v_view_src = k_pk, v_pk
        kv_layout = _lib.FMLM_LAYOUT_PACKED
        kv_rows = total_padded
    else:
        k_view = _lib.view_bhnd(k_main)
        v_view = _lib.view_bhnd(k_main if is_mla else v)
        k_view_src, v_view_src = k_main, (k_main if is_mla else v)
        kv_layout = _lib.FMLM_LAYOUT_PADDED
        kv_rows = total_tokens

    keep = _packed_launch(q_view=_lib.view_bhnd(q), k_view=k_view, v_view=v_view, q_layout=_lib.FMLM_LAYOUT_PADDED,
                          kv_layout=kv_layout, seq_len=n, total_q_len=max(kv_rows, total_tokens),
                          num_heads=num_heads, batch=b, d=d, dtype=q.dtype, is_mla=is_mla, prefill=prefill,
                          causal=causal_query_seq_attn, ctx=ctx, scale=scale, cu_seqlens_q=cu_seqlens_q, out=out,
                          out_rows_per_head=total_tokens, cache=inference_cache, device=q.device,
                          context_index=context_index, owners=(q, k_view_src, v_view_src),
                          out_padded=out_padded)
    del keep
    return out


def _pack_main_kv(k, v, q_meta, num_heads, is_mla, total_padded, packing, k_name, v_name):
    d = k.shape[3]

    def alloc(name, rows, template):
        if packing is None:
            return torch.empty((rows, d), dtype=template.dtype, device=template.device)
        return packing.get_2d(name, rows, d, dtype=template.dtype, device=template.device)

    if is_mla:
        k_src = k[:, :1, :, :]
        k_pk = _pack_flatten_for_kernel_into(k_src, q_meta, 1, total_padded, alloc(k_name, total_padded, k_src))
        return k_pk, k_pk
    k_pk = _pack_flatten_for_kernel_into(k, q_meta, num_heads, total_padded, alloc(k_name, num_heads * total_padded, k))
    v_pk = _pack_flatten_for_kernel_into(v, q_meta, num_heads, total_padded, alloc(v_name, num_heads * total_padded, v))
    return k_pk, v_pk


def _store_prefill(k, v, q_meta, num_heads, is_mla, block_m, block_n, auto_tune_tiles, cache, layer_id, d):
    """Pack this call's K/V into the layer's cache and register them (host.py:327-364).

    A layer with a reserved cache (``InferenceCache.reserve_kv_cache``) is
    emptied and receives the rows through one device append, with no new
    buffer; otherwise the K/V are packed into the layer's named workspaces,
    padded as the reference pads them."""
    r = cache.reserved(layer_id)
    if r is not None and r.is_mla == bool(is_mla) and r.head_dim == d and r.k.dtype == k.dtype \
            and r.k.device == k.device and (is_mla or r.num_heads == num_heads):
        cache.reset_kv_cache(layer_id)
        cache.append_kv_cache(layer_id, k, None if is_mla else v, q_meta)
        return r.k, (r.k if is_mla else r.v), r.capacity
    pad_block_m = _AUTO_TUNE_PAD_BLOCK_M if auto_tune_tiles else block_m
    total_padded = _compute_total_q_len_padded(q_meta.total_tokens, host_cu_seqlens(q_meta), pad_block_m, block_n)
    key = str(layer_id)
    k_pk, v_pk = _pack_main_kv(k, v, q_meta, num_heads, is_mla, total_padded, cache.packing,
                               f"layer:{key}:k_cache", f"layer:{key}:v_cache")
    cache._store_packed_prefill(layer_id, k_cache=k_pk, v_cache=None if is_mla else v_pk,
                                total_context_len=int(total_padded), cu_seqlens_kv=q_meta.cu_seqlens,
                                context_batch_size=int(q_meta.B), is_mla=is_mla, num_heads=num_heads, head_dim=d)
    return k_pk, v_pk, total_padded


def flash_attn_mlm_precompressed(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    num_heads: int,
    total_q_len: int,
    cu_seqlens_q: torch.Tensor,
    batch_ids_q: torch.Tensor,
    q_tile_starts_q: torch.Tensor,
    scale: float,
    inference_cache: InferenceCache | None = None,
    layer_id: int | str | None = None,
    is_mla: bool = False,
    context_batch_size: int | None = None,
    block_m: int = 64,
    block_n: int = 32,
    auto_tune_tiles: bool = False,
    prefill: bool = False,
    causal_query_seq_attn: bool = False,
) -> torch.Tensor:
    """Packed attention on already packed rank-2 inputs.

    q: [H * total_q_len, D]; k, v: [total_q_len, D] (MLA) or [H * total_q_len, D].
    ``batch_ids_q`` / ``q_tile_starts_q`` are validated for shape as in the
    reference; the device scheduler derives tiles from ``cu_seqlens_q``.
    Rows of the output that belong to no sequence are left unwritten, as in
    the reference.  Returns [H * total_q_len, D].
    """
    validate_cache_request(prefill=prefill, inference_cache=inference_cache, layer_id=layer_id)
    if q.ndim != 2 or k.ndim != 2 or v.ndim != 2:
        raise ValueError("q/k/v must be pre-packed rank-2 tensors")
    d = q.shape[1]
    if k.shape[1] != d or v.shape[1] != d:
        raise ValueError("q/k/v head_dim (dim 1) must match")
    if q.shape[0] != num_heads * total_q_len:
        raise ValueError("q first dim must equal num_heads * total_q_len")
    expected_main_rows = total_q_len if is_mla else num_heads * total_q_len
    if k.shape[0] != expected_main_rows or v.shape[0] != expected_main_rows:
        raise ValueError(f"k/v first dim mismatch: expected {expected_main_rows} rows for is_mla={is_mla}")
    batch = int(cu_seqlens_q.numel()) - 1
    ctx = _maybe_get_cache_context(inference_cache=inference_cache, layer_id=layer_id, batch_size=batch,
                                   is_mla=is_mla, num_heads=num_heads, head_dim=d,
                                   context_batch_size=context_batch_size, dtype=q.dtype, device=q.device,
                                   compressed=True)
    require_cuda_tensors(q, k, v, ctx.k_cache, ctx.v_cache, ctx.cu_seqlens_kv)
    validate_packed_cache_shapes(ctx.k_cache, ctx.v_cache, num_heads=num_heads,
                                 total_context_len=int(ctx.total_context_len), head_dim=d, is_mla=is_mla)
    _validate_head_dim(d, is_mla)
    validate_cu_seqlens_rank1_min2(cu_seqlens_q, ctx.cu_seqlens_kv)
    if ctx.context_batch_size < 1:
        raise ValueError("context_batch_size must be >= 1")
    if ctx.context_batch_size + 1 > ctx.cu_seqlens_kv.numel():
        raise ValueError("context_batch_size is incompatible with cu_seqlens_kv length")
    num_q_tiles = int(q_tile_starts_q.numel())
    if batch_ids_q.ndim != 1 or batch_ids_q.numel() != num_q_tiles:
        raise ValueError("batch_ids_q must be rank-1 with exactly one entry per query tile")
    if q_tile_starts_q.ndim != 1:
        raise ValueError("q_tile_starts_q must be rank-1")
    require_cuda_tensors(cu_seqlens_q, message="cu_seqlens_q must be a CUDA tensor")
    q, k, v, cu_seqlens_q = make_contiguous(q, k, v, cu_seqlens_q)
    out = torch.empty_like(q)
    if q.numel() and batch > 0:
        kv_heads = 1 if is_mla else num_heads
        keep = _packed_launch(q_view=_lib.view_packed(q, num_heads), k_view=_lib.view_packed(k, kv_heads),
                              v_view=_lib.view_packed(k if is_mla else v, kv_heads),
                              q_layout=_lib.FMLM_LAYOUT_PACKED, kv_layout=_lib.FMLM_LAYOUT_PACKED, seq_len=0,
                              total_q_len=int(total_q_len), num_heads=num_heads, batch=batch, d=d, dtype=q.dtype,
                              is_mla=is_mla, prefill=prefill, causal=causal_query_seq_attn, ctx=ctx, scale=scale,
                              cu_seqlens_q=cu_seqlens_q.to(torch.int32), out=out,
                              out_rows_per_head=int(total_q_len), cache=inference_cache, device=q.device,
                              owners=(q, k, v))
        del keep
    if prefill and inference_cache is not None:
        inference_cache._store_packed_prefill(layer_id, k_cache=k, v_cache=None if is_mla else v,
                                              total_context_len=int(total_q_len), cu_seqlens_kv=cu_seqlens_q,
                                              context_batch_size=batch, is_mla=is_mla, num_heads=num_heads,
                                              head_dim=d)
    return out
