"""Host utilities of the flash-mlm forward path: pack metadata, pack / pad /
unpack, cache-context resolution and argument validators.

Names, arguments, results and error messages follow the reference
(src/flash_mlm/host/host_utils.py).  Data movement runs in the CUDA library
(libflashmlm.so): metadata, pack, pad and unpack are single-pass kernels.
Only the small host-side decisions (validation, which cached context to use,
padding sizes) stay in Python.  CPU tensors are rejected: there is no CPU
implementation of any data path here.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import TYPE_CHECKING

import torch

from flash_mlm import _lib
from flash_mlm.host.cache import BATCH_MAJOR, HEADS_MAJOR, InferenceCache, LayerKVEntry, PackMetadata, host_cu_seqlens

if TYPE_CHECKING:
    from flash_mlm.host.cache import PackingCache, _Reserved


@dataclass
class CacheContext:
    k_cache: torch.Tensor
    v_cache: torch.Tensor | None
    context_batch_size: int
    context_len: int
    total_context_len: int
    cu_seqlens_kv: torch.Tensor | None
    # Dense path only: "batch_major" ([C][H][context_len] rows) or "heads_major"
    # ([H][total_context_len] rows, entry c at rows c * context_len of each head).
    layout: str = "batch_major"


# ---------------------------------------------------------------------------
# metadata (host_utils.py:27-130)


def _run_metadata(lengths_i32: torch.Tensor, N: int, block_n: int, want_tokens: bool):
    """Run the metadata kernel; returns (cu, token_indices | None, batch_ids, tile_starts, counters_host)."""
    device = lengths_i32.device
    B = int(lengths_i32.numel())
    n_tiles_cap = B * ((N + block_n - 1) // block_n) if N > 0 else 0
    cu = torch.empty(B + 1, dtype=torch.int32, device=device)
    tok = torch.empty(B * N if want_tokens else 0, dtype=torch.int64, device=device)
    bid = torch.empty(max(n_tiles_cap, 1), dtype=torch.int32, device=device)
    tst = torch.empty(max(n_tiles_cap, 1), dtype=torch.int32, device=device)
    counters = torch.empty(B + 5, dtype=torch.int32, device=device)
    L = _lib.lib()
    with torch.cuda.device(device):
        _lib.check(
            L.fmlm_build_pack_metadata(
                lengths_i32.data_ptr() if B else None, B, N, block_n, cu.data_ptr(),
                tok.data_ptr() if want_tokens and tok.numel() else None, bid.data_ptr(), tst.data_ptr(),
                counters.data_ptr(), _lib.stream_ptr(device)),
            "build_pack_metadata")
    host = torch.cat([counters[:3], cu]).to("cpu").tolist()  # one device read, like the reference's .item()
    return cu, tok, bid, tst, host


def build_pack_metadata(lengths: torch.Tensor, N: int, block_n: int) -> PackMetadata:
    """Offsets and index maps of a padded batch whose sequence b holds
    ``lengths[b]`` valid tokens out of ``N``.

    Runs one scan kernel and one fill kernel and reads the totals back once.
    The result carries int32 ``cu_seqlens`` [B+1], int64 ``token_indices``
    (flat b*N+t of every valid token), and the per-``block_n`` query tile map
    (``batch_ids_q``, ``q_tile_starts_q``) in the reference's exact order.
    """
    if lengths.ndim != 1:
        raise ValueError("lengths must be rank-1 [B]")
    if N < 0:
        raise ValueError("N must be >= 0")
    if block_n < 1:
        raise ValueError("block_n must be >= 1")
    _lib.require_cuda(lengths, what="build_pack_metadata")
    lengths_i32 = lengths.to(dtype=torch.int32).contiguous()
    cu, tok, bid, tst, host = _run_metadata(lengths_i32, N, block_n, want_tokens=True)
    total_tokens, n_tiles, bad = host[0], host[1], host[2]
    if bad:
        raise ValueError("lengths values must be in [0, N]")
    meta = PackMetadata(
        B=int(lengths_i32.numel()),
        N=N,
        lengths=lengths_i32,
        cu_seqlens=cu,
        token_indices=tok[:total_tokens],
        total_tokens=int(total_tokens),
        batch_ids_block_n=block_n,
        batch_ids_q=bid[:n_tiles],
        q_tile_starts_q=tst[:n_tiles],
    )
    meta._cu_host = [int(x) for x in host[3:]]
    return meta


def _build_query_tile_map_from_cu_seqlens(cu_seqlens_q: torch.Tensor, block_n: int):
    """Build per-batch query tile starts and tile-to-batch mapping (host_utils.py:74-107)."""
    if cu_seqlens_q.ndim != 1:
        raise ValueError("cu_seqlens_q must be rank-1")
    if cu_seqlens_q.numel() < 2:
        raise ValueError("cu_seqlens_q must have at least 2 elements")
    if block_n < 1:
        raise ValueError("block_n must be >= 1")
    _lib.require_cuda(cu_seqlens_q, what="_build_query_tile_map_from_cu_seqlens")
    cu_host = [int(x) for x in cu_seqlens_q.to("cpu").tolist()]
    lens = [b - a for a, b in zip(cu_host[:-1], cu_host[1:])]
    n_max = max(max(lens), 0)
    lengths = (cu_seqlens_q[1:] - cu_seqlens_q[:-1]).to(torch.int32).contiguous()
    _, _, bid, tst, host = _run_metadata(lengths, n_max, block_n, want_tokens=False)
    n_tiles = host[1]
    if n_tiles == 0:
        empty = torch.empty((0,), device=cu_seqlens_q.device, dtype=torch.int32)
        return empty, empty
    # Tile starts are relative to the given cu_seqlens (which need not start at 0).
    starts = tst[:n_tiles]
    if cu_host[0] != 0:
        starts = starts + cu_host[0]
    return starts.contiguous(), bid[:n_tiles].contiguous()


def build_batch_ids_from_cu_seqlens(cu_seqlens_q: torch.Tensor, block_n: int):
    """Sequence index of every ``block_n``-row query tile of a packed batch."""
    _, batch_ids = _build_query_tile_map_from_cu_seqlens(cu_seqlens_q, block_n)
    return batch_ids


def build_q_tile_starts_from_cu_seqlens(cu_seqlens_q: torch.Tensor, block_n: int):
    """Packed row at which every ``block_n``-row query tile starts."""
    q_tile_starts_q, _ = _build_query_tile_map_from_cu_seqlens(cu_seqlens_q, block_n)
    return q_tile_starts_q


def num_query_tiles_from_cu_seqlens(cu_seqlens_q: torch.Tensor, block_n: int) -> int:
    """Count of ``block_n``-row query tiles over all sequences of ``cu_seqlens_q``."""
    return int(build_q_tile_starts_from_cu_seqlens(cu_seqlens_q, block_n).numel())


def num_query_tiles_from_meta(meta: PackMetadata) -> int:
    """Count of query tiles in ``meta``'s precomputed tile map."""
    return int(meta.q_tile_starts_q.numel())


# ---------------------------------------------------------------------------
# validators (host_utils.py:142-153, :315-390)


def validate_cache_request(*, prefill: bool, inference_cache: InferenceCache | None,
                           layer_id: int | str | None) -> None:
    if prefill and inference_cache is None:
        raise ValueError("prefill=True requires inference_cache")
    if (inference_cache is None) != (layer_id is None):
        raise ValueError("inference_cache and layer_id must be provided together or both omitted")


def require_cuda_tensors(*tensors: torch.Tensor, message: str = "All tensors must be CUDA tensors"):
    if not all(t is None or t.is_cuda for t in tensors):
        raise ValueError(message)


def validate_qkv_same_shape_rank4(q, k, v, *, error_prefix: str) -> tuple[int, int, int, int]:
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError(f"{error_prefix} must be rank-4 tensors [B, H, N, D]")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("q, k, v must have the same shape")
    b, h, n, d = q.shape
    return int(b), int(h), int(n), int(d)


SUPPORTED_HEAD_DIMS = (16, 32, 64, 128, 256)


def validate_head_dim_supported(head_dim: int):
    if head_dim not in SUPPORTED_HEAD_DIMS:
        raise ValueError("HEAD_DIM must be one of {16, 32, 64, 128, 256}")


def validate_cu_seqlens_rank1_min2(*cu_seqlens: torch.Tensor):
    for x in cu_seqlens:
        if x.ndim != 1:
            raise ValueError("cu_seqlens tensors must be rank-1")
        if x.numel() < 2:
            raise ValueError("cu_seqlens tensors must have at least 2 elements")


def validate_packed_cache_shapes(k_cache, v_cache, *, num_heads: int, total_context_len: int, head_dim: int,
                                 is_mla: bool):
    if k_cache.ndim != 2:
        raise ValueError("k_cache must be a rank-2 packed tensor")
    if k_cache.shape[1] != head_dim:
        raise ValueError("k_cache second dim must match q/k/v head_dim")
    if is_mla:
        if v_cache is not None:
            if v_cache.ndim != 2:
                raise ValueError("MLA v_cache must be a rank-2 packed tensor")
            if v_cache.shape != k_cache.shape:
                raise ValueError("MLA v_cache shape must match k_cache shape")
    else:
        if v_cache is None:
            raise ValueError("non-MLA cache requires v_cache")
        if v_cache.ndim != 2:
            raise ValueError("v_cache must be a rank-2 packed tensor")
        if v_cache.shape != k_cache.shape:
            raise ValueError("v_cache shape must match k_cache shape")
        if v_cache.shape[1] != head_dim:
            raise ValueError("v_cache second dim must match q/k/v head_dim")
    expected = total_context_len if is_mla else num_heads * total_context_len
    if k_cache.shape[0] != expected:
        raise ValueError(f"k_cache first dim mismatch: expected {expected} rows for is_mla={is_mla}")
    if not is_mla and v_cache.shape[0] != expected:
        raise ValueError(f"v_cache first dim mismatch: expected {expected} rows for is_mla={is_mla}")


def make_contiguous(*tensors: torch.Tensor | None) -> tuple[torch.Tensor | None, ...]:
    return tuple(t if t is None else t.contiguous() for t in tensors)


# ---------------------------------------------------------------------------
# cache context (host_utils.py:156-263)


def _maybe_get_cache_context(*, inference_cache: InferenceCache | None, layer_id, batch_size: int, num_heads: int,
                             head_dim: int, is_mla: bool, context_batch_size: int | None, device: torch.device,
                             dtype: torch.dtype, compressed: bool) -> CacheContext:
    """Resolve the context K/V for a call (reference rules, host_utils.py:156-263).

    A missing or mismatching cache entry means "no context" (empty K/V).  A
    ``context_batch_size`` of 1 over a multi-entry cache selects one shared
    context covering every stored row.  The dense path needs a uniform
    context length.

    Beyond the reference, the row layout of the entry is honoured: the packed
    path reads a dense prefill's [C][H][ctx] entry through a head-major copy
    made once (``InferenceCache.as_heads_major``), and the dense path reads a
    head-major entry of uniform entries in place through its strides.  Where
    the two layouts coincide (MLA, one head or one entry) the reference's
    resolution is unchanged.
    """
    entry: LayerKVEntry | None = None
    if inference_cache is not None:
        try:
            entry = inference_cache.get_kv_cache(layer_id, is_mla=is_mla, num_heads=num_heads, head_dim=head_dim,
                                                 dtype=dtype, device=device)
        except ValueError:
            entry = None

    if entry is None:
        resolved = batch_size if context_batch_size is None else context_batch_size
        k_cache = torch.empty((0, head_dim), device=device, dtype=dtype)
        return CacheContext(k_cache=k_cache, v_cache=torch.empty_like(k_cache), context_batch_size=resolved,
                            context_len=0, total_context_len=0,
                            cu_seqlens_kv=torch.zeros(resolved + 1, device=device, dtype=torch.int32)
                            if compressed else None)

    stored = entry.context_batch_size
    if context_batch_size is None or context_batch_size == stored:
        resolved = stored
    elif context_batch_size == 1:
        resolved = 1
    else:
        raise ValueError(
            f"context_batch_size ({context_batch_size}) must match cached entry context_batch_size ({stored})"
        )
    if resolved < 1:
        raise ValueError("context_batch_size must be >= 1")

    # Layout matters only with several heads and several entries.
    layouts_differ = not is_mla and num_heads > 1 and stored > 1
    if compressed:
        return _packed_context(inference_cache, entry, resolved, layouts_differ, device)
    return _dense_context(inference_cache, entry, resolved, layouts_differ, is_mla, num_heads)


def _packed_context(cache, entry, resolved, layouts_differ, device) -> CacheContext:
    if layouts_differ and entry.layout == BATCH_MAJOR:
        entry = cache.as_heads_major(entry)
    total = int(entry.total_context_len)
    stored = entry.context_batch_size
    context_len = 0
    cu_kv = entry.cu_seqlens_kv
    if cu_kv is None:
        if total % stored != 0:
            raise ValueError("compressed path requires cu_seqlens_kv or uniform per-batch context lengths")
        context_len = total // stored
        cu_kv = torch.arange(stored + 1, device=device, dtype=torch.int32) * int(context_len)
    if resolved == 1 and stored != 1:
        cu_kv = torch.tensor([0, int(entry.used_context_len)], device=device, dtype=torch.int32)
    return CacheContext(k_cache=entry.k_cache, v_cache=entry.v_cache, context_batch_size=resolved,
                        context_len=context_len, total_context_len=total, cu_seqlens_kv=cu_kv,
                        layout=HEADS_MAJOR)


def _entry_offsets(entry: LayerKVEntry) -> list[int]:
    """Host copy of an entry's context offsets (one device read, memoised on the entry)."""
    if entry.cu_host is None:
        if entry.cu_seqlens_kv is None:
            step = int(entry.total_context_len) // entry.context_batch_size
            entry.cu_host = [c * step for c in range(entry.context_batch_size + 1)]
        else:
            entry.cu_host = [int(x) for x in entry.cu_seqlens_kv.to("cpu").tolist()]
    return entry.cu_host


def _dense_context(cache, entry, resolved, layouts_differ, is_mla, num_heads) -> CacheContext:
    stored = entry.context_batch_size
    layout = BATCH_MAJOR
    if layouts_differ and entry.layout == BATCH_MAJOR and resolved == 1:
        # one shared context over every stored row of a head: read it head-major
        entry = cache.as_heads_major(entry)
        layout = HEADS_MAJOR
    elif layouts_differ and entry.layout == HEADS_MAJOR and resolved == stored:
        # per-entry context from a head-major cache: uniform entries, read in place
        cu = _entry_offsets(entry)[: stored + 1]
        step = cu[1] - cu[0]
        if any(cu[c] != cu[0] + c * step for c in range(stored + 1)) or cu[0] != 0:
            raise ValueError("dense flash_attn_mlm requires uniform per-batch context lengths")
        return CacheContext(k_cache=entry.k_cache, v_cache=entry.v_cache, context_batch_size=resolved,
                            context_len=step, total_context_len=int(entry.total_context_len), cu_seqlens_kv=None,
                            layout=HEADS_MAJOR)
    elif entry.layout == HEADS_MAJOR and resolved == 1:
        layout = HEADS_MAJOR
    total = int(entry.total_context_len)
    if resolved == 1 and stored != 1:
        total = int(entry.used_context_len)
    if total % resolved != 0:
        raise ValueError("dense flash_attn_mlm requires uniform per-batch context lengths")
    context_len = total // resolved
    expected = int(entry.total_context_len) * (1 if is_mla else num_heads)
    if entry.k_cache.shape[0] != expected or (not is_mla and entry.v_cache.shape[0] != expected):
        raise ValueError("cached dense k/v rows mismatch expected layout for is_mla/num_heads")
    return CacheContext(k_cache=entry.k_cache, v_cache=entry.v_cache, context_batch_size=resolved,
                        context_len=context_len, total_context_len=int(entry.total_context_len),
                        cu_seqlens_kv=None, layout=layout)


# ---------------------------------------------------------------------------
# pack / pad / unpack (host_utils.py:266-312, :397-615)


def _elem_bytes(x: torch.Tensor) -> int:
    return x.element_size()


def _pack_into(x: torch.Tensor, meta: PackMetadata, heads: int, total_padded: int, out: torch.Tensor) -> torch.Tensor:
    """Gather valid rows of padded x [B, heads, N, D] into out [heads * total_padded, D] (zero pad rows)."""
    _lib.require_cuda(x, out, meta.cu_seqlens, what="pack")
    if x.stride(-1) != 1:
        x = x.contiguous()
    if out.dtype != x.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of x's dtype")
    v = _lib.view_bhnd(x)
    with torch.cuda.device(x.device):
        _lib.check(
            _lib.lib().fmlm_pack_rows(ctypes.byref(v), _elem_bytes(x), x.shape[3], meta.cu_seqlens.data_ptr(), meta.B,
                                      meta.total_tokens, total_padded, out.data_ptr(), _lib.stream_ptr(x.device)),
            "pack")
    return out


def pack_for_kernel(x: torch.Tensor, meta: PackMetadata, flatten_for_kernel: bool = False):
    """Pack padded (B, H, N, D) into token-packed representation using cached indices.

    Returns:
        packed: (H, total_tokens, D) or (H * total_tokens, D) if flatten_for_kernel=True
    """
    if x.ndim != 4:
        raise ValueError("x must be rank-4 [B, H, N, D]")
    B, H, N, D = x.shape
    if B != meta.B or N != meta.N:
        raise ValueError("x shape mismatch with PackMetadata")
    out = torch.empty((H * meta.total_tokens, D), dtype=x.dtype, device=x.device)
    if out.numel():
        _pack_into(x, meta, H, meta.total_tokens, out)
    return out if flatten_for_kernel else out.view(H, meta.total_tokens, D)


def _compute_total_q_len_padded(total_q_len_unpadded: int, cu_seqlens_q: torch.Tensor | list[int], block_m: int,
                                block_n: int) -> int:
    """Rows per head after padding so every sequence's last tile of max(block_m, block_n) rows is in bounds."""
    align = max(block_m, block_n)
    cu = cu_seqlens_q if isinstance(cu_seqlens_q, list) else [int(x) for x in cu_seqlens_q.to("cpu").tolist()]
    need = 0
    for a, b in zip(cu[:-1], cu[1:]):
        need = max(need, a + ((b - a + align - 1) // align) * align)
    return max(total_q_len_unpadded, need)


def _pack_flatten_for_kernel_into(x: torch.Tensor, meta: PackMetadata, expected_heads: int,
                                  total_q_len_padded: int, out: torch.Tensor) -> torch.Tensor:
    if x.ndim != 4:
        raise ValueError("x must be rank-4 [B, H, N, D]")
    b, h, n, d = x.shape
    if b != meta.B or n != meta.N:
        raise ValueError("x shape mismatch with PackMetadata")
    if h != expected_heads:
        raise ValueError("x head dimension mismatch for requested packed output")
    if out.shape != (expected_heads * total_q_len_padded, d):
        raise ValueError("out has unexpected shape for packed output")
    if out.numel():
        _pack_into(x, meta, expected_heads, total_q_len_padded, out)
    return out


def pack_and_pad_main_tensors_for_mlm_compressed(q, k, v, *, q_meta: PackMetadata, num_heads: int, is_mla: bool,
                                                 block_m: int, block_n: int,
                                                 packing_cache: "PackingCache | None" = None,
                                                 q_buffer_name: str = "q", k_buffer_name: str = "k",
                                                 v_buffer_name: str = "v"):
    """Fused pack + pad into final flattened q/k/v buffers for compressed kernel."""
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q/k/v must be rank-4 padded tensors [B, H, N, D]")
    b, h, n, d = q.shape
    if q_meta.B != b or q_meta.N != n:
        raise ValueError("q_meta shape metadata does not match q/k/v padded shape")
    if h != num_heads:
        raise ValueError("q/k/v head dimension must match num_heads")
    total = _compute_total_q_len_padded(q_meta.total_tokens, host_cu_seqlens(q_meta), block_m, block_n)

    def alloc(name, rows, template):
        if packing_cache is None:
            return torch.empty((rows, d), dtype=template.dtype, device=template.device)
        return packing_cache.get_2d(name, rows, d, dtype=template.dtype, device=template.device)

    q_out = _pack_flatten_for_kernel_into(q, q_meta, num_heads, total, alloc(q_buffer_name, num_heads * total, q))
    if is_mla:
        k_src = k[:, :1, :, :]
        k_out = _pack_flatten_for_kernel_into(k_src, q_meta, 1, total, alloc(k_buffer_name, total, k_src))
        v_out = k_out
    else:
        k_out = _pack_flatten_for_kernel_into(k, q_meta, num_heads, total, alloc(k_buffer_name, num_heads * total, k))
        v_out = _pack_flatten_for_kernel_into(v, q_meta, num_heads, total, alloc(v_buffer_name, num_heads * total, v))
    return q_out, k_out, v_out, total


def pad_packed_main_tensors_for_mlm_compressed(q, k, v, *, num_heads: int, is_mla: bool, total_q_len_unpadded: int,
                                               cu_seqlens_q: torch.Tensor, block_m: int, block_n: int,
                                               packing_cache: "PackingCache | None" = None):
    """Pad flattened packed main q/k/v rows for descriptor-safe tile loads.

    q is [heads * packed_len, D]; k/v are [heads * packed_len, D] (non-MLA) or
    [packed_len, D] (MLA).  Returns the inputs unchanged when no padding is needed.
    """
    total = _compute_total_q_len_padded(total_q_len_unpadded, cu_seqlens_q, block_m, block_n)
    if total == total_q_len_unpadded:
        return q, k, v, total_q_len_unpadded
    kv_heads = 1 if is_mla else num_heads

    def pad(x, heads, name):
        _lib.require_cuda(x, what="pad_packed_main_tensors_for_mlm_compressed")
        x = x.contiguous()
        d = x.shape[1]
        if packing_cache is None:
            out = torch.empty((heads * total, d), dtype=x.dtype, device=x.device)
        else:
            out = packing_cache.get_2d(name, heads * total, d, dtype=x.dtype, device=x.device)
        with torch.cuda.device(x.device):
            _lib.check(_lib.lib().fmlm_pad_packed_rows(x.data_ptr(), total_q_len_unpadded, total, heads, d,
                                                       _elem_bytes(x), out.data_ptr(), _lib.stream_ptr(x.device)),
                       "pad_packed_rows")
        return out

    return pad(q, num_heads, "q"), pad(k, kv_heads, "k"), pad(v, kv_heads, "v"), total


def unpack_from_kernel(packed: torch.Tensor, meta: PackMetadata, H: int):
    """Unpack token-packed representation back to padded (B, H, N, D)."""
    if packed.ndim == 3:
        _, total_tokens, D = packed.shape
    elif packed.ndim == 2:
        total_tokens = meta.total_tokens
        D = packed.shape[1]
        if total_tokens != 0 and packed.shape[0] != H * total_tokens:
            raise ValueError("packed first dim must be H * total_tokens")
    else:
        raise ValueError("packed must be rank-2 or rank-3")
    if total_tokens != meta.total_tokens:
        raise ValueError("packed token count mismatch with PackMetadata")
    _lib.require_cuda(packed, meta.cu_seqlens, what="unpack_from_kernel")
    src = packed.contiguous()
    out = torch.empty((meta.B, H, meta.N, D), device=packed.device, dtype=packed.dtype)
    if out.numel():
        with torch.cuda.device(packed.device):
            _lib.check(
                _lib.lib().fmlm_unpack_rows(src.data_ptr() if src.numel() else None, total_tokens, H, D,
                                            _elem_bytes(src), meta.cu_seqlens.data_ptr(), meta.B, meta.N,
                                            out.data_ptr(), _lib.stream_ptr(packed.device)),
                "unpack_from_kernel")
    return out


# ---------------------------------------------------------------------------
# context-cache appends (no reference counterpart: the reference stores a new
# packed buffer per prefill, src/flash_mlm/host/host.py:327-364)


def _append_launch(k_view, v_view, src_layout, elem_bytes, d, cu, B, total, k_dst, v_dst, capacity, cu_kv,
                   entries_before, device):
    err = _lib.error_word(device)
    with torch.cuda.device(device):
        _lib.check(
            _lib.lib().fmlm_cache_append(ctypes.byref(k_view), ctypes.byref(v_view) if v_view is not None else None,
                                         src_layout, elem_bytes, d, cu.data_ptr(), B, total, k_dst.data_ptr(),
                                         v_dst.data_ptr() if v_dst is not None else None, capacity,
                                         cu_kv.data_ptr(), entries_before, err.data_ptr(),
                                         _lib.stream_ptr(device)),
            "fmlm_cache_append")


def append_rows_into_cache(k: torch.Tensor, v: torch.Tensor | None, meta: PackMetadata, r: "_Reserved") -> None:
    """Append the valid rows of padded k / v [B, H, N, D] to reserved cache ``r`` (one launch)."""
    _lib.require_cuda(k, v, meta.cu_seqlens, what="append_kv_cache")
    if meta.B != k.shape[0] or meta.N != k.shape[2]:
        raise ValueError("k shape mismatch with PackMetadata")
    if k.stride(-1) != 1 or (v is not None and v.stride() != k.stride()):
        k = k.contiguous()
        v = None if v is None else v.contiguous()
    if meta.B == 0:
        return
    _append_launch(_lib.view_bhnd(k), None if v is None else _lib.view_bhnd(v), _lib.FMLM_LAYOUT_PADDED,
                   k.element_size(), k.shape[3], meta.cu_seqlens, meta.B, meta.total_tokens, r.k, r.v, r.capacity,
                   r.cu, r.entries, k.device)


def convert_batch_major_entry(entry: LayerKVEntry) -> LayerKVEntry:
    """Head-major copy of a dense-prefill entry: [C][H][ctx] rows -> [H][C * ctx] rows
    with cu_seqlens_kv = c * ctx (one ``fmlm_cache_append`` launch)."""
    C, H, d = entry.context_batch_size, entry.num_heads, entry.head_dim
    ctx = int(entry.total_context_len) // C
    dev = entry.device
    cu_src = torch.arange(C + 1, dtype=torch.int32, device=dev) * ctx
    cu_kv = torch.zeros(C + 1, dtype=torch.int32, device=dev)
    k_dst = torch.empty((H * C * ctx, d), dtype=entry.dtype, device=dev)
    v_dst = torch.empty_like(k_dst)

    def view(x):
        return _lib.view4(x, rows=ctx, heads=H, batch=C, row_stride=d, head_stride=ctx * d,
                          batch_stride=H * ctx * d)

    if C * ctx > 0:
        _append_launch(view(entry.k_cache), view(entry.v_cache), _lib.FMLM_LAYOUT_PADDED, k_dst.element_size(), d,
                       cu_src, C, C * ctx, k_dst, v_dst, C * ctx, cu_kv, 0, dev)
    return LayerKVEntry(k_cache=k_dst, v_cache=v_dst, total_context_len=C * ctx, cu_seqlens_kv=cu_kv,
                        context_batch_size=C, is_mla=False, num_heads=H, head_dim=d, dtype=entry.dtype,
                        device=dev, layout=HEADS_MAJOR, cu_host=[c * ctx for c in range(C + 1)])
