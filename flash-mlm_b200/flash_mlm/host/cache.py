"""Pack metadata, packing workspaces and the layer-scoped KV context cache.

Same public surface and error messages as the reference
(src/flash_mlm/host/cache.py:1-280): ``PackMetadata`` fields, ``PackingCache``
grow-only named workspaces and metadata memo, and ``InferenceCache`` holding
references (not copies) to per-layer packed K/V context.  This is host-side
bookkeeping only; every tensor it hands out lives wherever the caller put it.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass
class PackMetadata:
    """Reusable metadata for fast pack/unpack across layers."""

    B: int
    N: int
    lengths: torch.Tensor
    cu_seqlens: torch.Tensor
    token_indices: torch.Tensor
    total_tokens: int
    batch_ids_block_n: int
    batch_ids_q: torch.Tensor
    q_tile_starts_q: torch.Tensor


def host_cu_seqlens(meta: PackMetadata) -> list[int]:
    """Host copy of ``meta.cu_seqlens`` (one device read, memoised on the object)."""
    cached = getattr(meta, "_cu_host", None)
    if cached is None or len(cached) != meta.cu_seqlens.numel():
        cached = [int(x) for x in meta.cu_seqlens.to("cpu").tolist()]
        meta._cu_host = cached
    return cached


class PackingCache:
    """Reusable cache for pack metadata and packed main tensor workspaces (cache.py:20-73)."""

    def __init__(self):
        self._buffers: dict[tuple, torch.Tensor] = {}
        self._pack_meta: dict[tuple, PackMetadata] = {}
        # Device tile schedules of recent packed launches (see schedule_workspace).
        self._schedules: list[tuple[tuple, tuple, torch.Tensor]] = []

    _MAX_SCHEDULES = 8

    def schedule_workspace(self, tensors: tuple, scalars: tuple, nbytes: int,
                           device: torch.device) -> tuple[torch.Tensor, bool]:
        """Workspace for a packed launch's device tile schedule, and whether it already holds it.

        The schedule is a function of the sequence-offset tensors (``tensors``:
        cu_seqlens_q and, with a context, cu_seqlens_kv) and of ``scalars``.  An
        entry matches only the same tensor objects at the same in-place version
        (``Tensor._version``), so a new or modified offsets tensor builds a new
        schedule; entries keep their tensors alive, so an address cannot be
        reused by another tensor while an entry refers to it.  At most
        ``_MAX_SCHEDULES`` entries are kept (least recently used dropped).
        """
        versions = tuple(t._version for t in tensors)
        for i, (ts, key, ws) in enumerate(self._schedules):
            if (key == (scalars, versions) and len(ts) == len(tensors)
                    and all(a is b for a, b in zip(ts, tensors)) and ws.numel() * 4 >= nbytes):
                self._schedules.append(self._schedules.pop(i))
                return ws, True
        ws = torch.empty(((nbytes + 15) // 16, 4), dtype=torch.int32, device=device)
        self._schedules.append((tuple(tensors), (scalars, versions), ws))
        if len(self._schedules) > self._MAX_SCHEDULES:
            self._schedules.pop(0)
        return ws, False

    def get_2d(self, name: str, rows: int, cols: int, *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        if rows < 0:
            raise ValueError("rows must be >= 0")
        if cols < 1:
            raise ValueError("cols must be >= 1")
        key = (name, device.type, device.index, dtype, cols)
        buf = self._buffers.get(key)
        if buf is None or buf.shape[0] < rows:
            buf = torch.empty((rows, cols), dtype=dtype, device=device)
            self._buffers[key] = buf
        return buf[:rows]

    def get_pack_metadata(self, lengths: torch.Tensor, *, N: int, block_n: int) -> PackMetadata:
        signature = tuple(lengths.to(device="cpu", dtype=torch.int32).tolist())
        key = (lengths.device.type, lengths.device.index, N, block_n, signature)
        meta = self._pack_meta.get(key)
        if meta is None:
            from flash_mlm.host.host_utils import build_pack_metadata

            meta = build_pack_metadata(lengths, N, block_n)
            self._pack_meta[key] = meta
        return meta

    def clear(self):
        self._buffers.clear()
        self._pack_meta.clear()
        self._schedules.clear()


@dataclass
class LayerKVEntry:
    k_cache: torch.Tensor
    v_cache: torch.Tensor | None
    total_context_len: int
    cu_seqlens_kv: torch.Tensor | None
    context_batch_size: int
    is_mla: bool
    num_heads: int
    head_dim: int
    dtype: torch.dtype
    device: torch.device


def _check_rank2(x: torch.Tensor, what: str, head_dim: int, dim_msg: str) -> None:
    if x.ndim != 2:
        raise ValueError(f"{what} must be a rank-2 packed tensor")
    if x.shape[1] != head_dim:
        raise ValueError(dim_msg)


class InferenceCache:
    """Layer-scoped inference cache for packed KV context plus PackingCache reuse (cache.py:90-280)."""

    def __init__(self):
        self.packing = PackingCache()
        self._layer_kv: dict[str, LayerKVEntry] = {}

    @staticmethod
    def _layer_key(layer_id: int | str) -> str:
        return str(layer_id)

    @staticmethod
    def _validate_kv_common_inputs(*, k_cache, v_cache, total_context_len, is_mla, num_heads, head_dim) -> None:
        _check_rank2(k_cache, "k_cache", head_dim, "k_cache second dim must match head_dim")
        if not k_cache.is_contiguous():
            raise ValueError("k_cache must be contiguous")
        if is_mla:
            if v_cache is not None:
                if v_cache.ndim != 2:
                    raise ValueError("MLA v_cache must be a rank-2 packed tensor")
                if v_cache.shape != k_cache.shape:
                    raise ValueError("MLA v_cache shape must match k_cache shape")
                if not v_cache.is_contiguous():
                    raise ValueError("MLA v_cache must be contiguous")
        else:
            if v_cache is None:
                raise ValueError("non-MLA cache requires v_cache")
            if v_cache.ndim != 2:
                raise ValueError("v_cache must be a rank-2 packed tensor")
            if v_cache.shape != k_cache.shape:
                raise ValueError("v_cache shape must match k_cache shape")
            if v_cache.shape[1] != head_dim:
                raise ValueError("v_cache second dim must match head_dim")
            if not v_cache.is_contiguous():
                raise ValueError("v_cache must be contiguous")
        expected_rows = total_context_len if is_mla else num_heads * total_context_len
        if k_cache.shape[0] != expected_rows:
            raise ValueError(f"k_cache first dim mismatch: expected {expected_rows} rows for is_mla={is_mla}")
        if not is_mla and v_cache.shape[0] != expected_rows:
            raise ValueError(f"v_cache first dim mismatch: expected {expected_rows} rows for is_mla={is_mla}")

    @staticmethod
    def _validate_kv_entry_inputs(*, k_cache, v_cache, total_context_len, cu_seqlens_kv, context_batch_size,
                                  is_mla, num_heads, head_dim) -> None:
        InferenceCache._validate_kv_common_inputs(k_cache=k_cache, v_cache=v_cache,
                                                  total_context_len=total_context_len, is_mla=is_mla,
                                                  num_heads=num_heads, head_dim=head_dim)
        if cu_seqlens_kv.ndim != 1 or cu_seqlens_kv.numel() < 2:
            raise ValueError("cu_seqlens_kv must be rank-1 with at least 2 elements")
        if context_batch_size < 1:
            raise ValueError("context_batch_size must be >= 1")
        if context_batch_size + 1 > cu_seqlens_kv.numel():
            raise ValueError("context_batch_size is incompatible with cu_seqlens_kv length")

    def prefill_kv_cache(self, layer_id: int | str, *, k_cache: torch.Tensor, v_cache: torch.Tensor | None = None,
                         total_context_len: int | None = None, cu_seqlens_kv: torch.Tensor | None = None,
                         context_batch_size: int, is_mla: bool, num_heads: int, head_dim: int) -> None:
        """Store pre-packed KV cache buffers for a layer without copying."""
        if context_batch_size < 1:
            raise ValueError("context_batch_size must be >= 1")
        if num_heads < 1:
            raise ValueError("num_heads must be >= 1")
        if total_context_len is None:
            if is_mla:
                total_context_len = int(k_cache.shape[0])
            else:
                if k_cache.shape[0] % num_heads != 0:
                    raise ValueError("non-MLA k_cache rows must be divisible by num_heads")
                total_context_len = int(k_cache.shape[0] // num_heads)
        else:
            total_context_len = int(total_context_len)

        common = dict(k_cache=k_cache, v_cache=v_cache, total_context_len=total_context_len, is_mla=is_mla,
                      num_heads=num_heads, head_dim=head_dim)
        if cu_seqlens_kv is None:
            self._validate_kv_common_inputs(**common)
            if total_context_len % context_batch_size != 0:
                raise ValueError(
                    "when cu_seqlens_kv is omitted, total_context_len must be divisible by context_batch_size"
                )
        else:
            self._validate_kv_entry_inputs(**common, cu_seqlens_kv=cu_seqlens_kv,
                                           context_batch_size=context_batch_size)

        self._layer_kv[self._layer_key(layer_id)] = LayerKVEntry(
            k_cache=k_cache,
            v_cache=None if is_mla else v_cache,
            total_context_len=int(total_context_len),
            cu_seqlens_kv=cu_seqlens_kv.contiguous() if cu_seqlens_kv is not None else None,
            context_batch_size=int(context_batch_size),
            is_mla=bool(is_mla),
            num_heads=int(num_heads),
            head_dim=int(head_dim),
            dtype=k_cache.dtype,
            device=k_cache.device,
        )

    def get_kv_cache(self, layer_id: int | str, *, is_mla: bool, num_heads: int, head_dim: int,
                     dtype: torch.dtype, device: torch.device) -> LayerKVEntry:
        entry = self._layer_kv.get(self._layer_key(layer_id))
        if entry is None:
            raise ValueError(f"No cached KV context for layer_id={layer_id}")
        if entry.is_mla != is_mla:
            raise ValueError("Cached KV mode (is_mla) does not match request")
        if entry.num_heads != num_heads:
            raise ValueError("Cached num_heads does not match request")
        if entry.head_dim != head_dim:
            raise ValueError("Cached head_dim does not match request")
        if entry.dtype != dtype:
            raise ValueError("Cached KV dtype does not match request")
        if entry.device != device:
            raise ValueError("Cached KV device does not match request")
        return entry

    def clear_layer(self, layer_id: int | str):
        self._layer_kv.pop(self._layer_key(layer_id), None)

    def clear(self):
        self.packing.clear()
        self._layer_kv.clear()
