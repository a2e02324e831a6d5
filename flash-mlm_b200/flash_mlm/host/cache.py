"""Host-side bookkeeping of the forward path: pack metadata, reusable device
buffers and the per-layer context (KV) cache.

Public surface kept from the reference (src/flash_mlm/host/cache.py): the
``PackMetadata`` fields, ``PackingCache.get_2d`` / ``get_pack_metadata`` /
``clear``, ``LayerKVEntry``'s fields, and ``InferenceCache.prefill_kv_cache`` /
``get_kv_cache`` / ``clear_layer`` / ``clear`` / ``.packing`` with their
arguments and ``ValueError`` messages.  Callers match on those messages, so
they are kept word for word; everything else here is this package's own
design:

* ``PackingCache`` keeps every reusable object (grow-only 2-D workspaces,
  memoised pack metadata, memoised device tile schedules) in one keyed store,
  ``_Store``, whose bounded sections evict the least recently used entry.
* ``InferenceCache`` checks cache entries against one ordered rule table
  (``_ENTRY_RULES``) instead of nested branches.
* Beyond the reference: ``reserve_kv_cache`` / ``append_kv_cache`` give a
  layer a preallocated head-major cache with spare capacity that later calls
  append to on the device (``fmlm_cache_append``), and entries remember their
  row layout so a cache written by the dense path can serve the packed path
  and the other way round.

Nothing here copies tensor data on its own; device work is launched only by
``append_kv_cache`` and the layout conversion, through the CUDA library.
"""

from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Callable

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


# ---------------------------------------------------------------------------
# one keyed store for every reusable object of a PackingCache


class _Store:
    """Sections of keyed objects; a section created with a bound keeps only its
    ``bound`` most recently used entries."""

    def __init__(self):
        self._sections: dict[str, OrderedDict] = {}
        self._bounds: dict[str, int | None] = {}

    def section(self, name: str, bound: int | None = None) -> OrderedDict:
        sec = self._sections.get(name)
        if sec is None:
            sec = self._sections[name] = OrderedDict()
            self._bounds[name] = bound
        return sec

    def lookup(self, name: str, key: Any) -> Any:
        sec = self.section(name)
        val = sec.get(key)
        if val is not None:
            sec.move_to_end(key)
        return val

    def insert(self, name: str, key: Any, val: Any) -> Any:
        sec = self.section(name)
        sec[key] = val
        sec.move_to_end(key)
        bound = self._bounds.get(name)
        while bound is not None and len(sec) > bound:
            sec.popitem(last=False)
        return val

    def size(self, name: str) -> int:
        return len(self.section(name))

    def clear(self) -> None:
        for sec in self._sections.values():
            sec.clear()


class PackingCache:
    """Reusable cache for pack metadata and packed main tensor workspaces.

    Sections of its store: ``"workspace"`` (grow-only 2-D buffers keyed by
    name, device, dtype and column count), ``"metadata"`` (``PackMetadata``
    keyed by device, N, block_n and the lengths) and ``"schedule"`` (device
    tile schedules of recent packed launches, at most ``_MAX_SCHEDULES``).
    """

    _MAX_SCHEDULES = 8

    def __init__(self):
        self._store = _Store()
        self._store.section("schedule", bound=self._MAX_SCHEDULES)

    def get_2d(self, name: str, rows: int, cols: int, *, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
        """A [rows, cols] view of the named workspace, grown (never shrunk) to fit."""
        if rows < 0:
            raise ValueError("rows must be >= 0")
        if cols < 1:
            raise ValueError("cols must be >= 1")
        key = (name, device.type, device.index, dtype, cols)
        buf = self._store.lookup("workspace", key)
        if buf is None or buf.shape[0] < rows:
            buf = self._store.insert("workspace", key, torch.empty((rows, cols), dtype=dtype, device=device))
        return buf[:rows]

    def get_pack_metadata(self, lengths: torch.Tensor, *, N: int, block_n: int) -> PackMetadata:
        """Pack metadata for ``lengths``, built once per distinct length vector."""
        lens = tuple(int(x) for x in lengths.to(device="cpu", dtype=torch.int32).tolist())
        key = (lengths.device.type, lengths.device.index, N, block_n, lens)
        meta = self._store.lookup("metadata", key)
        if meta is None:
            from flash_mlm.host.host_utils import build_pack_metadata

            meta = self._store.insert("metadata", key, build_pack_metadata(lengths, N, block_n))
        return meta

    def schedule_workspace(self, tensors: tuple, scalars: tuple, nbytes: int,
                           device: torch.device) -> tuple[torch.Tensor, bool]:
        """Workspace for a packed launch's device tile schedule, and whether it already holds it.

        A schedule is a function of the sequence-offset tensors (``tensors``:
        cu_seqlens_q and, with a context, cu_seqlens_kv and context_index) and
        of ``scalars``.  A stored schedule is reused only for the very same
        tensor objects at the same in-place version (``Tensor._version``) and
        the same scalars, so a new or modified offsets tensor builds a new
        schedule.  Entries hold their tensors, so no other tensor can take
        over an address an entry refers to.
        """
        key = (tuple(id(t) for t in tensors), tuple(t._version for t in tensors), scalars)
        hit = self._store.lookup("schedule", key)
        if hit is not None:
            held, ws = hit
            if all(a is b for a, b in zip(held, tensors)) and ws.numel() * 4 >= nbytes:
                return ws, True
        ws = torch.empty(((nbytes + 15) // 16, 4), dtype=torch.int32, device=device)
        self._store.insert("schedule", key, (tuple(tensors), ws))
        return ws, False

    def clear(self):
        self._store.clear()


# ---------------------------------------------------------------------------
# per-layer context cache

# Row layouts of a cached entry (non-MLA; an MLA cache has one latent head, so
# both layouts coincide):
#   "heads_major": [H][total_context_len] rows, entries at cu_seqlens_kv offsets
#                  (what the packed path's prefill and append store).
#   "batch_major": [C][H][context_len] rows, uniform per-entry length
#                  (what the dense path's prefill stores).
#   "as_given":    buffers handed to prefill_kv_cache; as in the reference, the
#                  packed path reads them head-major and the dense path
#                  batch-major, with no conversion.
HEADS_MAJOR = "heads_major"
BATCH_MAJOR = "batch_major"
AS_GIVEN = "as_given"


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
    # --- beyond the reference ---
    layout: str = AS_GIVEN
    # Rows per head that hold context (a reserved cache has spare rows after them).
    used_context_len: int | None = None
    # Host copy of cu_seqlens_kv when the writer knew it (saves a device read).
    cu_host: list[int] | None = None
    # Memoised heads-major copy of a batch-major entry (see InferenceCache.as_heads_major).
    converted: "LayerKVEntry | None" = field(default=None, repr=False)

    def __post_init__(self):
        if self.used_context_len is None:
            self.used_context_len = int(self.total_context_len)


@dataclass
class _Reserved:
    """A layer's preallocated head-major cache with room for appends."""

    k: torch.Tensor                # [H * capacity, D]  (MLA: [capacity, D])
    v: torch.Tensor | None
    cu: torch.Tensor               # int32 [max_entries + 1] on the device
    capacity: int
    max_entries: int
    is_mla: bool
    num_heads: int
    head_dim: int
    entries: int = 0
    used: int = 0
    cu_host: list[int] = field(default_factory=lambda: [0])


# Ordered rules for cache entries: (applies, violated, message).  The first
# violated rule that applies raises.  `a` carries k, v, rows (rows a cache
# must have), mla and head_dim.
_Rule = tuple[Callable[[Any], bool], Callable[[Any], bool], Callable[[Any], str]]


def _msg(text: str) -> Callable[[Any], str]:
    return lambda a: text


_ENTRY_RULES: list[_Rule] = [
    (lambda a: True, lambda a: a.k.ndim != 2, _msg("k_cache must be a rank-2 packed tensor")),
    (lambda a: True, lambda a: a.k.shape[1] != a.head_dim, _msg("k_cache second dim must match head_dim")),
    (lambda a: True, lambda a: not a.k.is_contiguous(), _msg("k_cache must be contiguous")),
    # MLA: a v_cache is optional, and must mirror k_cache when given
    (lambda a: a.mla and a.v is not None, lambda a: a.v.ndim != 2, _msg("MLA v_cache must be a rank-2 packed tensor")),
    (lambda a: a.mla and a.v is not None, lambda a: a.v.shape != a.k.shape,
     _msg("MLA v_cache shape must match k_cache shape")),
    (lambda a: a.mla and a.v is not None, lambda a: not a.v.is_contiguous(), _msg("MLA v_cache must be contiguous")),
    # non-MLA: v_cache is required and mirrors k_cache
    (lambda a: not a.mla, lambda a: a.v is None, _msg("non-MLA cache requires v_cache")),
    (lambda a: not a.mla, lambda a: a.v.ndim != 2, _msg("v_cache must be a rank-2 packed tensor")),
    (lambda a: not a.mla, lambda a: a.v.shape != a.k.shape, _msg("v_cache shape must match k_cache shape")),
    (lambda a: not a.mla, lambda a: a.v.shape[1] != a.head_dim, _msg("v_cache second dim must match head_dim")),
    (lambda a: not a.mla, lambda a: not a.v.is_contiguous(), _msg("v_cache must be contiguous")),
    # row counts: [H * total_context_len] (MLA: [total_context_len])
    (lambda a: True, lambda a: a.k.shape[0] != a.rows,
     lambda a: f"k_cache first dim mismatch: expected {a.rows} rows for is_mla={a.mla}"),
    (lambda a: not a.mla, lambda a: a.v.shape[0] != a.rows,
     lambda a: f"v_cache first dim mismatch: expected {a.rows} rows for is_mla={a.mla}"),
]

_OFFSET_RULES: list[_Rule] = [
    (lambda a: True, lambda a: a.cu.ndim != 1 or a.cu.numel() < 2,
     _msg("cu_seqlens_kv must be rank-1 with at least 2 elements")),
    (lambda a: True, lambda a: a.cbs < 1, _msg("context_batch_size must be >= 1")),
    (lambda a: True, lambda a: a.cbs + 1 > a.cu.numel(),
     _msg("context_batch_size is incompatible with cu_seqlens_kv length")),
]


class _Args:
    def __init__(self, **kw):
        self.__dict__.update(kw)


def _check(rules: list[_Rule], args: _Args) -> None:
    for applies, violated, message in rules:
        if applies(args) and violated(args):
            raise ValueError(message(args))


class InferenceCache:
    """Layer-scoped inference cache for packed KV context plus PackingCache reuse.

    An entry references the caller's tensors (nothing is copied).  Entries are
    keyed by ``str(layer_id)``.
    """

    def __init__(self):
        self.packing = PackingCache()
        self._entries: dict[str, LayerKVEntry] = {}
        self._reserved: dict[str, _Reserved] = {}

    # ------------------------------------------------------------------ reference surface
    def prefill_kv_cache(self, layer_id: int | str, *, k_cache: torch.Tensor, v_cache: torch.Tensor | None = None,
                         total_context_len: int | None = None, cu_seqlens_kv: torch.Tensor | None = None,
                         context_batch_size: int, is_mla: bool, num_heads: int, head_dim: int) -> None:
        """Store pre-packed KV cache buffers for a layer without copying.

        ``k_cache`` / ``v_cache`` are [H * total_context_len, D] head-major
        (MLA: [total_context_len, D], ``v_cache`` optional).  Without
        ``cu_seqlens_kv`` the context is ``context_batch_size`` entries of equal
        length; ``total_context_len`` defaults to the rows per head.
        """
        self._store_entry(layer_id, k_cache=k_cache, v_cache=v_cache, total_context_len=total_context_len,
                          cu_seqlens_kv=cu_seqlens_kv, context_batch_size=context_batch_size, is_mla=is_mla,
                          num_heads=num_heads, head_dim=head_dim, layout=AS_GIVEN)

    def get_kv_cache(self, layer_id: int | str, *, is_mla: bool, num_heads: int, head_dim: int,
                     dtype: torch.dtype, device: torch.device) -> LayerKVEntry:
        """The layer's entry, if it was stored for exactly this kind of request."""
        entry = self._entries.get(str(layer_id))
        if entry is None:
            raise ValueError(f"No cached KV context for layer_id={layer_id}")
        mismatches = (
            (entry.is_mla != is_mla, "Cached KV mode (is_mla) does not match request"),
            (entry.num_heads != num_heads, "Cached num_heads does not match request"),
            (entry.head_dim != head_dim, "Cached head_dim does not match request"),
            (entry.dtype != dtype, "Cached KV dtype does not match request"),
            (entry.device != device, "Cached KV device does not match request"),
        )
        for bad, message in mismatches:
            if bad:
                raise ValueError(message)
        return entry

    def clear_layer(self, layer_id: int | str):
        self._entries.pop(str(layer_id), None)
        self._reserved.pop(str(layer_id), None)

    def clear(self):
        self.packing.clear()
        self._entries.clear()
        self._reserved.clear()

    # ------------------------------------------------------------------ entry construction
    def _store_entry(self, layer_id, *, k_cache, v_cache, total_context_len, cu_seqlens_kv, context_batch_size,
                     is_mla, num_heads, head_dim, layout, used_context_len=None, cu_host=None) -> LayerKVEntry:
        if context_batch_size < 1:
            raise ValueError("context_batch_size must be >= 1")
        if num_heads < 1:
            raise ValueError("num_heads must be >= 1")
        if total_context_len is None:
            rows = int(k_cache.shape[0])
            if not is_mla and rows % num_heads != 0:
                raise ValueError("non-MLA k_cache rows must be divisible by num_heads")
            total_context_len = rows if is_mla else rows // num_heads
        total_context_len = int(total_context_len)
        args = _Args(k=k_cache, v=v_cache, mla=is_mla, head_dim=head_dim,
                     rows=total_context_len if is_mla else num_heads * total_context_len)
        _check(_ENTRY_RULES, args)
        if cu_seqlens_kv is None:
            if total_context_len % context_batch_size != 0:
                raise ValueError(
                    "when cu_seqlens_kv is omitted, total_context_len must be divisible by context_batch_size")
        else:
            _check(_OFFSET_RULES, _Args(cu=cu_seqlens_kv, cbs=context_batch_size))
        entry = LayerKVEntry(
            k_cache=k_cache, v_cache=None if is_mla else v_cache, total_context_len=total_context_len,
            cu_seqlens_kv=None if cu_seqlens_kv is None else cu_seqlens_kv.contiguous(),
            context_batch_size=int(context_batch_size), is_mla=bool(is_mla), num_heads=int(num_heads),
            head_dim=int(head_dim), dtype=k_cache.dtype, device=k_cache.device,
            layout=layout, used_context_len=used_context_len, cu_host=cu_host)
        self._entries[str(layer_id)] = entry
        return entry

    def _store_packed_prefill(self, layer_id, **kw) -> None:
        """Entry written by a packed launcher's prefill: head-major rows (host.py:351-364)."""
        self._store_entry(layer_id, layout=HEADS_MAJOR, **kw)

    def _store_dense_prefill(self, layer_id, *, k_cache, v_cache, context_batch_size, is_mla, num_heads,
                             head_dim) -> None:
        """Entry written by the dense path's prefill: [C][H][context_len] rows (host.py:206-223)."""
        self._store_entry(layer_id, k_cache=k_cache, v_cache=v_cache, total_context_len=None, cu_seqlens_kv=None,
                          context_batch_size=context_batch_size, is_mla=is_mla, num_heads=num_heads,
                          head_dim=head_dim, layout=BATCH_MAJOR)

    # ------------------------------------------------------------------ preallocated caches (beyond the reference)
    def reserve_kv_cache(self, layer_id: int | str, *, capacity: int, max_entries: int, is_mla: bool,
                         num_heads: int, head_dim: int, dtype: torch.dtype, device: torch.device) -> None:
        """Give a layer a head-major cache of ``capacity`` rows per head and room
        for ``max_entries`` context entries.  Later ``append_kv_cache`` calls,
        and ``prefill=True`` calls of the packed launchers, write into it on the
        device instead of allocating; the layer's entry is empty until then.
        (The dense launcher's prefill and ``flash_attn_mlm_precompressed``'s
        prefill store their own buffers, as in the reference, replacing the
        entry; the reservation stays for later appends.)"""
        if capacity < 0 or max_entries < 1 or num_heads < 1:
            raise ValueError("capacity must be >= 0, max_entries >= 1 and num_heads >= 1")
        rows = capacity if is_mla else num_heads * capacity
        # Zero-filled: the attention kernel's last key block of an entry may
        # read rows past it (masked, P = 0), which must not hold NaN.
        k = torch.zeros((rows, head_dim), dtype=dtype, device=device)
        v = None if is_mla else torch.zeros_like(k)
        cu = torch.zeros(max_entries + 1, dtype=torch.int32, device=device)
        self._reserved[str(layer_id)] = _Reserved(k=k, v=v, cu=cu, capacity=int(capacity),
                                                 max_entries=int(max_entries), is_mla=bool(is_mla),
                                                 num_heads=int(num_heads), head_dim=int(head_dim))
        self._entries.pop(str(layer_id), None)

    def reserved(self, layer_id: int | str) -> _Reserved | None:
        return self._reserved.get(str(layer_id))

    def reset_kv_cache(self, layer_id: int | str) -> None:
        """Empty a reserved cache (keeps its memory); the layer then has no entry."""
        r = self._reserved.get(str(layer_id))
        if r is None:
            raise ValueError(f"No reserved KV cache for layer_id={layer_id}")
        r.entries, r.used, r.cu_host = 0, 0, [0]
        self._entries.pop(str(layer_id), None)

    def append_kv_cache(self, layer_id: int | str, k: torch.Tensor, v: torch.Tensor | None,
                        q_meta: PackMetadata) -> LayerKVEntry:
        """Append the valid rows of padded k / v [B, H, N, D] (MLA: k [B, 1 or H, N, D],
        head 0 used; v ignored) as B new context entries of the layer's reserved
        cache, on the device (one ``fmlm_cache_append`` launch; the entry
        offsets are updated on the device, their host copy from ``q_meta``)."""
        from flash_mlm.host.host_utils import append_rows_into_cache

        r = self._reserved.get(str(layer_id))
        if r is None:
            raise ValueError(f"No reserved KV cache for layer_id={layer_id}")
        if r.entries + q_meta.B > r.max_entries:
            raise ValueError(f"append of {q_meta.B} entries exceeds max_entries={r.max_entries} "
                             f"({r.entries} stored)")
        if r.used + q_meta.total_tokens > r.capacity:
            raise ValueError(f"append of {q_meta.total_tokens} rows exceeds capacity={r.capacity} "
                             f"({r.used} stored)")
        if k.ndim != 4 or k.shape[3] != r.head_dim or k.dtype != r.k.dtype or k.device != r.k.device:
            raise ValueError("k must be [B, H, N, D] with the reserved cache's head_dim, dtype and device")
        if r.is_mla:
            k, v = k[:, :1], None
        elif k.shape[1] != r.num_heads or v is None or v.shape != k.shape or v.dtype != k.dtype:
            raise ValueError("non-MLA append needs k and v of shape [B, num_heads, N, D]")
        append_rows_into_cache(k, v, q_meta, r)
        cu_q = host_cu_seqlens(q_meta)
        base = r.used
        r.cu_host = r.cu_host + [base + x - cu_q[0] for x in cu_q[1:]]
        r.used += q_meta.total_tokens
        r.entries += q_meta.B
        return self._store_entry(layer_id, k_cache=r.k, v_cache=r.v, total_context_len=r.capacity,
                                 cu_seqlens_kv=r.cu[: r.entries + 1], context_batch_size=r.entries,
                                 is_mla=r.is_mla, num_heads=r.num_heads, head_dim=r.head_dim, layout=HEADS_MAJOR,
                                 used_context_len=r.used, cu_host=list(r.cu_host))

    # ------------------------------------------------------------------ layout conversion
    def as_heads_major(self, entry: LayerKVEntry) -> LayerKVEntry:
        """The entry in the head-major layout the packed path reads: the entry
        itself, or (for a batch-major entry of a dense prefill with several
        entries and heads) a converted copy made once on the device by
        ``fmlm_cache_append`` and kept on the entry."""
        if entry.layout != BATCH_MAJOR or entry.is_mla or entry.context_batch_size == 1 or entry.num_heads == 1:
            return entry
        if entry.converted is None:
            from flash_mlm.host.host_utils import convert_batch_major_entry

            entry.converted = convert_batch_major_entry(entry)
        return entry.converted
