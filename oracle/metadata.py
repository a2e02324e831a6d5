"""Integer / byte-copy parts of the reference host utilities, restated in numpy.

Reference: src/flash_mlm/host/host_utils.py (TEST INFRASTRUCTURE ONLY).
"""

from __future__ import annotations

import numpy as np


def build_pack_metadata(lengths, N: int, block_n: int) -> dict:
    """host_utils.py:27-71: cu_seqlens, token_indices (b*N+t of valid tokens), tile map, total."""
    lengths = np.asarray(lengths, dtype=np.int64)
    if lengths.ndim != 1:
        raise ValueError("lengths must be rank-1 [B]")
    if N < 0:
        raise ValueError("N must be >= 0")
    if block_n < 1:
        raise ValueError("block_n must be >= 1")
    if np.any(lengths < 0) or np.any(lengths > N):
        raise ValueError("lengths values must be in [0, N]")
    B = lengths.size
    cu = np.zeros(B + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lengths).astype(np.int32)
    tok = [b * N + t for b in range(B) for t in range(int(lengths[b]))]
    starts, bids = tile_map_from_cu_seqlens(cu, block_n)
    return {
        "cu_seqlens": cu,
        "token_indices": np.asarray(tok, dtype=np.int64),
        "total_tokens": int(cu[-1]),
        "batch_ids_q": bids,
        "q_tile_starts_q": starts,
    }


def tile_map_from_cu_seqlens(cu, block_n: int):
    """host_utils.py:74-107: per-sequence tiles of block_n rows; start = cu[b] + i*block_n."""
    cu = np.asarray(cu, dtype=np.int64)
    starts, bids = [], []
    for b in range(cu.size - 1):
        L = int(cu[b + 1] - cu[b])
        for i in range((L + block_n - 1) // block_n):
            starts.append(int(cu[b]) + i * block_n)
            bids.append(b)
    return np.asarray(starts, dtype=np.int32), np.asarray(bids, dtype=np.int32)


def total_q_len_padded(total_unpadded: int, cu, block_m: int, block_n: int) -> int:
    """host_utils.py:292-312: max over sequences of cu[b] + roundup(len_b, max(block_m, block_n))."""
    a = max(block_m, block_n)
    cu = [int(x) for x in cu]
    need = max([s + ((e - s + a - 1) // a) * a for s, e in zip(cu[:-1], cu[1:])], default=0)
    return max(int(total_unpadded), need)


def pack_rows(x: np.ndarray, cu, total_padded: int) -> np.ndarray:
    """host_utils.py:397-420: [B,H,N,D] -> [H*total_padded, D], valid rows in (b, t) order, zero pad rows."""
    B, H, N, D = x.shape
    cu = [int(c) for c in cu]
    T = cu[-1]
    out = np.zeros((H, total_padded, D), dtype=x.dtype)
    for b in range(B):
        L = cu[b + 1] - cu[b]
        out[:, cu[b]:cu[b] + L, :] = x[b, :, :L, :]
    assert T <= total_padded
    return out.reshape(H * total_padded, D)


def unpack_rows(packed: np.ndarray, cu, H: int, N: int) -> np.ndarray:
    """host_utils.py:587-615: [H*T, D] -> zero-padded [B,H,N,D]."""
    cu = [int(c) for c in cu]
    B, T = len(cu) - 1, cu[-1]
    D = packed.shape[-1]
    ph = packed.reshape(H, T, D)
    out = np.zeros((B, H, N, D), dtype=packed.dtype)
    for b in range(B):
        L = cu[b + 1] - cu[b]
        out[b, :, :L, :] = ph[:, cu[b]:cu[b] + L, :]
    return out


def pad_packed_rows(x: np.ndarray, heads: int, old_len: int, new_len: int) -> np.ndarray:
    """host_utils.py:514-527: per-head zero rows appended from old_len to new_len."""
    D = x.shape[1]
    out = np.zeros((heads, new_len, D), dtype=x.dtype)
    out[:, :old_len, :] = x.reshape(heads, old_len, D)
    return out.reshape(heads * new_len, D)


def cache_append(cache: np.ndarray, cu_kv: list, x: np.ndarray, cu_src) -> tuple[np.ndarray, list]:
    """Append the valid rows of padded x [B, H, N, D] to a head-major cache
    [H * capacity, D] holding entries cu_kv (host list); returns the new cache
    and offsets.  Restates what the reference's prefill stores for each
    sequence (packed rows per head, src/flash_mlm/host/host.py:327-364) written
    after the rows already held instead of into a new buffer."""
    B, H, _, D = x.shape
    cap = cache.shape[0] // H
    out = cache.copy().reshape(H, cap, D)
    cu = [int(c) for c in cu_src]
    base = int(cu_kv[-1])
    new_cu = list(cu_kv)
    for b in range(B):
        L = cu[b + 1] - cu[b]
        out[:, base + cu[b] - cu[0]: base + cu[b] - cu[0] + L] = x[b, :, :L]
        new_cu.append(base + cu[b + 1] - cu[0])
    return out.reshape(H * cap, D), new_cu
