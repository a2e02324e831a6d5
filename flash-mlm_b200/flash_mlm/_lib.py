"""ctypes binding of libflashmlm.so (the sm_100a CUDA library, C ABI in include/flash_mlm.h).

There is no CPU implementation behind this module: if the shared library is
missing or a tensor is not on a CUDA device, calls raise instead of falling
back to anything else.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_native" / "libflashmlm.so"

FMLM_DTYPE_F16 = 0
FMLM_DTYPE_BF16 = 1
FMLM_LAYOUT_PADDED = 0
FMLM_LAYOUT_PACKED = 1


class View4(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("heads", ctypes.c_int64),
        ("batch", ctypes.c_int64),
        ("row_stride", ctypes.c_int64),
        ("head_stride", ctypes.c_int64),
        ("batch_stride", ctypes.c_int64),
    ]


class DenseArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("is_mla", ctypes.c_int32),
        ("prefill", ctypes.c_int32),
        ("context_batch_size", ctypes.c_int32),
        ("context_len", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q", View4),
        ("k", View4),
        ("v", View4),
        ("k_cache", View4),
        ("v_cache", View4),
        ("out", ctypes.c_void_p),
        ("error_word", ctypes.c_void_p),
    ]


class PackedArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("is_mla", ctypes.c_int32),
        ("prefill", ctypes.c_int32),
        ("causal_query_seq_attn", ctypes.c_int32),
        ("context_batch_size", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("q_layout", ctypes.c_int32),
        ("kv_layout", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("total_q_len", ctypes.c_int64),
        ("q", View4),
        ("k", View4),
        ("v", View4),
        ("k_cache", View4),
        ("v_cache", View4),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("cu_seqlens_kv", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_rows_per_head", ctypes.c_int64),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("error_word", ctypes.c_void_p),
        ("reuse_schedule", ctypes.c_int32),
        ("context_index", ctypes.c_void_p),
        ("out_padded", ctypes.c_int32),
    ]


_lib = None
_lib_lock = threading.Lock()


def lib() -> ctypes.CDLL:
    """Load (once) and return the CUDA library; raise if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("FLASH_MLM_LIB", _LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"flash_mlm CUDA library not found at {path}; build it with "
                "`python flash-mlm_b200/build.py` (there is no CPU fallback)"
            )
        L = ctypes.CDLL(str(path))
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        L.fmlm_attn_dense_fwd.argtypes = [ctypes.POINTER(DenseArgs), vp]
        L.fmlm_attn_dense_fwd.restype = ctypes.c_int
        L.fmlm_attn_packed_fwd.argtypes = [ctypes.POINTER(PackedArgs), vp]
        L.fmlm_attn_packed_fwd.restype = ctypes.c_int
        L.fmlm_attn_packed_fwd_noalloc.argtypes = [ctypes.POINTER(PackedArgs), vp]
        L.fmlm_attn_packed_fwd_noalloc.restype = ctypes.c_int
        L.fmlm_selftest_bounded_wait.argtypes = [vp, ctypes.c_uint64, vp]
        L.fmlm_selftest_bounded_wait.restype = ctypes.c_int
        L.fmlm_packed_workspace_bytes.argtypes = [i32, i64, i32]
        L.fmlm_packed_workspace_bytes.restype = ctypes.c_size_t
        L.fmlm_build_pack_metadata.argtypes = [vp, i32, i32, i32, vp, vp, vp, vp, vp, vp]
        L.fmlm_build_pack_metadata.restype = ctypes.c_int
        L.fmlm_pack_rows.argtypes = [ctypes.POINTER(View4), i32, i32, vp, i32, i64, i64, vp, vp]
        L.fmlm_pack_rows.restype = ctypes.c_int
        L.fmlm_unpack_rows.argtypes = [vp, i64, i32, i32, i32, vp, i32, i32, vp, vp]
        L.fmlm_unpack_rows.restype = ctypes.c_int
        L.fmlm_pad_packed_rows.argtypes = [vp, i64, i64, i32, i32, i32, vp, vp]
        L.fmlm_pad_packed_rows.restype = ctypes.c_int
        L.fmlm_cache_append.argtypes = [ctypes.POINTER(View4), ctypes.POINTER(View4), i32, i32, i32, vp, i32, i64,
                                        vp, vp, i64, vp, i32, vp, vp]
        L.fmlm_cache_append.restype = ctypes.c_int
        L.fmlm_last_error.argtypes = []
        L.fmlm_last_error.restype = ctypes.c_char_p
        L.fmlm_version.argtypes = []
        L.fmlm_version.restype = ctypes.c_int
        _lib = L
        return _lib


class FlashMLMError(RuntimeError):
    pass


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = lib().fmlm_last_error().decode(errors="replace")
        if rc == -1 or rc == -2:
            raise ValueError(f"{what}: {msg}")
        raise FlashMLMError(f"{what} failed ({rc}): {msg}")


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.float16:
        return FMLM_DTYPE_F16
    if dtype == torch.bfloat16:
        return FMLM_DTYPE_BF16
    raise ValueError(f"unsupported dtype {dtype}: flash_mlm kernels take float16 or bfloat16")


def view4(x: torch.Tensor | None, *, rows: int = 0, heads: int = 0, batch: int = 0,
          row_stride: int = 0, head_stride: int = 0, batch_stride: int = 0) -> View4:
    if x is None:
        return View4(None, 0, 0, 0, 0, 0, 0)
    return View4(x.data_ptr() if x.numel() > 0 else None, rows, heads, batch, row_stride, head_stride, batch_stride)


def view_bhnd(x: torch.Tensor) -> View4:
    """[B, H, N, D] tensor (innermost dim contiguous) as a View4."""
    b, h, n, _ = x.shape
    return view4(x, rows=n, heads=h, batch=b, row_stride=x.stride(2), head_stride=x.stride(1), batch_stride=x.stride(0))


def view_packed(x: torch.Tensor, heads: int) -> View4:
    """Packed rank-2 [heads * rows, D] tensor as a View4 with batch 1."""
    rows = x.shape[0] // heads if heads > 0 else 0
    d = x.shape[1]
    return view4(x, rows=rows, heads=heads, batch=1, row_stride=x.stride(0), head_stride=rows * x.stride(0),
                 batch_stride=heads * rows * x.stride(0) if rows else d)


_err_words: dict[int, torch.Tensor] = {}


def error_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word that kernels set when a bounded wait gives up."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    w = _err_words.get(idx)
    if w is None:
        w = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _err_words[idx] = w
    return w


def check_device_errors(device: torch.device | None = None) -> None:
    """Synchronise and raise if any kernel on `device` reported an error.

    Codes: 1 = a bounded wait gave up; 2 = the dynamic shared-memory window
    was not 1024-byte aligned (the kernel returned without touching memory);
    3 = a context_index entry was out of range (that sequence attended no
    context); 4 = a packed sequence had more than 65536 work items (it was
    not computed); 5 = a cache append would have passed the cache capacity
    (nothing was written).
    """
    devs = [device] if device is not None else [torch.device("cuda", i) for i in list(_err_words)]
    for d in devs:
        w = error_word(d)
        v = int(w[0].item())
        if v != 0:
            w.zero_()
            what = {1: "gave up waiting", 2: "found its shared memory misaligned",
                    3: "met a context_index entry out of range",
                    4: "met a sequence too long for the tile schedule",
                    5: "would have overrun a context cache's capacity (nothing appended)"}.get(v, "failed")
            raise FlashMLMError(f"flash_mlm kernel on {d} {what} (code {v}); results are invalid")


def require_cuda(*tensors: torch.Tensor | None, what: str = "flash_mlm") -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError(f"{what} requires CUDA tensors (there is no CPU path)")
