"""fp32 attention semantics of the reference kernels, restated in numpy.

TEST INFRASTRUCTURE ONLY.  Inputs are float32 arrays holding the (already
f16/bf16-rounded) values the GPU sees; softmax and both products run in fp32
with no intermediate rounding of P.

References:
  packed:  src/flash_mlm/mlm_kernel_impl.py:219-390 (+ host.py:228-530)
  dense:   src/flash_mlm/mlm_kernel_impl.py:65-216  (+ host.py:47-225)
"""

from __future__ import annotations

import numpy as np


def _softmax_attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """softmax(scale * q k^T) v in fp32; a row with no keys gives zeros (mlm_kernel_impl.py:381)."""
    if k.shape[0] == 0:
        return np.zeros((q.shape[0], v.shape[1]), dtype=np.float32)
    s = (q.astype(np.float32) @ k.astype(np.float32).T) * np.float32(scale)
    s = s - s.max(axis=1, keepdims=True)
    p = np.exp(s, dtype=np.float32)
    p /= p.sum(axis=1, keepdims=True)
    return (p @ v.astype(np.float32)).astype(np.float32)


def attention_packed(q, k, v, cu_q, scale, *, k_cache=None, v_cache=None, cu_kv=None, context_batch_size=1,
                     total_context_len=0, is_mla=False, causal_query_seq_attn=False, prefill=False,
                     context_index=None) -> np.ndarray:
    """Packed varlen attention.  q/k/v padded [B,H,N,D]; returns packed [H*T, D].

    Query b (tokens [0, L_b)) attends to context rows [cu_kv[c], cu_kv[c+1])
    (c = b if context_batch_size > 1 else 0; head-offset h*total_context_len
    unless MLA; skipped when prefill) followed by its own tokens, or with
    causal_query_seq_attn by all tokens of sequences 0..b.  MLA keys and
    values are k[:, 0].  ``context_index`` (no counterpart in the reference,
    whose README plans it) replaces the choice of c: c = context_index[b].
    """
    B, H, N, D = q.shape
    cu = [int(x) for x in cu_q]
    T = cu[-1]
    out = np.zeros((H, T, D), dtype=np.float32)
    for b in range(B):
        L = cu[b + 1] - cu[b]
        if L == 0:
            continue
        if not prefill and cu_kv is not None and k_cache is not None and total_context_len > 0:
            c = int(context_index[b]) if context_index is not None else (b if context_batch_size > 1 else 0)
            c0, c1 = int(cu_kv[c]), int(cu_kv[c + 1])
        else:
            c0 = c1 = 0
        seqs = range(b + 1) if causal_query_seq_attn else [b]
        for h in range(H):
            kh = 0 if is_mla else h
            k_main = np.concatenate([k[j, kh, : cu[j + 1] - cu[j]] for j in seqs], axis=0)
            v_main = k_main if is_mla else np.concatenate([v[j, h, : cu[j + 1] - cu[j]] for j in seqs], axis=0)
            if c1 > c0:
                off = 0 if is_mla else h * total_context_len
                k_ctx = k_cache[off + c0: off + c1]
                v_ctx = k_ctx if is_mla else v_cache[off + c0: off + c1]
                k_all = np.concatenate([k_ctx, k_main], axis=0)
                v_all = np.concatenate([v_ctx, v_main], axis=0)
            else:
                k_all, v_all = k_main, v_main
            out[h, cu[b]: cu[b] + L] = _softmax_attend(q[b, h, :L], k_all, v_all, scale)
    return out.reshape(H * T, D)


def attention_dense(q, k, v, scale, *, k_cache=None, v_cache=None, context_len=0, context_batch_size=1,
                    is_mla=False, prefill=False) -> np.ndarray:
    """Dense attention.  q/k/v [B,H,N,D]; every query attends to its uniform
    context then all N tokens of k[b, h] (MLA too: the dense kernel reads the
    per-head keys, mlm_kernel_impl.py:124,188-206).  Returns [B,H,N,D]."""
    B, H, N, D = q.shape
    out = np.zeros((B, H, N, D), dtype=np.float32)
    for b in range(B):
        cb = b if context_batch_size > 1 else 0
        for h in range(H):
            k_main = k[b, h]
            v_main = k_main if is_mla else v[b, h]
            if not prefill and context_len > 0:
                off = cb * context_len if is_mla else (cb * H + h) * context_len
                k_ctx = k_cache[off: off + context_len]
                v_ctx = k_ctx if is_mla else v_cache[off: off + context_len]
                k_all = np.concatenate([k_ctx, k_main], axis=0)
                v_all = np.concatenate([v_ctx, v_main], axis=0)
            else:
                k_all, v_all = k_main, v_main
            out[b, h] = _softmax_attend(q[b, h], k_all, v_all, scale)
    return out
