"""The reference's CPU attention path, restated with torch -- TEST INFRASTRUCTURE ONLY.

The reference measures its kernels against plain torch loops: per (sequence,
head), ``logits = q @ [k_ctx; k_main]^T * scale``, ``softmax`` in fp32, then
``probs @ [v_ctx; v_main]`` (src/flash_mlm/host/test_host.py:48-105 with the
causal prefix; src/benchmark/standard_kernel/utils.py:365-407 varlen with a
shared or per-sequence context; :520-567 dense).  This module performs that
same loop on fp32 copies of the inputs, on all host threads, and is what
bench.py times as the reference's CPU path (`cpu_baseline`, `--impl
reference`).  tests/test_oracle_golden.py pins it to the golden vectors.

Unlike the numpy oracle it can restrict the work to a subset of the
sequences (``only``), which bounds the CPU time on large configurations.
"""

from __future__ import annotations

import torch


def varlen_attention_with_cache(q, k, v, cu_q, scale, *, k_cache=None, v_cache=None, cu_kv=None,
                                context_batch_size=1, total_context_len=0, is_mla=False,
                                causal_query_seq_attn=False, context_index=None, only=None) -> torch.Tensor:
    """Packed varlen attention; q/k/v padded [B, H, N, D] fp32; returns packed [H * T, D] fp32.

    Sequence b's queries attend its context entry (b, or 0 when the context is
    shared; ``context_index[b]`` when given) followed by its own tokens, or the
    tokens of sequences 0..b with ``causal_query_seq_attn``.  Head-major cache
    rows: head h of entry c is rows h * total_context_len + [cu_kv[c], cu_kv[c+1]).
    MLA: keys and values are k[:, 0] and the cache has one head.
    Rows of sequences outside ``only`` stay zero.
    """
    B, H, N, D = q.shape
    cu = [int(x) for x in cu_q]
    T = cu[-1]
    out = torch.zeros((H, T, D), dtype=torch.float32)
    seqs = range(B) if only is None else sorted(set(int(b) for b in only))
    for b in seqs:
        L = cu[b + 1] - cu[b]
        if L == 0:
            continue
        c0 = c1 = 0
        if k_cache is not None and cu_kv is not None and total_context_len > 0:
            c = int(context_index[b]) if context_index is not None else (0 if context_batch_size == 1 else b)
            c0, c1 = int(cu_kv[c]), int(cu_kv[c + 1])
        prefix = range(b + 1) if causal_query_seq_attn else (b,)
        for h in range(H):
            kh = 0 if is_mla else h
            k_main = torch.cat([k[j, kh, : cu[j + 1] - cu[j]] for j in prefix], dim=0)
            v_main = k_main if is_mla else torch.cat([v[j, h, : cu[j + 1] - cu[j]] for j in prefix], dim=0)
            if c1 > c0:
                off = 0 if is_mla else h * total_context_len
                k_ctx = k_cache[off + c0: off + c1]
                v_ctx = k_ctx if is_mla else v_cache[off + c0: off + c1]
                k_all, v_all = torch.cat([k_ctx, k_main]), torch.cat([v_ctx, v_main])
            else:
                k_all, v_all = k_main, v_main
            logits = (q[b, h, :L] @ k_all.T) * scale
            probs = torch.softmax(logits.float(), dim=-1)
            out[h, cu[b]: cu[b] + L] = probs @ v_all
    return out.reshape(H * T, D)


def dense_attention_with_cache(q, k, v, scale, *, k_cache=None, v_cache=None, context_len=0,
                               context_batch_size=1, is_mla=False) -> torch.Tensor:
    """Dense attention [B, H, N, D] fp32 with a [C][H][context_len] flat cache
    (utils.py:520-567; the dense kernel's MLA reads per-head main keys)."""
    B, H, N, D = q.shape
    out = torch.zeros_like(q)
    for b in range(B):
        cb = 0 if context_batch_size == 1 else b
        for h in range(H):
            k_main = k[b, h]
            v_main = k_main if is_mla else v[b, h]
            if context_len > 0:
                off = cb * context_len if is_mla else (cb * H + h) * context_len
                k_ctx = k_cache[off: off + context_len]
                v_ctx = k_ctx if is_mla else v_cache[off: off + context_len]
                k_main, v_main = torch.cat([k_ctx, k_main]), torch.cat([v_ctx, v_main])
            logits = (q[b, h] @ k_main.T) * scale
            out[b, h] = torch.softmax(logits.float(), dim=-1) @ v_main
    return out
