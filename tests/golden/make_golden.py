"""Generate the golden fixtures in this folder from the reference implementation.

Run here (CPU is enough) with the reference checkout available:

    python tests/golden/make_golden.py --reference /path/to/flash-mlm

It imports the reference package from <reference>/src and records outputs of
its own functions:

* metadata / pack / pad / unpack: src/flash_mlm/host/host_utils.py (run on CPU
  tensors, exactly as the reference's own unit tests run them);
* attention: the fp32 torch reference math of src/flash_mlm/host/test_host.py:30-145
  (those three functions are taken from the file's syntax tree, because the
  module itself needs a GPU at import time) and of
  src/benchmark/standard_kernel/utils.py:365-407.  Inputs are f16/bf16-rounded
  and upcast to fp32, so these functions compute exact fp32 attention (their
  probability cast is to the fp32 input dtype).

Outputs: metadata.json, pack.npz, attention.npz.  The fixtures are committed;
the GPU box never needs the reference.
"""

from __future__ import annotations

import argparse
import ast
import json
import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _load_test_host_refs(ref_root: Path) -> dict:
    src = (ref_root / "src/flash_mlm/host/test_host.py").read_text()
    tree = ast.parse(src)
    wanted = {"reference_attention", "_reference_varlen_attention_with_cache", "_reference_dense_attention_with_flat_cache"}
    mod = ast.Module(body=[n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted], type_ignores=[])
    ns = {"torch": torch}
    exec(compile(mod, "test_host_refs", "exec"), ns)
    return ns


def _rounded(shape, dtype, gen, scale=1.0):
    x = torch.randn(shape, generator=gen) * scale
    return x.to(dtype).to(torch.float32)


def metadata_cases(hu):
    cases = []
    specs = [
        ([4, 2], 4, 3),          # test_host_utils.py:19-43
        ([5, 2], 5, 4),
        ([1, 1], 2, 1),
        ([0, 3, 0, 5], 6, 2),
        ([7], 7, 32),
        ([0, 0], 3, 4),
        ([64, 1, 33, 17, 128, 5], 128, 32),
    ]
    g = torch.Generator().manual_seed(7)
    for B, N, bn in [(32, 512, 64), (17, 300, 32), (64, 256, 128)]:
        lengths = torch.randint(0, N + 1, (B,), generator=g).tolist()
        specs.append((lengths, N, bn))
    for lengths, N, bn in specs:
        meta = hu.build_pack_metadata(torch.tensor(lengths, dtype=torch.int32), N, bn)
        cu = meta.cu_seqlens
        tiles_cu = {}
        for bn2 in (1, 3, 4, 16):
            s, bid = hu._build_query_tile_map_from_cu_seqlens(cu, bn2)
            tiles_cu[str(bn2)] = {"starts": s.tolist(), "batch_ids": bid.tolist()}
        pads = {}
        for bm, bn2 in ((4, 4), (32, 32), (64, 32), (128, 64)):
            pads[f"{bm},{bn2}"] = hu._compute_total_q_len_padded(meta.total_tokens, cu, bm, bn2)
        cases.append({
            "lengths": lengths, "N": N, "block_n": bn,
            "cu_seqlens": cu.tolist(), "token_indices": meta.token_indices.tolist(),
            "total_tokens": meta.total_tokens, "batch_ids_q": meta.batch_ids_q.tolist(),
            "q_tile_starts_q": meta.q_tile_starts_q.tolist(), "tile_maps_from_cu": tiles_cu,
            "total_q_len_padded": pads,
        })
    return cases


def pack_cases(hu):
    out = {}
    g = torch.Generator().manual_seed(11)
    specs = [([4, 2], 2, 4, 1, 4, 4), ([5, 0, 3], 3, 6, 8, 4, 4), ([9, 7, 5], 2, 32, 64, 32, 32),
             ([48, 37], 3, 48, 64, 32, 32), ([1], 1, 1, 16, 64, 32)]
    for i, (lengths, H, N, D, bm, bn) in enumerate(specs):
        B = len(lengths)
        meta = hu.build_pack_metadata(torch.tensor(lengths, dtype=torch.int32), N, bn)
        x = torch.randn((B, H, N, D), generator=g)
        packed = hu.pack_for_kernel(x, meta, flatten_for_kernel=True)
        unpacked = hu.unpack_from_kernel(packed, meta, H=H)
        k = x + 100
        v = x + 200
        qp, kp, vp, tot = hu.pack_and_pad_main_tensors_for_mlm_compressed(
            x, k, v, q_meta=meta, num_heads=H, is_mla=False, block_m=bm, block_n=bn)
        _, kpm, _, totm = hu.pack_and_pad_main_tensors_for_mlm_compressed(
            x, k, v, q_meta=meta, num_heads=H, is_mla=True, block_m=bm, block_n=bn)
        qpad, kpad, vpad, totpad = hu.pad_packed_main_tensors_for_mlm_compressed(
            packed, hu.pack_for_kernel(k, meta, True), hu.pack_for_kernel(v, meta, True), num_heads=H,
            is_mla=False, total_q_len_unpadded=meta.total_tokens, cu_seqlens_q=meta.cu_seqlens, block_m=bm,
            block_n=bn)
        p = f"c{i}_"
        out[p + "spec"] = np.array([B, H, N, D, bm, bn], dtype=np.int64)
        out[p + "lengths"] = np.array(lengths, dtype=np.int32)
        out[p + "x"] = x.numpy()
        out[p + "packed"] = packed.numpy()
        out[p + "unpacked"] = unpacked.numpy()
        out[p + "qpp"] = qp.numpy()
        out[p + "kpp"] = kp.numpy()
        out[p + "kpp_mla"] = kpm.numpy()
        out[p + "total_padded"] = np.array([tot, totm, totpad], dtype=np.int64)
        out[p + "qpad"] = qpad.numpy()
    return out


def attention_cases(refs, bu):
    """Each case: inputs (rounded to its dtype, stored as fp32) + the reference's fp32 output."""
    out = {}
    manifest = []

    def add(name, arrays, params):
        # Inputs are stored in their own 16-bit format (bf16 as raw int16 bits); outputs as fp32.
        dt = torch.float16 if params["dtype"] == "f16" else torch.bfloat16
        for k, v in arrays.items():
            if isinstance(v, torch.Tensor) and v.is_floating_point() and k != "out":
                v = v.to(dt)
                v = v.numpy() if dt == torch.float16 else v.view(torch.int16).numpy()
            out[f"{name}__{k}"] = v.numpy() if isinstance(v, torch.Tensor) else np.asarray(v)
        manifest.append({"name": name, **params})

    f16, bf16 = torch.float16, torch.bfloat16

    # compressed, no cache (test_host.py:313-365 shapes); fp32 oracle = reference_attention
    for is_mla in (False, True):
        for dt, dtn in ((f16, "f16"), (bf16, "bf16")):
            g = torch.Generator().manual_seed(12)
            B, H, N, D = 2, 3, 24, 64
            lengths = torch.tensor([24, 15], dtype=torch.int32)
            q, k, v = (_rounded((B, H, N, D), dt, g) for _ in range(3))
            if is_mla:
                v = k
            ref = refs["reference_attention"](q, k, v, lengths, 0.6, is_mla)
            add(f"cmp_nocache_mla{int(is_mla)}_{dtn}", {"q": q, "k": k, "v": v, "lengths": lengths, "out": ref},
                {"kind": "compressed", "dtype": dtn, "scale": 0.6, "is_mla": is_mla, "causal": False, "ctx": "none"})

    # compressed with per-batch cache (test_host.py:548-617)
    for is_mla in (False, True):
        g = torch.Generator().manual_seed(1)
        B, H, N, D = 2, 3, 48, 64
        lengths = torch.tensor([48, 37], dtype=torch.int32)
        ctx_lengths = torch.tensor([13, 9], dtype=torch.int32)
        q, k, v = (_rounded((B, H, N, D), f16, g) for _ in range(3))
        cu_kv = torch.zeros(B + 1, dtype=torch.int32)
        cu_kv[1:] = ctx_lengths.cumsum(0)
        tcl = int(cu_kv[-1])
        rows = tcl if is_mla else H * tcl
        kc = _rounded((rows, D), f16, g)
        vc = _rounded((rows, D), f16, g)
        ref = refs["_reference_varlen_attention_with_cache"](q, k, v, lengths, kc, vc, cu_kv, 0.5, is_mla)
        add(f"cmp_cache_mla{int(is_mla)}_f16", {"q": q, "k": k, "v": v, "lengths": lengths, "k_cache": kc,
                                                 "v_cache": vc, "cu_kv": cu_kv, "out": ref},
            {"kind": "compressed", "dtype": "f16", "scale": 0.5, "is_mla": is_mla, "causal": False, "ctx": "batch",
             "total_context_len": tcl, "context_batch_size": B})

    # causal_query_seq_attn (test_host.py:475-545), with and without per-batch context
    for is_mla in (False, True):
        for with_ctx in (False, True):
            g = torch.Generator().manual_seed(2)
            B, H, N, D = 3, 2, 32, 64
            lengths = torch.tensor([9, 7, 5], dtype=torch.int32)
            q, k, v = (_rounded((B, H, N, D), f16, g) for _ in range(3))
            if with_ctx:
                ctx_lengths = torch.tensor([4, 0, 11], dtype=torch.int32)
            else:
                ctx_lengths = torch.zeros(B, dtype=torch.int32)
            cu_kv = torch.zeros(B + 1, dtype=torch.int32)
            cu_kv[1:] = ctx_lengths.cumsum(0)
            tcl = int(cu_kv[-1])
            rows = tcl if is_mla else H * tcl
            kc = _rounded((rows, D), f16, g)
            vc = _rounded((rows, D), f16, g)
            ref = refs["_reference_varlen_attention_with_cache"](q, k, v, lengths, kc, vc, cu_kv, 0.65, is_mla,
                                                                 causal_query_seq_attn=True)
            add(f"cmp_causal_ctx{int(with_ctx)}_mla{int(is_mla)}_f16",
                {"q": q, "k": k, "v": v, "lengths": lengths, "k_cache": kc, "v_cache": vc, "cu_kv": cu_kv,
                 "out": ref},
                {"kind": "compressed", "dtype": "f16", "scale": 0.65, "is_mla": is_mla, "causal": True,
                 "ctx": "batch" if with_ctx else "none", "total_context_len": tcl, "context_batch_size": B})

    # shared context (context_batch_size = 1), benchmark reference math (utils.py:365-407), non-MLA
    for dt, dtn, D in ((bf16, "bf16", 64), (f16, "f16", 128), (bf16, "bf16", 32), (f16, "f16", 16), (bf16, "bf16", 256)):
        g = torch.Generator().manual_seed(31 + D)
        B, H, N = 3, 2, 80
        lengths = torch.tensor([80, 1, 45], dtype=torch.int32)
        q, k, v = (_rounded((B, H, N, D), dt, g) for _ in range(3))
        tcl = 150
        cu_kv = torch.tensor([0, tcl], dtype=torch.int32)
        kc = _rounded((H * tcl, D), dt, g)
        vc = _rounded((H * tcl, D), dt, g)
        scale = 1.0 / math.sqrt(D)
        ref = bu._reference_varlen_attention_with_cache(q, k, v, lengths, kc, vc, cu_kv, scale, False, 1)
        add(f"cmp_shared_d{D}_{dtn}", {"q": q, "k": k, "v": v, "lengths": lengths, "k_cache": kc, "v_cache": vc,
                                      "cu_kv": cu_kv, "out": ref},
            {"kind": "compressed", "dtype": dtn, "scale": scale, "is_mla": False, "causal": False, "ctx": "shared",
             "total_context_len": tcl, "context_batch_size": 1})

    # dense, no cache (test_host.py:174-212) and with a flat per-batch / shared cache (:215-279)
    for is_mla in (False, True):
        g = torch.Generator().manual_seed(22)
        B, H, N, D = 2, 3, 24, 64
        q, k, v = (_rounded((B, H, N, D), f16, g) for _ in range(3))
        if is_mla:
            v = k
        empty = torch.empty((0, D))
        ref = refs["_reference_dense_attention_with_flat_cache"](q, k, v, empty, empty, 0, 0.6, is_mla, B)
        add(f"dense_nocache_mla{int(is_mla)}_f16", {"q": q, "k": k, "v": v, "out": ref},
            {"kind": "dense", "dtype": "f16", "scale": 0.6, "is_mla": is_mla, "context_len": 0,
             "context_batch_size": B})
        for ctx_bs in (B, 1):
            g = torch.Generator().manual_seed(23)
            Nc = 20
            q1, k1, v1 = (_rounded((B, H, Nc, D), f16, g) for _ in range(3))
            q2, k2, v2 = (_rounded((B, H, Nc, D), f16, g) for _ in range(3))
            if is_mla:
                kc = k1[:, 0].reshape(B * Nc, D)
                vc = kc
            else:
                kc = k1.reshape(B * H * Nc, D)
                vc = v1.reshape(B * H * Nc, D)
            ctx_len = Nc if ctx_bs == B else B * Nc
            ref = refs["_reference_dense_attention_with_flat_cache"](q2, k2, v2, kc, vc, ctx_len, 0.55, is_mla, ctx_bs)
            add(f"dense_cache_bs{ctx_bs}_mla{int(is_mla)}_f16",
                {"q": q2, "k": k2, "v": v2, "k_cache": kc, "v_cache": vc, "out": ref},
                {"kind": "dense", "dtype": "f16", "scale": 0.55, "is_mla": is_mla, "context_len": ctx_len,
                 "context_batch_size": ctx_bs})

    # dense B=2 H=8 N=128 D=64, N(0,1) fp32 cast to fp16, scale 1/8, no cache
    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn((2, 8, 128, 64), generator=g).to(f16).to(torch.float32) for _ in range(3))
    empty = torch.empty((0, 64))
    ref = refs["_reference_dense_attention_with_flat_cache"](q, k, v, empty, empty, 0, 0.125, False, 2)
    add("dense_config1_f16", {"q": q, "k": k, "v": v, "out": ref},
        {"kind": "dense", "dtype": "f16", "scale": 0.125, "is_mla": False, "context_len": 0, "context_batch_size": 2})
    return out, manifest


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the reference checkout (contains src/flash_mlm)")
    args = ap.parse_args()
    ref_root = Path(args.reference)
    sys.path.insert(0, str(ref_root / "src"))
    from flash_mlm.host import host_utils as hu  # noqa: E402  (reference package)
    from benchmark.standard_kernel import utils as bu  # noqa: E402

    refs = _load_test_host_refs(ref_root)
    (HERE / "metadata.json").write_text(json.dumps(metadata_cases(hu), indent=None, separators=(",", ":")))
    np.savez_compressed(HERE / "pack.npz", **pack_cases(hu))
    att, manifest = attention_cases(refs, bu)
    np.savez_compressed(HERE / "attention.npz", **att)
    (HERE / "attention_manifest.json").write_text(json.dumps(manifest, indent=1))
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".json", ".npz")))


if __name__ == "__main__":
    main()
