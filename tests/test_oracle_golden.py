"""The CPU oracle against golden vectors produced by the reference itself (CPU only)."""

import numpy as np
import pytest

import oracle
from golden_io import attention_case, attention_manifest, metadata_cases, pack_npz


@pytest.mark.parametrize("case", metadata_cases(), ids=lambda c: f"B{len(c['lengths'])}N{c['N']}bn{c['block_n']}")
def test_oracle_metadata_matches_reference(case):
    m = oracle.build_pack_metadata(case["lengths"], case["N"], case["block_n"])
    assert m["cu_seqlens"].tolist() == case["cu_seqlens"]
    assert m["token_indices"].tolist() == case["token_indices"]
    assert m["total_tokens"] == case["total_tokens"]
    assert m["batch_ids_q"].tolist() == case["batch_ids_q"]
    assert m["q_tile_starts_q"].tolist() == case["q_tile_starts_q"]
    for bn, tm in case["tile_maps_from_cu"].items():
        s, b = oracle.tile_map_from_cu_seqlens(case["cu_seqlens"], int(bn))
        assert s.tolist() == tm["starts"] and b.tolist() == tm["batch_ids"]
    for key, tot in case["total_q_len_padded"].items():
        bm, bn = map(int, key.split(","))
        assert oracle.total_q_len_padded(case["total_tokens"], case["cu_seqlens"], bm, bn) == tot


def test_reference_unit_test_golden_vector():
    # src/flash_mlm/host/test_host_utils.py:19-43
    m = oracle.build_pack_metadata([4, 2], 4, 3)
    assert m["cu_seqlens"].tolist() == [0, 4, 6]
    assert m["token_indices"].tolist() == [0, 1, 2, 3, 4, 5]
    assert m["batch_ids_q"].tolist() == [0, 0, 1]
    assert m["q_tile_starts_q"].tolist() == [0, 3, 4]


def test_oracle_rejects_bad_lengths():
    with pytest.raises(ValueError, match=r"lengths values must be in \[0, N\]"):
        oracle.build_pack_metadata([5, 1], 4, 2)
    with pytest.raises(ValueError, match="block_n must be >= 1"):
        oracle.build_pack_metadata([1, 1], 2, 0)


def _pack_case_ids():
    z = pack_npz()
    return sorted({k.split("_")[0] for k in z})


@pytest.mark.parametrize("cid", _pack_case_ids())
def test_oracle_pack_pad_unpack_match_reference(cid):
    z = pack_npz()
    B, H, N, D, bm, bn = z[cid + "_spec"].tolist()
    lengths = z[cid + "_lengths"]
    x = z[cid + "_x"]
    m = oracle.build_pack_metadata(lengths, N, bn)
    cu = m["cu_seqlens"]
    T = m["total_tokens"]
    packed = oracle.pack_rows(x, cu, T)
    np.testing.assert_array_equal(packed, z[cid + "_packed"])
    np.testing.assert_array_equal(oracle.unpack_rows(packed, cu, H, N), z[cid + "_unpacked"])
    tot, totm, totpad = z[cid + "_total_padded"].tolist()
    assert oracle.total_q_len_padded(T, cu, bm, bn) == tot == totm == totpad
    np.testing.assert_array_equal(oracle.pack_rows(x, cu, tot), z[cid + "_qpp"])
    np.testing.assert_array_equal(oracle.pack_rows(x + 100, cu, tot), z[cid + "_kpp"])
    np.testing.assert_array_equal(oracle.pack_rows((x + 100)[:, :1], cu, tot), z[cid + "_kpp_mla"])
    np.testing.assert_array_equal(oracle.pad_packed_rows(packed, H, T, totpad), z[cid + "_qpad"])


def _as_np(t):
    return t.float().numpy()


def run_oracle_case(params, t):
    """Run the oracle on a golden attention case; returns an array shaped like the golden `out`."""
    q, k, v = _as_np(t["q"]), _as_np(t["k"]), _as_np(t["v"])
    if params["kind"] == "dense":
        return oracle.attention_dense(
            q, k, v, params["scale"], k_cache=_as_np(t["k_cache"]) if "k_cache" in t else None,
            v_cache=_as_np(t["v_cache"]) if "v_cache" in t else None, context_len=params["context_len"],
            context_batch_size=params["context_batch_size"], is_mla=params["is_mla"])
    lengths = t["lengths"].numpy()
    B, H, N, D = q.shape
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    kw = {}
    if params["ctx"] != "none":
        kw = dict(k_cache=_as_np(t["k_cache"]), v_cache=_as_np(t["v_cache"]), cu_kv=t["cu_kv"].numpy(),
                  context_batch_size=params["context_batch_size"], total_context_len=params["total_context_len"])
    packed = oracle.attention_packed(q, k, v, cu, params["scale"], is_mla=params["is_mla"],
                                     causal_query_seq_attn=params["causal"], **kw)
    return oracle.unpack_rows(packed, cu, H, N)


@pytest.mark.parametrize("name", [c["name"] for c in attention_manifest()])
def test_oracle_attention_matches_reference_fp32(name):
    params, t = attention_case(name)
    got = run_oracle_case(params, t)
    np.testing.assert_allclose(got, t["out"].numpy(), atol=2e-5, rtol=0)


def run_torch_ref_case(params, t):
    """The torch restatement of the reference's CPU path on a golden case."""
    import torch

    from oracle import torch_ref

    q, k, v = (t[x].float() for x in ("q", "k", "v"))
    if params["kind"] == "dense":
        return torch_ref.dense_attention_with_cache(
            q, k, v, params["scale"], k_cache=t["k_cache"].float() if "k_cache" in t else None,
            v_cache=t["v_cache"].float() if "v_cache" in t else None, context_len=params["context_len"],
            context_batch_size=params["context_batch_size"], is_mla=params["is_mla"]).numpy()
    lengths = t["lengths"].numpy()
    B, H, N, D = q.shape
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int64)
    kw = {}
    if params["ctx"] != "none":
        kw = dict(k_cache=t["k_cache"].float(), v_cache=t["v_cache"].float(), cu_kv=t["cu_kv"].tolist(),
                  context_batch_size=params["context_batch_size"], total_context_len=params["total_context_len"])
    packed = torch_ref.varlen_attention_with_cache(q, k, v, cu, params["scale"], is_mla=params["is_mla"],
                                                   causal_query_seq_attn=params["causal"], **kw)
    return oracle.unpack_rows(packed.numpy(), cu, H, N)


@pytest.mark.parametrize("name", [c["name"] for c in attention_manifest()])
def test_torch_cpu_path_matches_reference_fp32(name):
    params, t = attention_case(name)
    got = run_torch_ref_case(params, t)
    np.testing.assert_allclose(got, t["out"].numpy(), atol=2e-5, rtol=0)
