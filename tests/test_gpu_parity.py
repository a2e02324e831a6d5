"""GPU parity: the CUDA path (through the public API and the C ABI) against the
reference's golden vectors and the CPU oracle.

Bars: metadata / pack / pad / unpack bit-exact; attention max-abs error
<= 2e-3 (fp16) and <= 8e-3 (bf16) against fp32 math on the same rounded inputs.
"""

import ctypes
import math

import numpy as np
import pytest
import torch

import oracle
from golden_io import attention_case, attention_manifest, metadata_cases, pack_npz

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 8e-3}
DEV = "cuda"


def fm():
    import flash_mlm

    return flash_mlm


def half_ulp(ref: torch.Tensor, dtype) -> torch.Tensor:
    """Half the spacing of `dtype` values at |ref| (the unavoidable output-rounding error)."""
    mant = 10 if dtype == torch.float16 else 7
    e = torch.floor(torch.log2(ref.abs().clamp_min(2.0 ** -14)))
    return 0.5 * torch.pow(2.0, e - mant)


# Raw max-abs-error bound of the north star: 2e-3 (f16), 8e-3 (bf16) against
# fp32 math on the same rounded inputs.  One exception, bf16 only: where
# |o| >= 2 the output format itself cannot get nearer than 7.8e-3 (half its
# spacing in [2, 4)), so there the bound is TOL plus that half-spacing.  Every
# call reports how many positions the exception covered (`last_tol_report`).
last_tol_report: dict = {}


def assert_close_tol(got: torch.Tensor, ref, dtype, what=""):
    ref_t = torch.as_tensor(ref, dtype=torch.float32)
    g = got.detach().float().cpu()
    assert torch.isfinite(g).all(), f"{what}: non-finite output"
    if not g.numel():
        return 0.0
    raw = (g - ref_t).abs()
    bound = torch.full_like(raw, TOL[dtype])
    wide = torch.zeros_like(raw, dtype=torch.bool)
    if dtype == torch.bfloat16:
        wide = ref_t.abs() >= 2.0
        bound = torch.where(wide, bound + half_ulp(ref_t, dtype), bound)
    last_tol_report.update(what=what, max_abs_err=raw.max().item(), n=raw.numel(), n_wide=int(wide.sum()))
    bad = raw > bound
    assert not bad.any(), (f"{what}: max abs err {raw.max().item():.3e} > {TOL[dtype]:.0e} at "
                           f"{int(bad.sum())} of {raw.numel()} positions")
    return raw.max().item()


def no_device_errors():
    fm().check_device_errors(torch.device(DEV, torch.cuda.current_device()))


# ----------------------------------------------------------------- metadata / pack


@pytest.mark.parametrize("case", metadata_cases(), ids=lambda c: f"B{len(c['lengths'])}N{c['N']}bn{c['block_n']}")
def test_build_pack_metadata_bit_exact(case):
    from flash_mlm.host.host_utils import _build_query_tile_map_from_cu_seqlens

    lengths = torch.tensor(case["lengths"], dtype=torch.int32, device=DEV)
    meta = fm().build_pack_metadata(lengths, case["N"], case["block_n"])
    assert meta.total_tokens == case["total_tokens"]
    assert meta.cu_seqlens.dtype == torch.int32 and meta.token_indices.dtype == torch.int64
    assert meta.cu_seqlens.cpu().tolist() == case["cu_seqlens"]
    assert meta.token_indices.cpu().tolist() == case["token_indices"]
    assert meta.batch_ids_q.cpu().tolist() == case["batch_ids_q"]
    assert meta.q_tile_starts_q.cpu().tolist() == case["q_tile_starts_q"]
    for bn, tm in case["tile_maps_from_cu"].items():
        s, b = _build_query_tile_map_from_cu_seqlens(meta.cu_seqlens, int(bn))
        assert s.cpu().tolist() == tm["starts"] and b.cpu().tolist() == tm["batch_ids"]


def test_build_pack_metadata_rejects_bad_lengths():
    with pytest.raises(ValueError, match=r"lengths values must be in \[0, N\]"):
        fm().build_pack_metadata(torch.tensor([5, 1], dtype=torch.int32, device=DEV), 4, 2)
    with pytest.raises(ValueError, match="block_n must be >= 1"):
        fm().build_pack_metadata(torch.tensor([1, 1], dtype=torch.int32, device=DEV), 2, 0)


def _pack_ids():
    return sorted({k.split("_")[0] for k in pack_npz()})


@pytest.mark.parametrize("cid", _pack_ids())
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_pack_pad_unpack_bit_exact(cid, dtype):
    from flash_mlm.host.host_utils import (
        pack_and_pad_main_tensors_for_mlm_compressed,
        pack_for_kernel,
        pad_packed_main_tensors_for_mlm_compressed,
    )

    z = pack_npz()
    B, H, N, D, bm, bn = z[cid + "_spec"].tolist()
    x32 = torch.from_numpy(z[cid + "_x"])
    x = x32.to(dtype).to(DEV)
    xk, xv = (x32 + 100).to(dtype).to(DEV), (x32 + 200).to(dtype).to(DEV)
    meta = fm().build_pack_metadata(torch.from_numpy(z[cid + "_lengths"]).to(DEV), N, bn)

    def ref(key):
        return torch.from_numpy(z[cid + key]).to(dtype)

    packed = pack_for_kernel(x, meta, flatten_for_kernel=True)
    assert torch.equal(packed.cpu(), ref("_packed"))
    assert torch.equal(pack_for_kernel(x, meta).cpu(), ref("_packed").view(H, -1, D))
    assert torch.equal(fm().unpack_from_kernel(packed, meta, H).cpu(), ref("_unpacked"))
    tot = int(z[cid + "_total_padded"][0])
    qp, kp, vp, t2 = pack_and_pad_main_tensors_for_mlm_compressed(
        x, xk, xv, q_meta=meta, num_heads=H, is_mla=False, block_m=bm, block_n=bn)
    assert t2 == tot
    assert torch.equal(qp.cpu(), ref("_qpp"))
    assert torch.equal(kp.cpu(), ref("_kpp"))
    _, kpm, vpm, _ = pack_and_pad_main_tensors_for_mlm_compressed(
        x, xk, xv, q_meta=meta, num_heads=H, is_mla=True, block_m=bm, block_n=bn)
    assert vpm is kpm and torch.equal(kpm.cpu(), ref("_kpp_mla"))
    qpad, _, _, t3 = pad_packed_main_tensors_for_mlm_compressed(
        packed, pack_for_kernel(xk, meta, True), pack_for_kernel(xv, meta, True), num_heads=H,
        is_mla=False, total_q_len_unpadded=meta.total_tokens, cu_seqlens_q=meta.cu_seqlens, block_m=bm, block_n=bn)
    assert t3 == tot
    assert torch.equal(qpad.cpu(), ref("_qpad"))


def test_unpack_writes_zeros_over_garbage():
    lengths = torch.tensor([3, 0, 5], dtype=torch.int32, device=DEV)
    meta = fm().build_pack_metadata(lengths, 6, 4)
    packed = torch.randn(2 * 8, 16, device=DEV)
    out = fm().unpack_from_kernel(packed, meta, H=2)
    ref = oracle.unpack_rows(packed.cpu().numpy(), meta.cu_seqlens.cpu().numpy(), 2, 6)
    assert torch.equal(out.cpu(), torch.from_numpy(ref))


# ----------------------------------------------------------------- attention vs golden


def _cuda(t):
    return t.to(DEV)


def run_case_gpu(params, t):
    """Run a golden case through the public API; returns a [B,H,N,D] result (CPU fp32)."""
    dt = t["q"].dtype
    q, k, v = _cuda(t["q"]), _cuda(t["k"]), _cuda(t["v"])
    B, H, N, D = q.shape
    scale = params["scale"]
    if params["kind"] == "dense":
        cache, lid = None, None
        if params["context_len"] > 0:
            cache, lid = fm().InferenceCache(), 5
            total = params["context_len"] * params["context_batch_size"]
            cache.prefill_kv_cache(lid, k_cache=_cuda(t["k_cache"]), v_cache=_cuda(t["v_cache"]),
                                   total_context_len=total if params["context_batch_size"] == 1 else None,
                                   context_batch_size=params["context_batch_size"], is_mla=params["is_mla"],
                                   num_heads=H, head_dim=D)
        out = fm().flash_attn_mlm(q, k, v, scale=scale, inference_cache=cache, layer_id=lid, is_mla=params["is_mla"],
                                  context_batch_size=params["context_batch_size"] if cache else None)
        return out.float().cpu()
    lengths = _cuda(t["lengths"])
    meta = fm().build_pack_metadata(lengths, N, 32)
    cache = fm().InferenceCache()
    if params["ctx"] != "none":
        cache.prefill_kv_cache(0, k_cache=_cuda(t["k_cache"]), v_cache=_cuda(t["v_cache"]),
                               total_context_len=params["total_context_len"], cu_seqlens_kv=_cuda(t["cu_kv"]),
                               context_batch_size=params["context_batch_size"], is_mla=params["is_mla"], num_heads=H,
                               head_dim=D)
    packed = fm().flash_attn_mlm_compressed(q, k, v, num_heads=H, q_meta=meta, scale=scale, inference_cache=cache,
                                            layer_id=0, is_mla=params["is_mla"], block_m=32, block_n=32,
                                            causal_query_seq_attn=params["causal"],
                                            context_batch_size=params.get("context_batch_size"))
    assert packed.shape == (H * meta.total_tokens, D) and packed.dtype == dt
    return fm().unpack_from_kernel(packed, meta, H).float().cpu()


@pytest.mark.parametrize("name", [c["name"] for c in attention_manifest()])
def test_attention_matches_reference_golden(name):
    params, t = attention_case(name)
    got = run_case_gpu(params, t)
    assert_close_tol(got, t["out"], t["q"].dtype, name)
    no_device_errors()


# ----------------------------------------------------------------- reference test scenarios


@pytest.mark.parametrize("is_mla", [False, True])
def test_prefill_requires_cache(is_mla):
    q = torch.randn(2, 2, 16, 64, device=DEV, dtype=torch.float16)
    with pytest.raises(ValueError, match="prefill=True requires inference_cache"):
        fm().flash_attn_mlm(q, q, q, scale=0.5, is_mla=is_mla, prefill=True)
    meta = fm().build_pack_metadata(torch.tensor([16, 9], device=DEV, dtype=torch.int32), 16, block_n=32)
    with pytest.raises(ValueError, match="prefill=True requires inference_cache"):
        fm().flash_attn_mlm_compressed(q, q, q, num_heads=2, scale=0.5, q_meta=meta, is_mla=is_mla, block_m=32,
                                       block_n=32, prefill=True)


@pytest.mark.parametrize("is_mla", [False, True])
def test_dense_prefill_then_cached_context(is_mla):
    torch.manual_seed(23)
    B, H, N, D = 2, 2, 20, 64
    q1, k1, v1, q2, k2, v2 = (torch.randn(B, H, N, D, device=DEV, dtype=torch.float16) for _ in range(6))
    cache = fm().InferenceCache()
    out1 = fm().flash_attn_mlm(q1, k1, v1, scale=0.55, inference_cache=cache, layer_id=3, is_mla=is_mla, prefill=True)
    ref1 = oracle.attention_dense(q1.float().cpu().numpy(), k1.float().cpu().numpy(), v1.float().cpu().numpy(), 0.55,
                                  is_mla=is_mla)
    assert_close_tol(out1, ref1, torch.float16, "prefill call")
    out2 = fm().flash_attn_mlm(q2, k2, v2, scale=0.55, inference_cache=cache, layer_id=3, is_mla=is_mla,
                               context_batch_size=B)
    e = cache.get_kv_cache(3, is_mla=is_mla, num_heads=H, head_dim=D, dtype=q2.dtype, device=q2.device)
    ctx_len = e.total_context_len // e.context_batch_size
    ref2 = oracle.attention_dense(q2.float().cpu().numpy(), k2.float().cpu().numpy(), v2.float().cpu().numpy(), 0.55,
                                  k_cache=e.k_cache.float().cpu().numpy(),
                                  v_cache=(e.k_cache if is_mla else e.v_cache).float().cpu().numpy(),
                                  context_len=ctx_len, context_batch_size=e.context_batch_size, is_mla=is_mla)
    assert_close_tol(out2, ref2, torch.float16, "cached call")
    no_device_errors()


@pytest.mark.parametrize("is_mla", [False, True])
def test_compressed_prefill_stores_entry_then_serves_it(is_mla):
    torch.manual_seed(13)
    B, H, N, D = 2, 2, 20, 64
    lengths = torch.tensor([20, 7], device=DEV, dtype=torch.int32)
    q, k, v = (torch.randn(B, H, N, D, device=DEV, dtype=torch.float16) for _ in range(3))
    meta = fm().build_pack_metadata(lengths, N, block_n=32)
    cache = fm().InferenceCache()
    out = fm().flash_attn_mlm_compressed(q, k, v, num_heads=H, scale=0.55, q_meta=meta, inference_cache=cache,
                                         layer_id=7, is_mla=is_mla, block_m=32, block_n=32, prefill=True)
    stored = cache.get_kv_cache(7, is_mla=is_mla, num_heads=H, head_dim=D, dtype=q.dtype, device=q.device)
    assert int(stored.cu_seqlens_kv[-1].item()) == 27
    assert stored.total_context_len == 32 + 0 or stored.total_context_len >= 27
    rows = stored.total_context_len if is_mla else H * stored.total_context_len
    assert stored.k_cache.shape[0] == rows and stored.context_batch_size == B
    # stored K/V equal the reference pack (+ zero padding)
    cu = meta.cu_seqlens.cpu().numpy()
    ksrc = k[:, :1] if is_mla else k
    ref_k = oracle.pack_rows(ksrc.float().cpu().numpy(), cu, stored.total_context_len)
    assert np.array_equal(stored.k_cache.float().cpu().numpy(), ref_k)
    # prefill output attends only to its own tokens
    qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
    ref = oracle.attention_packed(qn, kn, vn, cu, 0.55, is_mla=is_mla)
    assert_close_tol(out, ref, torch.float16, "prefill")
    # a later query call sees that context
    q2 = torch.randn(B, H, N, D, device=DEV, dtype=torch.float16)
    out2 = fm().flash_attn_mlm_compressed(q2, k, v, num_heads=H, scale=0.55, q_meta=meta, inference_cache=cache,
                                          layer_id=7, is_mla=is_mla, block_m=32, block_n=32)
    ref2 = oracle.attention_packed(q2.float().cpu().numpy(), kn, vn, cu, 0.55,
                                   k_cache=stored.k_cache.float().cpu().numpy(),
                                   v_cache=(stored.k_cache if is_mla else stored.v_cache).float().cpu().numpy(),
                                   cu_kv=cu, context_batch_size=B, total_context_len=stored.total_context_len,
                                   is_mla=is_mla)
    assert_close_tol(out2, ref2, torch.float16, "query after prefill")
    no_device_errors()


def _pre_inputs(q, k, v, meta, is_mla):
    from flash_mlm.host.host_utils import pack_for_kernel

    qp = pack_for_kernel(q, meta, flatten_for_kernel=True)
    if is_mla:
        kp = pack_for_kernel(k[:, :1], meta, flatten_for_kernel=False).squeeze(0)
        vp = kp
    else:
        kp = pack_for_kernel(k, meta, flatten_for_kernel=True)
        vp = pack_for_kernel(v, meta, flatten_for_kernel=True)
    return qp, kp, vp


@pytest.mark.parametrize("is_mla", [False, True])
@pytest.mark.parametrize("with_cache", [False, True])
def test_precompressed_matches_compressed(is_mla, with_cache):
    torch.manual_seed(51)
    B, H, N, D = 2, 3, 48, 64
    lengths = torch.tensor([48, 37], device=DEV, dtype=torch.int32)
    q, k, v = (torch.randn(B, H, N, D, device=DEV, dtype=torch.float16) for _ in range(3))
    ctx_l = torch.tensor([13, 9] if with_cache else [0, 0], device=DEV, dtype=torch.int32)
    cu_kv = torch.zeros(B + 1, device=DEV, dtype=torch.int32)
    cu_kv[1:] = ctx_l.cumsum(0)
    tcl = int(cu_kv[-1])
    rows = tcl if is_mla else H * tcl
    kc = torch.randn(rows, D, device=DEV, dtype=torch.float16)
    vc = torch.randn_like(kc)

    def mk():
        c = fm().InferenceCache()
        c.prefill_kv_cache(0, k_cache=kc, v_cache=vc, total_context_len=tcl, cu_seqlens_kv=cu_kv,
                           context_batch_size=B, is_mla=is_mla, num_heads=H, head_dim=D)
        return c

    meta = fm().build_pack_metadata(lengths, N, block_n=32)
    ref = fm().flash_attn_mlm_compressed(q, k, v, num_heads=H, scale=0.5, q_meta=meta, inference_cache=mk(),
                                         layer_id=0, is_mla=is_mla, block_m=32, block_n=32)
    qp, kp, vp = _pre_inputs(q, k, v, meta, is_mla)
    pre = fm().flash_attn_mlm_precompressed(qp, kp, vp, num_heads=H, total_q_len=qp.shape[0] // H,
                                            cu_seqlens_q=meta.cu_seqlens, batch_ids_q=meta.batch_ids_q,
                                            q_tile_starts_q=meta.q_tile_starts_q, scale=0.5, inference_cache=mk(),
                                            layer_id=0, is_mla=is_mla, block_m=32, block_n=32)
    torch.testing.assert_close(pre, ref, atol=1e-5, rtol=0)
    no_device_errors()


@pytest.mark.parametrize("is_mla", [False, True])
def test_precompressed_prefill_stores_entry(is_mla):
    torch.manual_seed(52)
    B, H, N, D = 2, 2, 20, 64
    lengths = torch.tensor([20, 7], device=DEV, dtype=torch.int32)
    q, k, v = (torch.randn(B, H, N, D, device=DEV, dtype=torch.float16) for _ in range(3))
    meta = fm().build_pack_metadata(lengths, N, block_n=32)
    qp, kp, vp = _pre_inputs(q, k, v, meta, is_mla)
    cache = fm().InferenceCache()
    fm().flash_attn_mlm_precompressed(qp, kp, vp, num_heads=H, total_q_len=qp.shape[0] // H,
                                      cu_seqlens_q=meta.cu_seqlens, batch_ids_q=meta.batch_ids_q,
                                      q_tile_starts_q=meta.q_tile_starts_q, scale=0.55, inference_cache=cache,
                                      layer_id=7, is_mla=is_mla, block_m=32, block_n=32, prefill=True)
    stored = cache.get_kv_cache(7, is_mla=is_mla, num_heads=H, head_dim=D, dtype=q.dtype, device=q.device)
    assert int(stored.cu_seqlens_kv[-1].item()) == 27
    assert stored.total_context_len >= 27
    assert stored.context_batch_size == B


# ----------------------------------------------------------------- randomized sweeps vs oracle


def _rand(shape, dtype, gen, scale=1.0):
    return (torch.randn(shape, generator=gen) * scale).to(dtype)


@pytest.mark.parametrize("D", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("is_mla", [False, True])
def test_compressed_random_vs_oracle(D, dtype, is_mla):
    g = torch.Generator().manual_seed(1000 + D)
    B, H, N = 4, 3, 300
    lengths = torch.tensor([300, 1, 129, 257], dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), dtype, g) for _ in range(3))
    ctx = torch.tensor([0, 200, 33, 140], dtype=torch.int32)
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1]) + 5  # a few unused padding rows at the end of the cache
    rows = tcl if is_mla else H * tcl
    kc, vc = _rand((rows, D), dtype, g), _rand((rows, D), dtype, g)
    scale = 1.0 / math.sqrt(D)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(1, k_cache=kc.to(DEV), v_cache=vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=B, is_mla=is_mla, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=scale,
                                         inference_cache=cache, layer_id=1, is_mla=is_mla, block_n=64)
    cu = meta.cu_seqlens.cpu().numpy()
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(), cu, scale,
                                  k_cache=kc.float().numpy(), v_cache=vc.float().numpy(), cu_kv=cu_kv.numpy(),
                                  context_batch_size=B, total_context_len=tcl, is_mla=is_mla)
    assert_close_tol(out, ref, dtype, f"D={D}")
    no_device_errors()


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("shared", [False, True])
def test_causal_prefix_long_vs_oracle(D, shared):
    g = torch.Generator().manual_seed(77 + D)
    B, H, N = 5, 2, 260
    lengths = torch.tensor([260, 3, 200, 0, 131], dtype=torch.int32)
    dtype = torch.float16
    q, k, v = (_rand((B, H, N, D), dtype, g) for _ in range(3))
    tcl = 700
    cu_kv = torch.tensor([0, tcl], dtype=torch.int32) if shared else torch.tensor([0, 100, 300, 300, 650, 700],
                                                                                     dtype=torch.int32)
    kc, vc = _rand((H * tcl, D), dtype, g), _rand((H * tcl, D), dtype, g)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(2, k_cache=kc.to(DEV), v_cache=vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=1 if shared else B, is_mla=False,
                           num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 32)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=0.125,
                                         inference_cache=cache, layer_id=2, causal_query_seq_attn=True)
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), 0.125, k_cache=kc.float().numpy(),
                                  v_cache=vc.float().numpy(), cu_kv=cu_kv.numpy(),
                                  context_batch_size=1 if shared else B, total_context_len=tcl,
                                  causal_query_seq_attn=True)
    assert_close_tol(out, ref, dtype, "causal")
    no_device_errors()


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_dense_random_vs_oracle(D, dtype):
    g = torch.Generator().manual_seed(5 + D)
    B, H, N = 3, 2, 333
    q, k, v = (_rand((B, H, N, D), dtype, g) for _ in range(3))
    ctx_len = 190
    kc, vc = _rand((B * H * ctx_len, D), dtype, g), _rand((B * H * ctx_len, D), dtype, g)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), v_cache=vc.to(DEV), context_batch_size=B, is_mla=False,
                           num_heads=H, head_dim=D)
    out = fm().flash_attn_mlm(q.to(DEV), k.to(DEV), v.to(DEV), scale=1.0 / math.sqrt(D), inference_cache=cache,
                              layer_id=0, context_batch_size=B)
    ref = oracle.attention_dense(q.float().numpy(), k.float().numpy(), v.float().numpy(), 1.0 / math.sqrt(D),
                                 k_cache=kc.float().numpy(), v_cache=vc.float().numpy(), context_len=ctx_len,
                                 context_batch_size=B)
    assert_close_tol(out, ref, dtype, "dense")
    no_device_errors()


def test_nonfinite_padding_is_ignored():
    """Padding positions of q/k/v (t >= length) may hold NaN/Inf; results must not change."""
    g = torch.Generator().manual_seed(3)
    B, H, N, D = 3, 2, 200, 64
    lengths = torch.tensor([77, 200, 130], dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), torch.bfloat16, g) for _ in range(3))
    qn, kn, vn = q.clone(), k.clone(), v.clone()
    for b, L in enumerate(lengths.tolist()):
        for x in (qn, kn, vn):
            x[b, :, L:] = float("nan")
        kn[b, :, L:L + 3] = float("inf")
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 32)
    for is_mla in (False, True):
        a = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=0.125,
                                           is_mla=is_mla)
        b_ = fm().flash_attn_mlm_compressed(qn.to(DEV), kn.to(DEV), vn.to(DEV), num_heads=H, q_meta=meta,
                                            scale=0.125, is_mla=is_mla)
        assert torch.isfinite(b_.float()).all()
        torch.testing.assert_close(a, b_, atol=0, rtol=0)
    no_device_errors()


def test_empty_and_ragged_edges():
    """All-empty batch, a single-token batch and a batch whose sequences are all empty but one."""
    dtype = torch.float16
    for lengths, N in (([0, 0, 0], 8), ([1], 1), ([0, 0, 513, 0], 513)):
        g = torch.Generator().manual_seed(len(lengths) * 7 + N)
        B, H, D = len(lengths), 2, 64
        q, k, v = (_rand((B, H, N, D), dtype, g) for _ in range(3))
        meta = fm().build_pack_metadata(torch.tensor(lengths, dtype=torch.int32, device=DEV), N, 32)
        out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=0.1)
        assert out.shape == (H * sum(lengths), D)
        ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                      meta.cu_seqlens.cpu().numpy(), 0.1)
        assert_close_tol(out, ref, dtype, f"lengths={lengths}")
    no_device_errors()


# Covers the O rescale of every TMEM layout: separate P (64, 256), P over S
# with two tiles (128), and the MLA double S buffer (512), where the rescale
# first waits for the previous block's PV.
@pytest.mark.parametrize("D", [64, 128, 256, 512])
def test_large_logits_rescale_path(D):
    """Logit scales that force the running-max correction many times per row."""
    g = torch.Generator().manual_seed(9 + D)
    is_mla = D == 512
    B, H, N = 2, 2, 640
    dt = torch.float16
    q = _rand((B, H, N, D), dt, g, 3.0)
    # Key norms grow along the sequence, so later blocks raise the row max many
    # times over.  Such logits make the softmax nearly one-hot, and then P's
    # rounding to f16 before P V (as in the reference kernel) costs up to
    # 2^-11 * |V| per output: keys and values are clamped to |x| <= 1.5
    # (with MLA V is K), which keeps that under the raw 2e-3 bound.
    ramp = torch.linspace(0.1, 1.0, N).view(1, 1, N, 1)
    k = (torch.randn((B, H, N, D), generator=g) * ramp).clamp(-1.5, 1.5).to(dt)
    v = k if is_mla else torch.randn((B, H, N, D), generator=g).clamp(-1.5, 1.5).to(dt)
    scale = 4.0 / math.sqrt(D)
    out = fm().flash_attn_mlm(q.to(DEV), k.to(DEV), v.to(DEV), scale=scale, is_mla=is_mla)
    ref = oracle.attention_dense(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale, is_mla=is_mla)
    assert_close_tol(out, ref, dt, f"rescale D={D}")
    no_device_errors()


# ----------------------------------------------------------------- index-mapped context (no reference counterpart)
# Query sequence b attends context entry context_index[b]; several sequences
# share entries and the entry count differs from the batch size.


@pytest.mark.parametrize("D,dt,is_mla", [(64, torch.bfloat16, False), (128, torch.float16, False),
                                         (512, torch.bfloat16, True)])
def test_context_index_vs_oracle(D, dt, is_mla):
    g = torch.Generator().manual_seed(77 + D)
    B, H, N = 5, 1 if is_mla else 3, 130
    lengths = torch.tensor([130, 17, 64, 1, 99], dtype=torch.int32)
    q = _rand((B, H, N, D), dt, g, 0.5)
    k = _rand((B, 1 if is_mla else H, N, D), dt, g, 0.5).expand(B, H, N, D) if is_mla else _rand((B, H, N, D), dt, g)
    v = k if is_mla else _rand((B, H, N, D), dt, g)
    ctx = torch.tensor([300, 0, 129], dtype=torch.int32)  # three entries, one empty
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1])
    rows = tcl if is_mla else H * tcl
    kc = _rand((rows, D), dt, g, 0.5)
    vc = kc if is_mla else _rand((rows, D), dt, g)
    index = torch.tensor([2, 0, 2, 1, 0], dtype=torch.int32)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), v_cache=None if is_mla else vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=3, is_mla=is_mla, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 32)
    scale = D ** -0.5
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=scale,
                                         inference_cache=cache, layer_id=0, is_mla=is_mla,
                                         context_index=index.to(DEV))
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), scale, k_cache=kc.float().numpy(),
                                  v_cache=vc.float().numpy(), cu_kv=cu_kv.numpy(), context_batch_size=3,
                                  total_context_len=tcl, is_mla=is_mla, context_index=index.numpy())
    assert_close_tol(out, ref, dt, f"context_index D={D}")
    no_device_errors()


def test_context_index_rejections():
    g = torch.Generator().manual_seed(5)
    B, H, N, D = 2, 2, 16, 64
    q = _rand((B, H, N, D), torch.float16, g).to(DEV)
    cache = fm().InferenceCache()
    kc = _rand((H * 8, D), torch.float16, g).to(DEV)
    cache.prefill_kv_cache(0, k_cache=kc, v_cache=kc.clone(), total_context_len=8,
                           cu_seqlens_kv=torch.tensor([0, 5, 8], dtype=torch.int32, device=DEV),
                           context_batch_size=2, is_mla=False, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(torch.tensor([16, 9], dtype=torch.int32, device=DEV), N, 32)
    call = lambda **kw: fm().flash_attn_mlm_compressed(q, q, q, num_heads=H, q_meta=meta, scale=0.125, **kw)
    idx = torch.tensor([1, 0], dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match="requires inference_cache"):
        call(context_index=idx)
    with pytest.raises(ValueError, match="shape \\[B\\]"):
        call(inference_cache=cache, layer_id=0, context_index=idx.long())
    with pytest.raises(ValueError, match="lie in \\[0, 2\\)"):
        call(inference_cache=cache, layer_id=0, context_index=torch.tensor([1, 2], dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError, match="prefill"):
        call(inference_cache=cache, layer_id=1, context_index=idx, prefill=True)
    with pytest.raises(ValueError, match="leave context_batch_size unset"):
        call(inference_cache=cache, layer_id=0, context_index=idx, context_batch_size=2)
    no_device_errors()


# ----------------------------------------------------------------- head_dim 128, both item granularities
# At head_dim 128 a problem with fewer 256-row tile pairs than SMs runs one
# 128-row tile per work item; larger ones run two tiles per item.  Small and
# large problems exercise both.


@pytest.mark.parametrize("B,H", [(2, 3), (16, 16)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_head_dim_128_both_item_sizes(B, H, dt):
    g = torch.Generator().manual_seed(128 + B + H)
    N, D = 256, 128
    lengths = torch.randint(1, N + 1, (B,), generator=g, dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), dt, g) for _ in range(3))
    ctx = torch.randint(0, 200, (B,), generator=g, dtype=torch.int32)
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1])
    kc, vc = (_rand((H * tcl, D), dt, g) for _ in range(2))
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), v_cache=vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=B, is_mla=False, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta,
                                         scale=D ** -0.5, inference_cache=cache, layer_id=0, block_n=64)
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), D ** -0.5, k_cache=kc.float().numpy(),
                                  v_cache=vc.float().numpy(), cu_kv=cu_kv.numpy(), context_batch_size=B,
                                  total_context_len=tcl)
    assert_close_tol(out, ref, dt, f"D=128 B={B} H={H}")
    no_device_errors()


# ----------------------------------------------------------------- long per-sequence contexts
# Few work items, each walking a long context (up to 47 key blocks) then its
# own tokens; two identical calls must give bit-identical outputs.


@pytest.mark.parametrize("D,dt", [(64, torch.bfloat16), (64, torch.float16), (128, torch.bfloat16), (256, torch.float16)])
def test_long_context_vs_oracle_and_repeatable(D, dt):
    g = torch.Generator().manual_seed(900 + D)
    B, H, N = 3, 2, 300
    lengths = torch.tensor([300, 7, 170], dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), dt, g) for _ in range(3))
    ctx = torch.tensor([3000, 129, 1500], dtype=torch.int32)
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1])
    kc, vc = (_rand((H * tcl, D), dt, g) for _ in range(2))
    scale = D ** -0.5
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), v_cache=vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=B, is_mla=False, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=scale,
                                         inference_cache=cache, layer_id=0, block_n=64)
    out2 = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=scale,
                                          inference_cache=cache, layer_id=0, block_n=64)
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), scale, k_cache=kc.float().numpy(),
                                  v_cache=vc.float().numpy(), cu_kv=cu_kv.numpy(), context_batch_size=B,
                                  total_context_len=tcl)
    assert_close_tol(out, ref, dt, f"long context D={D}")
    assert torch.equal(out, out2)
    no_device_errors()


# ----------------------------------------------------------------- MLA with a 512-wide latent (no reference counterpart)


# H=64 gives more work items than CTAs, so CTAs run several items back to back,
# each ending on a partial key block whose caller padding is cleared in shared memory.
@pytest.mark.parametrize("H", [4, 64])
@pytest.mark.parametrize("causal", [False, True])
def test_mla_latent512_compressed_vs_oracle(causal, H):
    g = torch.Generator().manual_seed(512 + causal + H)
    B, N, D = 3, 70, 512
    lengths = torch.tensor([70, 5, 41], dtype=torch.int32)
    q = (_rand((B, H, N, D), torch.bfloat16, g, 0.5))
    k = (_rand((B, 1, N, D), torch.bfloat16, g, 0.5)).expand(B, H, N, D)
    ctx = torch.tensor([100, 0, 37], dtype=torch.int32)
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1])
    kc = _rand((tcl, D), torch.bfloat16, g, 0.5)
    scale = 1.0 / math.sqrt(D)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), total_context_len=tcl, cu_seqlens_kv=cu_kv.to(DEV),
                           context_batch_size=B, is_mla=True, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 32)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), k.to(DEV), num_heads=H, q_meta=meta, scale=scale,
                                         inference_cache=cache, layer_id=0, is_mla=True,
                                         causal_query_seq_attn=causal)
    kn = k.float().numpy()
    ref = oracle.attention_packed(q.float().numpy(), kn, kn, meta.cu_seqlens.cpu().numpy(), scale,
                                  k_cache=kc.float().numpy(), v_cache=kc.float().numpy(), cu_kv=cu_kv.numpy(),
                                  context_batch_size=B, total_context_len=tcl, is_mla=True,
                                  causal_query_seq_attn=causal)
    assert_close_tol(out, ref, torch.bfloat16, "mla512")
    no_device_errors()


def test_mla_latent512_dense_and_rejections():
    g = torch.Generator().manual_seed(77)
    B, H, N, D = 2, 3, 50, 512
    q, k = (_rand((B, H, N, D), torch.bfloat16, g, 0.5) for _ in range(2))
    out = fm().flash_attn_mlm(q.to(DEV), k.to(DEV), k.to(DEV), scale=0.05, is_mla=True)
    ref = oracle.attention_dense(q.float().numpy(), k.float().numpy(), k.float().numpy(), 0.05, is_mla=True)
    assert_close_tol(out, ref, torch.bfloat16, "mla512 dense")
    with pytest.raises(ValueError, match="HEAD_DIM must be one of"):
        fm().flash_attn_mlm(q.to(DEV), k.to(DEV), k.to(DEV), scale=0.05, is_mla=False)
    no_device_errors()


@pytest.mark.gpu
def test_bounded_wait_gives_up_and_context_stays_usable():
    """A wait on a barrier nobody arrives on ends after its limit with an error
    status; the context keeps working (a normal call afterwards is correct)."""
    import time

    from flash_mlm import _lib

    dev = torch.device("cuda", 0)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    L = _lib.lib()
    t0 = time.perf_counter()
    assert L.fmlm_selftest_bounded_wait(ctypes.c_void_p(err.data_ptr()), 2_000_000, _lib.stream_ptr(dev)) == 0
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(err.item()) == 1
    q = torch.randn(1, 2, 64, 64, device=dev, dtype=torch.float16)
    out = fm().flash_attn_mlm(q, q, q, scale=0.125)
    ref = torch.softmax((q.float() @ q.float().transpose(-1, -2)) * 0.125, -1) @ q.float()
    assert (out.float() - ref).abs().max().item() < 2e-3


# ----------------------------------------------------------------- precompressed entry against the oracle


@pytest.mark.parametrize("is_mla,causal,dt", [(False, False, torch.float16), (False, True, torch.bfloat16),
                                              (True, False, torch.bfloat16), (True, True, torch.float16)])
def test_precompressed_vs_oracle(is_mla, causal, dt):
    """flash_attn_mlm_precompressed on packed inputs with a per-sequence context, against the fp32 oracle."""
    from flash_mlm.host.host_utils import pack_for_kernel

    g = torch.Generator().manual_seed(600 + 2 * is_mla + causal)
    B, H, N, D = 4, 3, 150, (512 if is_mla and not causal else 64)
    lengths = torch.tensor([150, 1, 77, 129], dtype=torch.int32)
    q = _rand((B, H, N, D), dt, g, 0.5 if is_mla else 1.0)
    k = _rand((B, H, N, D), dt, g, 0.5 if is_mla else 1.0)
    v = _rand((B, H, N, D), dt, g)
    ctx = torch.tensor([64, 0, 200, 31], dtype=torch.int32)
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1])
    rows = tcl if is_mla else H * tcl
    kc = _rand((rows, D), dt, g, 0.5 if is_mla else 1.0)
    vc = kc if is_mla else _rand((rows, D), dt, g)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), v_cache=None if is_mla else vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=B, is_mla=is_mla, num_heads=H,
                           head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 32)
    qp = pack_for_kernel(q.to(DEV), meta, flatten_for_kernel=True)
    if is_mla:
        kp = pack_for_kernel(k[:, :1].to(DEV), meta, flatten_for_kernel=True)
        vp = kp
    else:
        kp = pack_for_kernel(k.to(DEV), meta, flatten_for_kernel=True)
        vp = pack_for_kernel(v.to(DEV), meta, flatten_for_kernel=True)
    T = meta.total_tokens
    scale = D ** -0.5
    out = fm().flash_attn_mlm_precompressed(qp, kp, vp, num_heads=H, total_q_len=T, cu_seqlens_q=meta.cu_seqlens,
                                            batch_ids_q=meta.batch_ids_q, q_tile_starts_q=meta.q_tile_starts_q,
                                            scale=scale, inference_cache=cache, layer_id=0, is_mla=is_mla,
                                            block_m=32, block_n=32, causal_query_seq_attn=causal)
    kk = k[:, :1].expand(B, H, N, D) if is_mla else k
    ref = oracle.attention_packed(q.float().numpy(), kk.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), scale, k_cache=kc.float().numpy(),
                                  v_cache=vc.float().numpy(), cu_kv=cu_kv.numpy(), context_batch_size=B,
                                  total_context_len=tcl, is_mla=is_mla, causal_query_seq_attn=causal)
    assert out.shape == (H * T, D)
    assert_close_tol(out, ref, dt, f"precompressed mla={is_mla} causal={causal}")
    no_device_errors()


# ----------------------------------------------------------------- padded output written by the epilogue


@pytest.mark.parametrize("D,dt,is_mla,causal", [(16, torch.float16, False, False), (64, torch.bfloat16, False, True),
                                                (128, torch.bfloat16, False, False), (128, torch.float16, True, False),
                                                (256, torch.float16, False, False), (512, torch.bfloat16, True, True)])
def test_padded_output_equals_unpacked_packed_output(D, dt, is_mla, causal):
    """out_layout="padded" is unpack_from_kernel(packed output), bit for bit: data rows,
    zero rows past each sequence (including empty sequences and rows past the last tile)."""
    g = torch.Generator().manual_seed(700 + D + is_mla + causal)
    B, H, N = 6, (2 if D == 512 else 3), 300
    lengths = torch.tensor([300, 0, 129, 1, 256, 40], dtype=torch.int32)
    q = _rand((B, H, N, D), dt, g, 0.5)
    k = _rand((B, H, N, D), dt, g, 0.5)
    v = _rand((B, H, N, D), dt, g)
    ctx = torch.tensor([10, 300, 0, 64, 129, 7], dtype=torch.int32)
    cu_kv = torch.cat([torch.zeros(1, dtype=torch.int32), ctx.cumsum(0).to(torch.int32)])
    tcl = int(cu_kv[-1])
    rows = tcl if is_mla else H * tcl
    kc, vc = _rand((rows, D), dt, g, 0.5), _rand((rows, D), dt, g)
    cache = fm().InferenceCache()
    cache.prefill_kv_cache(0, k_cache=kc.to(DEV), v_cache=None if is_mla else vc.to(DEV), total_context_len=tcl,
                           cu_seqlens_kv=cu_kv.to(DEV), context_batch_size=B, is_mla=is_mla, num_heads=H, head_dim=D)
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    kw = dict(num_heads=H, q_meta=meta, scale=D ** -0.5, inference_cache=cache, layer_id=0, is_mla=is_mla,
              causal_query_seq_attn=causal, block_n=64)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    packed = fm().flash_attn_mlm_compressed(qd, kd, vd, **kw)
    # the padded output over a buffer full of NaN: every position must be written
    padded = fm().flash_attn_mlm_compressed(qd, kd, vd, out_layout="padded", **kw)
    assert padded.shape == (B, H, N, D) and padded.dtype == dt
    assert torch.equal(padded, fm().unpack_from_kernel(packed, meta, H))
    with pytest.raises(ValueError, match="out_layout"):
        fm().flash_attn_mlm_compressed(qd, kd, vd, out_layout="bhnd", **kw)
    no_device_errors()


def test_padded_output_overwrites_stale_memory():
    """Rows past each sequence are written as zeros even when the allocator hands back dirty memory."""
    g = torch.Generator().manual_seed(81)
    B, H, N, D, dt = 3, 2, 200, 64, torch.float16
    lengths = torch.tensor([0, 200, 70], dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), dt, g).to(DEV) for _ in range(3))
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    for _ in range(3):
        junk = torch.full((B, H, N, D), float("nan"), dtype=dt, device=DEV)
        del junk
        out = fm().flash_attn_mlm_compressed(q, k, v, num_heads=H, q_meta=meta, scale=0.125, block_n=64,
                                             out_layout="padded")
        assert torch.isfinite(out.float()).all()
        assert bool((out[0] == 0).all()) and bool((out[2, :, 70:] == 0).all())
    no_device_errors()
