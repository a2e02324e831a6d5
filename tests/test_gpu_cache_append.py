"""GPU tests of the context-cache append kernel (fmlm_cache_append) and of
cache-layout unification (no reference counterpart: the reference stores a
new packed buffer per prefill, src/flash_mlm/host/host.py:327-364, and its
dense prefill layout, host.py:206-223, cannot serve its packed path).

Bars: cache rows and offsets bit-exact against the oracle's restatement;
attention through an appended / converted cache within the north-star bound
(max abs error 2e-3 f16, 8e-3 bf16) against the fp32 oracle.
"""

import ctypes

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float16: 2e-3, torch.bfloat16: 8e-3}


def fm():
    import flash_mlm

    return flash_mlm


def _rand(shape, dtype, g):
    return torch.randn(shape, generator=g).to(dtype)


def _assert_raw(got, ref, dtype, what):
    g = got.detach().float().cpu()
    err = (g - torch.as_tensor(ref, dtype=torch.float32)).abs().max().item() if g.numel() else 0.0
    assert err <= TOL[dtype], f"{what}: max abs err {err:.3e} > {TOL[dtype]:.0e}"


@pytest.mark.parametrize("is_mla", [False, True])
def test_append_twice_bit_exact_and_offsets_on_device(is_mla):
    g = torch.Generator().manual_seed(31 + is_mla)
    H, D, dt = (1 if is_mla else 3), 64, torch.float16
    cache = fm().InferenceCache()
    cap = 900
    cache.reserve_kv_cache(4, capacity=cap, max_entries=8, is_mla=is_mla, num_heads=H, head_dim=D, dtype=dt,
                           device=torch.device(DEV))
    host_cache_k = np.zeros((H * cap, D), np.float32)
    host_cache_v = np.zeros((H * cap, D), np.float32)
    cu_kv = [0]
    for lengths, N in (([130, 0, 77], 130), ([5, 300, 64, 1], 300)):
        k = _rand((len(lengths), H, N, D), dt, g)
        v = _rand((len(lengths), H, N, D), dt, g)
        meta = fm().build_pack_metadata(torch.tensor(lengths, dtype=torch.int32, device=DEV), N, 64)
        entry = cache.append_kv_cache(4, k.to(DEV), None if is_mla else v.to(DEV), meta)
        cu_src = meta.cu_seqlens.cpu().tolist()
        new_k, new_cu = oracle.cache_append(host_cache_k, cu_kv, k.float().numpy(), cu_src)
        if not is_mla:
            host_cache_v, _ = oracle.cache_append(host_cache_v, cu_kv, v.float().numpy(), cu_src)
        host_cache_k, cu_kv = new_k, new_cu
        torch.cuda.synchronize()
        fm().check_device_errors(torch.device(DEV, torch.cuda.current_device()))
        assert entry.cu_seqlens_kv.cpu().tolist() == cu_kv
        assert entry.cu_host == cu_kv and entry.context_batch_size == len(cu_kv) - 1
        used = cu_kv[-1]
        got_k = entry.k_cache.float().cpu().numpy().reshape(H, cap, D)[:, :used]
        assert np.array_equal(got_k, host_cache_k.reshape(H, cap, D)[:, :used])
        if not is_mla:
            got_v = entry.v_cache.float().cpu().numpy().reshape(H, cap, D)[:, :used]
            assert np.array_equal(got_v, host_cache_v.reshape(H, cap, D)[:, :used])

    # a query call over the appended cache (7 entries) sees entry b's rows
    B, N = 7, 90
    lengths = torch.tensor([90, 3, 0, 41, 90, 17, 60], dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), dt, g) for _ in range(3))
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=0.125,
                                         inference_cache=cache, layer_id=4, is_mla=is_mla, block_n=64)
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), 0.125, k_cache=host_cache_k,
                                  v_cache=host_cache_k if is_mla else host_cache_v, cu_kv=np.array(cu_kv),
                                  context_batch_size=B, total_context_len=cap, is_mla=is_mla)
    _assert_raw(out, ref, dt, "query over appended cache")


def test_prefill_into_reserved_cache_matches_unreserved_prefill():
    """prefill=True into a reserved cache: same outputs as the reference-style
    prefill (new packed buffer), the rows land in the reserved memory, and a
    later query call gives the same result from either cache."""
    g = torch.Generator().manual_seed(77)
    B, H, N, D, dt = 3, 2, 200, 128, torch.bfloat16
    lengths = torch.tensor([200, 9, 133], dtype=torch.int32, device=DEV)
    meta = fm().build_pack_metadata(lengths, N, 64)
    pq, pk, pv, q, k, v = (_rand((B, H, N, D), dt, g).to(DEV) for _ in range(6))
    plain, reserved = fm().InferenceCache(), fm().InferenceCache()
    reserved.reserve_kv_cache(0, capacity=400, max_entries=4, is_mla=False, num_heads=H, head_dim=D, dtype=dt,
                              device=torch.device(DEV))
    outs = []
    for c in (plain, reserved):
        o1 = fm().flash_attn_mlm_compressed(pq, pk, pv, num_heads=H, q_meta=meta, scale=D ** -0.5,
                                            inference_cache=c, layer_id=0, block_n=64, prefill=True)
        o2 = fm().flash_attn_mlm_compressed(q, k, v, num_heads=H, q_meta=meta, scale=D ** -0.5,
                                            inference_cache=c, layer_id=0, block_n=64)
        outs.append((o1, o2))
    e = reserved.get_kv_cache(0, is_mla=False, num_heads=H, head_dim=D, dtype=dt, device=q.device)
    assert e.k_cache.data_ptr() == reserved.reserved(0).k.data_ptr() and e.used_context_len == 342
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
    # a second prefill replaces the entry (the reserved cache is emptied first)
    fm().flash_attn_mlm_compressed(pq, pk, pv, num_heads=H, q_meta=meta, scale=D ** -0.5, inference_cache=reserved,
                                   layer_id=0, block_n=64, prefill=True)
    e2 = reserved.get_kv_cache(0, is_mla=False, num_heads=H, head_dim=D, dtype=dt, device=q.device)
    assert e2.context_batch_size == B and e2.cu_seqlens_kv.cpu().tolist() == meta.cu_seqlens.cpu().tolist()
    fm().check_device_errors(torch.device(DEV, torch.cuda.current_device()))


@pytest.mark.parametrize("shared", [False, True])
def test_dense_prefill_serves_packed_query(shared):
    """A dense prefill stores [C][H][ctx]; a packed query reads it through a head-major copy."""
    g = torch.Generator().manual_seed(5 + shared)
    B, H, N, D, dt = 3, 4, 96, 64, torch.float16
    pq, pk, pv = (_rand((B, H, N, D), dt, g).to(DEV) for _ in range(3))
    cache = fm().InferenceCache()
    fm().flash_attn_mlm(pq, pk, pv, scale=0.125, inference_cache=cache, layer_id=2, prefill=True)
    lengths = torch.tensor([50, 96, 7], dtype=torch.int32)
    q, k, v = (_rand((B, H, N, D), dt, g) for _ in range(3))
    meta = fm().build_pack_metadata(lengths.to(DEV), N, 64)
    out = fm().flash_attn_mlm_compressed(q.to(DEV), k.to(DEV), v.to(DEV), num_heads=H, q_meta=meta, scale=0.125,
                                         inference_cache=cache, layer_id=2, block_n=64,
                                         context_batch_size=1 if shared else None)
    # oracle: the same context in head-major order ([H][C * N], entry c at rows c * N)
    kc = pk.float().cpu().numpy().transpose(1, 0, 2, 3).reshape(H * B * N, D)
    vc = pv.float().cpu().numpy().transpose(1, 0, 2, 3).reshape(H * B * N, D)
    cu_kv = np.array([0, B * N]) if shared else np.arange(B + 1) * N
    ref = oracle.attention_packed(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                  meta.cu_seqlens.cpu().numpy(), 0.125, k_cache=kc, v_cache=vc, cu_kv=cu_kv,
                                  context_batch_size=1 if shared else B, total_context_len=B * N)
    _assert_raw(out, ref, dt, "packed query over dense prefill")
    e = cache.get_kv_cache(2, is_mla=False, num_heads=H, head_dim=D, dtype=dt, device=pq.device)
    assert e.layout == "batch_major" and e.converted is not None
    assert np.array_equal(e.converted.k_cache.float().cpu().numpy(), kc)
    fm().check_device_errors(torch.device(DEV, torch.cuda.current_device()))


def test_packed_prefill_serves_dense_query():
    """A head-major cache of equal-length entries serves the dense path in place."""
    g = torch.Generator().manual_seed(11)
    B, H, N, D, dt = 2, 3, 64, 64, torch.bfloat16
    pq, pk, pv = (_rand((B, H, N, D), dt, g).to(DEV) for _ in range(3))
    cache = fm().InferenceCache()
    cache.reserve_kv_cache(1, capacity=200, max_entries=2, is_mla=False, num_heads=H, head_dim=D, dtype=dt,
                           device=torch.device(DEV))
    meta = fm().build_pack_metadata(torch.tensor([N, N], dtype=torch.int32, device=DEV), N, 64)
    fm().flash_attn_mlm_compressed(pq, pk, pv, num_heads=H, q_meta=meta, scale=0.125, inference_cache=cache,
                                   layer_id=1, block_n=64, prefill=True)
    q, k, v = (_rand((B, H, 40, D), dt, g) for _ in range(3))
    out = fm().flash_attn_mlm(q.to(DEV), k.to(DEV), v.to(DEV), scale=0.125, inference_cache=cache, layer_id=1)
    # oracle: dense context of batch b = prefill batch b's rows ([C][H][ctx] order)
    kc = pk.float().cpu().numpy().reshape(B * H * N, D)
    vc = pv.float().cpu().numpy().reshape(B * H * N, D)
    ref = oracle.attention_dense(q.float().numpy(), k.float().numpy(), v.float().numpy(), 0.125, k_cache=kc,
                                 v_cache=vc, context_len=N, context_batch_size=B)
    _assert_raw(out, ref, dt, "dense query over packed prefill")
    fm().check_device_errors(torch.device(DEV, torch.cuda.current_device()))


def test_c_abi_append_past_capacity_writes_nothing():
    from flash_mlm import _lib

    dev = torch.device(DEV, torch.cuda.current_device())
    H, D, cap = 2, 64, 16
    kc = torch.full((H * cap, D), 7.0, dtype=torch.float16, device=dev)
    cu_kv = torch.tensor([0, 10, 0, 0], dtype=torch.int32, device=dev)
    x = torch.ones((1, H, 8, D), dtype=torch.float16, device=dev)
    cu = torch.tensor([0, 8], dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    view = _lib.view_bhnd(x)
    rc = _lib.lib().fmlm_cache_append(ctypes.byref(view), None, _lib.FMLM_LAYOUT_PADDED, 2, D, cu.data_ptr(), 1, 8,
                                      kc.data_ptr(), None, cap, cu_kv.data_ptr(), 1, err.data_ptr(),
                                      _lib.stream_ptr(dev))
    assert rc == 0
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 5
    assert bool((kc == 7).all()) and cu_kv.cpu().tolist() == [0, 10, 0, 0]
    # a fitting append from a packed source lands after the held rows
    packed = torch.arange(H * 4 * D, dtype=torch.float32, device=dev).to(torch.float16).view(H * 4, D)
    pv = _lib.view_packed(packed, H)
    cu2 = torch.tensor([0, 1, 4], dtype=torch.int32, device=dev)
    err.zero_()
    rc = _lib.lib().fmlm_cache_append(ctypes.byref(pv), None, _lib.FMLM_LAYOUT_PACKED, 2, D, cu2.data_ptr(), 2, 4,
                                      kc.data_ptr(), None, cap, cu_kv.data_ptr(), 1, err.data_ptr(),
                                      _lib.stream_ptr(dev))
    assert rc == 0
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0 and cu_kv.cpu().tolist() == [0, 10, 11, 14]
    got = kc.view(H, cap, D)[:, 10:14].cpu()
    assert torch.equal(got, packed.view(H, 4, D).cpu())
    assert bool((kc.view(H, cap, D)[:, 14:] == 7).all())
