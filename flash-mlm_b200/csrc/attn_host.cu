// C-ABI entry points for the attention forward path: argument validation,
// TMA tensor-map encoding, the on-device tile scheduler and kernel dispatch.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "attn_fwd.cuh"
#include "common.h"

namespace fmlm {

std::string& last_error_slot() {
  static thread_local std::string s;
  return s;
}

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Encodes a 4-D tiled map {D, rows, heads, batch} over `v` with a box of
// {swizzle_bytes / 2, box_rows, 1, 1} and the matching shared-memory swizzle.
// Empty views get a 1-row map over `fallback` that the kernel never loads.
int encode_view(CUtensorMap* m, const fmlm_view4& v, int D, int box_rows, int dtype, const void* fallback,
                const char* name) {
  auto enc = encode_fn();
  if (!enc) return set_error(FMLM_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int swb = std::min(128, D * 2);
  const bool empty = v.data == nullptr || v.rows <= 0 || v.heads <= 0 || v.batch <= 0;
  const void* base = empty ? fallback : v.data;
  if (!aligned16(base)) return set_error(FMLM_ERR_INVALID, "%s: base address must be 16-byte aligned", name);
  cuuint64_t dims[4], strides[3];
  dims[0] = static_cast<cuuint64_t>(D);
  dims[1] = empty ? 1 : static_cast<cuuint64_t>(v.rows);
  dims[2] = empty ? 1 : static_cast<cuuint64_t>(v.heads);
  dims[3] = empty ? 1 : static_cast<cuuint64_t>(v.batch);
  const int64_t rs = empty ? D : v.row_stride;
  int64_t hs = empty ? D : v.head_stride;
  int64_t bs = empty ? D : v.batch_stride;
  if (!empty) {
    if (rs < D || (rs * 2) % 16 != 0) return set_error(FMLM_ERR_INVALID, "%s: row stride must be >= head_dim and a multiple of 8 elements", name);
    if (v.heads == 1 && (hs <= 0 || (hs * 2) % 16 != 0)) hs = rs * v.rows;
    if (v.batch == 1 && (bs <= 0 || (bs * 2) % 16 != 0)) bs = hs * v.heads;
    if ((hs * 2) % 16 != 0 || hs <= 0 || (bs * 2) % 16 != 0 || bs <= 0)
      return set_error(FMLM_ERR_INVALID, "%s: head/batch strides must be positive multiples of 8 elements", name);
  }
  strides[0] = static_cast<cuuint64_t>(rs) * 2;
  strides[1] = static_cast<cuuint64_t>(hs) * 2;
  strides[2] = static_cast<cuuint64_t>(bs) * 2;
  cuuint32_t box[4] = {static_cast<cuuint32_t>(swb / 2), static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapSwizzle sw = swb == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                            : CU_TENSOR_MAP_SWIZZLE_32B;
  const CUtensorMapDataType dt =
      dtype == FMLM_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(m, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FMLM_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", name, (int)r);
  return FMLM_OK;
}

// Builds the packed-mode work list: one entry per (sequence, query pair of
// PAIR rows), sequences ordered by decreasing key count (longest first) so
// the static round-robin over persistent CTAs balances.  Ties keep batch
// order.  Single CTA; sorting is skipped above kSortMax sequences.
constexpr int kSchedThreads = 1024;
constexpr int kSortMax = 2048;

__device__ __forceinline__ int seq_key_rows(const int* cu_q, const int* cu_kv, const int* ctx_index, int b,
                                            int ctx_bs, int has_ctx, int causal) {
  const int L = cu_q[b + 1] - cu_q[b];
  int kv = causal ? cu_q[b + 1] : L;
  if (has_ctx) {
    const int c = ctx_index ? ctx_index[b] : ctx_bs > 1 ? b : 0;
    if (c >= 0 && c < ctx_bs) kv += cu_kv[c + 1] - cu_kv[c];
  }
  return kv;
}

__device__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    if (lane < nw) warp_sums[lane] = s;  // inclusive
    if (lane == nw - 1) *total = s;
  }
  __syncthreads();
  const int before = warp > 0 ? warp_sums[warp - 1] : 0;
  const int r = before + x - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kSchedThreads) sched_kernel(const int* __restrict__ cu_q,
                                                              const int* __restrict__ cu_kv,
                                                              const int* __restrict__ ctx_index, int B, int ctx_bs,
                                                              int has_ctx, int causal, int pair, int* work,
                                                              int cap, int* err, int min_items) {
  __shared__ int key[kSortMax];
  __shared__ int order[kSortMax];
  __shared__ int warp_sums[32];
  __shared__ int total;
  __shared__ int running;
  const bool sort = B <= kSortMax;
  if (threadIdx.x == 0) running = 0;
  if (sort) {
    for (int b = threadIdx.x; b < B; b += blockDim.x) key[b] = seq_key_rows(cu_q, cu_kv, ctx_index, b, ctx_bs, has_ctx, causal);
    __syncthreads();
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
      const int kb = key[b];
      int r = 0;
      for (int b2 = 0; b2 < B; ++b2) {
        const int k2 = key[b2];
        r += (k2 > kb) || (k2 == kb && b2 < b);
      }
      order[r] = b;
    }
  }
  __syncthreads();
  for (int base = 0; base < B; base += blockDim.x) {
    const int s = base + threadIdx.x;
    const int b = s < B ? (sort ? order[s] : s) : -1;
    int n = b >= 0 ? (cu_q[b + 1] - cu_q[b] + pair - 1) / pair : 0;
    // A work entry keeps the item's index within its sequence in 16 bits:
    // a longer sequence is not scheduled and the call reports the error.
    if (n > 65536) {
      atomicExch(err, kErrSeqTooLong);
      n = 0;
    }
    if (b >= 0 && n < min_items) n = min_items;  // padded output: empty sequences still get their zero rows
    const int ex = block_exclusive_scan(n, warp_sums, &total);
    const int off = running;
    for (int i = 0; i < n; ++i) {
      const int idx = off + ex + i;
      if (idx < cap) work[kWorkHeader + idx] = (b << 16) | i;
    }
    __syncthreads();
    if (threadIdx.x == 0) running += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    work[0] = running < cap ? running : cap;
    work[1] = 0;  // item counter and finished-CTA count of the attention kernel
    work[2] = 0;
    work[3] = 0;
  }
}

int head_dim_supported(int d) { return d == 16 || d == 32 || d == 64 || d == 128 || d == 256 || d == 512; }
#ifndef FMLM_NQ_D64
#define FMLM_NQ_D64 1  // one tile per CTA, two CTAs per SM (measured faster than two tiles per CTA)
#endif
// Query tiles (of 128 rows) per work item for a head dimension.
int nq_for(int d) { return d >= 256 ? 1 : d == 64 ? FMLM_NQ_D64 : 2; }
int pair_rows(int d) { return 128 * nq_for(d); }

template <int D, int NQ, bool BF16>
int launch_attn(const CUtensorMap* m, const AttnParams& p, long long items, cudaStream_t s) {
  using C = AttnCfg<D, NQ>;
  auto kern = attn_fwd_kernel<D, NQ, BF16>;
  // Shared memory is padded so that exactly CTAS_PER_SM CTAs (TMEM owners)
  // fit on an SM: more would block in tcgen05.alloc.
#ifdef FMLM_ONE_CTA_PER_SM  // experiment: one resident CTA per SM whatever the layout
  const int smem = std::max(C::SMEM_BYTES, 150 * 1024);
#else
  const int smem = C::CTAS_PER_SM == 1 ? std::max(C::SMEM_BYTES, 116 * 1024) : std::max(C::SMEM_BYTES, 80 * 1024);
#endif
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return set_error(FMLM_ERR_CUDA, "device ordinal %d out of range", dev);
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return set_error(FMLM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return set_error(FMLM_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  // A persistent grid of CTAS_PER_SM CTAs per SM; items are handed out
  // dynamically, so CTAs that cannot be resident at once only start late.
  const int grid = (int)std::min<long long>(items, (long long)device_sm_count() * C::CTAS_PER_SM);
  kern<<<grid, C::THREADS, smem, s>>>(m[0], m[1], m[2], m[3], m[4], p);
  return check_launch("attn_fwd_kernel");
}

// single_tile (head_dim 128 only): one 128-row query tile per work item, for
// problems with fewer tile pairs than SMs (twice the items; P gets its own
// TMEM columns, so S(j+1) does not wait for PV(j)).
template <bool BF16>
int dispatch(int D, const CUtensorMap* m, const AttnParams& p, long long items, cudaStream_t s,
             bool single_tile = false) {
  switch (D) {
    case 16: return launch_attn<16, 2, BF16>(m, p, items, s);
    case 32: return launch_attn<32, 2, BF16>(m, p, items, s);
    case 64: return launch_attn<64, FMLM_NQ_D64, BF16>(m, p, items, s);
    case 128: return single_tile ? launch_attn<128, 1, BF16>(m, p, items, s) : launch_attn<128, 2, BF16>(m, p, items, s);
    case 256: return launch_attn<256, 1, BF16>(m, p, items, s);
    case 512: return launch_attn<512, 1, BF16>(m, p, items, s);
    default: return set_error(FMLM_ERR_UNSUPPORTED, "head_dim %d is not supported", D);
  }
}

// K/V tensor-map box height = the kernel's key block (AttnCfg::BN) for the
// instantiation dispatch() launches, so the two cannot disagree.
int kv_box_rows(int D) {
  switch (D) {
    case 16: return AttnCfg<16, 2>::BN;
    case 32: return AttnCfg<32, 2>::BN;
    case 64: return AttnCfg<64, FMLM_NQ_D64>::BN;
    case 128: return AttnCfg<128, 2>::BN;
    case 256: return AttnCfg<256, 1>::BN;
    default: return AttnCfg<512, 1>::BN;
  }
}
int o_halves(int D) { return D == 512 ? 2 : 1; }

constexpr unsigned long long kTimeoutNs = 2000000000ull;  // 2 s per wait

#ifdef FMLM_TRACE
unsigned long long* g_trace_buffer = nullptr;
#endif

int check_common(int dtype, int D, const void* out) {
  if (dtype != FMLM_DTYPE_F16 && dtype != FMLM_DTYPE_BF16) return set_error(FMLM_ERR_INVALID, "dtype must be f16 or bf16");
  if (!head_dim_supported(D))
    return set_error(FMLM_ERR_UNSUPPORTED, "HEAD_DIM must be one of {16, 32, 64, 128, 256} (512 with is_mla)");
  if (!out || !aligned16(out)) return set_error(FMLM_ERR_INVALID, "out must be a 16-byte aligned device pointer");
  return FMLM_OK;
}

}  // namespace
}  // namespace fmlm

using namespace fmlm;

extern "C" int fmlm_attn_dense_fwd(const fmlm_dense_args* a, void* stream) {
  if (!a) return set_error(FMLM_ERR_INVALID, "null args");
  int rc = check_common(a->dtype, a->head_dim, a->out);
  if (rc) return rc;
  const int D = a->head_dim;
  if (D == 512 && !a->is_mla) return set_error(FMLM_ERR_UNSUPPORTED, "HEAD_DIM 512 is supported for MLA only");
  if (a->batch <= 0 || a->num_heads <= 0 || a->seq_len < 0) return set_error(FMLM_ERR_INVALID, "bad B/H/N");
  if (a->seq_len == 0) return FMLM_OK;
  const bool has_ctx = !a->prefill && a->context_len > 0;
  if (has_ctx && a->context_batch_size > 1 && a->context_batch_size < a->batch)
    return set_error(FMLM_ERR_INVALID, "context_batch_size (%d) must be 1 or >= batch (%d)", a->context_batch_size, a->batch);
  CUtensorMap m[5];
  const int kb = kv_box_rows(D);
  if ((rc = encode_view(&m[0], a->q, D, 128, a->dtype, a->q.data, "q"))) return rc;
  if ((rc = encode_view(&m[1], a->k, D, kb, a->dtype, a->q.data, "k"))) return rc;
  if ((rc = encode_view(&m[2], a->is_mla ? a->k : a->v, D, kb, a->dtype, a->q.data, "v"))) return rc;
  fmlm_view4 empty = {nullptr, 0, 0, 0, 0, 0, 0};
  if ((rc = encode_view(&m[3], has_ctx ? a->k_cache : empty, D, kb, a->dtype, a->q.data, "k_cache"))) return rc;
  if ((rc = encode_view(&m[4], has_ctx ? (a->is_mla ? a->k_cache : a->v_cache) : empty, D, kb, a->dtype, a->q.data,
                        "v_cache")))
    return rc;
  AttnParams p{};
  p.mode = 0;
  p.has_ctx = has_ctx;
  p.is_mla = a->is_mla;
  p.B = a->batch; p.H = a->num_heads; p.N = a->seq_len;
  p.ctx_bs = a->context_batch_size;
  p.ctx_len = a->context_len;
  const int pr = pair_rows(D);
  const long long items = (long long)a->batch * a->num_heads * ((a->seq_len + pr - 1) / pr) * o_halves(D);
  if (items > 0x7fffffffLL) return set_error(FMLM_ERR_INVALID, "problem too large");
  p.num_items = (int)items;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.out = a->out;
  if (!a->error_word) return set_error(FMLM_ERR_INVALID, "error_word is required");
  p.err = a->error_word;
  p.q_ptr = reinterpret_cast<const uint16_t*>(a->q.data);
  p.q_sb = a->q.batch_stride;
  p.q_sh = a->q.head_stride;
  p.q_sr = a->q.row_stride;
  p.timeout_ns = kTimeoutNs;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return a->dtype == FMLM_DTYPE_BF16 ? dispatch<true>(D, m, p, items, s) : dispatch<false>(D, m, p, items, s);
}

// Packed launches at head_dim 128 use single-tile items when the problem has
// fewer tile pairs than the GPU has SMs.
#ifndef FMLM_SINGLE_TILE_FACTOR
#define FMLM_SINGLE_TILE_FACTOR 1
#endif
bool packed_single_tile(int D, int64_t total_q_len, int batch, int heads) {
  return D == 128 &&
         (total_q_len / pair_rows(D) + batch) * (int64_t)heads < (int64_t)FMLM_SINGLE_TILE_FACTOR * device_sm_count();
}

extern "C" size_t fmlm_packed_workspace_bytes(int32_t batch, int64_t total_q_len, int32_t head_dim) {
  // sized for the finer of the two item granularities head_dim 128 may use
  const int64_t pr = head_dim > 0 ? (head_dim == 128 ? 128 : pair_rows(head_dim)) : 128;
  const int64_t cap = total_q_len / pr + batch + 2;
  return (size_t)((cap + kWorkHeader) * sizeof(int32_t) + 15) / 16 * 16;
}

extern "C" int fmlm_attn_packed_fwd(const fmlm_packed_args* a, void* stream) {
  if (!a) return set_error(FMLM_ERR_INVALID, "null args");
  int rc = check_common(a->dtype, a->head_dim, a->out);
  if (rc) return rc;
  const int D = a->head_dim;
  if (D == 512 && !a->is_mla) return set_error(FMLM_ERR_UNSUPPORTED, "HEAD_DIM 512 is supported for MLA only");
  if (a->batch <= 0 || a->num_heads <= 0) return set_error(FMLM_ERR_INVALID, "bad batch / num_heads");
  if (a->batch >= 32768) return set_error(FMLM_ERR_INVALID, "batch must be < 32768");
  if (a->total_q_len < 0) return set_error(FMLM_ERR_INVALID, "total_q_len must be >= 0");
  if (a->total_q_len > 0x7fff0000LL) return set_error(FMLM_ERR_INVALID, "total_q_len must be < 2^31 - 2^16");
  // Work entries hold the 128-row tile index of a sequence in 16 bits.
  if (a->q_layout != FMLM_LAYOUT_PADDED && a->total_q_len / 128 > 65535)
    return set_error(FMLM_ERR_INVALID, "packed q: total_q_len must be below 65536 * 128 rows per head");
  if (!a->cu_seqlens_q) return set_error(FMLM_ERR_INVALID, "cu_seqlens_q is required");
  if (!a->error_word) return set_error(FMLM_ERR_INVALID, "error_word is required");
  const bool q_padded = a->q_layout == FMLM_LAYOUT_PADDED;
  const bool out_padded = a->out_padded != 0;
  const bool kv_padded = a->kv_layout == FMLM_LAYOUT_PADDED;
  if (kv_padded && a->causal_query_seq_attn)
    return set_error(FMLM_ERR_INVALID, "causal_query_seq_attn needs packed main k/v");
  if ((q_padded || kv_padded || out_padded) && a->seq_len <= 0)
    return set_error(FMLM_ERR_INVALID, "seq_len required for padded layouts");
  if ((int64_t)a->seq_len > 65535LL * pair_rows(D)) return set_error(FMLM_ERR_INVALID, "sequence too long");
  const bool has_ctx = !a->prefill && a->cu_seqlens_kv != nullptr && a->k_cache.data != nullptr &&
                       a->k_cache.rows > 0;
  const int32_t* ctx_index = has_ctx ? a->context_index : nullptr;
  if (has_ctx && !ctx_index && a->context_batch_size > 1 && a->context_batch_size < a->batch)
    return set_error(FMLM_ERR_INVALID, "context_batch_size (%d) must be 1 or >= batch (%d)", a->context_batch_size, a->batch);
  if (ctx_index && a->context_batch_size < 1) return set_error(FMLM_ERR_INVALID, "context_batch_size must be >= 1");
  const size_t need = fmlm_packed_workspace_bytes(a->batch, a->total_q_len, D);
  if (!a->workspace || a->workspace_bytes < need || !aligned16(a->workspace))
    return set_error(FMLM_ERR_INVALID, "workspace too small (%zu bytes needed)", need);

  CUtensorMap m[5];
  const int kb = kv_box_rows(D);
  if ((rc = encode_view(&m[0], a->q, D, 128, a->dtype, a->q.data, "q"))) return rc;
  if ((rc = encode_view(&m[1], a->k, D, kb, a->dtype, a->q.data, "k"))) return rc;
  if ((rc = encode_view(&m[2], a->is_mla ? a->k : a->v, D, kb, a->dtype, a->q.data, "v"))) return rc;
  fmlm_view4 empty = {nullptr, 0, 0, 0, 0, 0, 0};
  if ((rc = encode_view(&m[3], has_ctx ? a->k_cache : empty, D, kb, a->dtype, a->q.data, "k_cache"))) return rc;
  if ((rc = encode_view(&m[4], has_ctx ? (a->is_mla ? a->k_cache : a->v_cache) : empty, D, kb, a->dtype, a->q.data,
                        "v_cache")))
    return rc;

  const bool single = packed_single_tile(D, a->total_q_len, a->batch, a->num_heads);
  const int pr = single ? 128 : pair_rows(D);
  const int64_t cap = a->total_q_len / pr + a->batch + 2;
  int* work = reinterpret_cast<int*>(a->workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!a->reuse_schedule) {
    sched_kernel<<<1, kSchedThreads, 0, s>>>(a->cu_seqlens_q, has_ctx ? a->cu_seqlens_kv : a->cu_seqlens_q,
                                             ctx_index, a->batch, a->context_batch_size, has_ctx, a->causal_query_seq_attn, pr,
                                             work, (int)cap, a->error_word, out_padded ? 1 : 0);
    if ((rc = check_launch("sched_kernel"))) return rc;
  }

  AttnParams p{};
  p.mode = 1;
  p.q_padded = q_padded;
  p.main_padded = kv_padded;
  p.causal = a->causal_query_seq_attn;
  p.has_ctx = has_ctx;
  p.is_mla = a->is_mla;
  p.B = a->batch; p.H = a->num_heads; p.N = a->seq_len;
  p.ctx_bs = a->context_batch_size;
  p.t_out = a->out_rows_per_head;
  p.out_padded = out_padded;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  p.cu_q = a->cu_seqlens_q;
  p.cu_kv = has_ctx ? a->cu_seqlens_kv : a->cu_seqlens_q;
  p.ctx_index = ctx_index;
  p.work = work;
  p.out = a->out;
  p.err = a->error_word;
  p.q_ptr = reinterpret_cast<const uint16_t*>(a->q.data);
  p.q_sb = a->q.batch_stride;
  p.q_sh = a->q.head_stride;
  p.q_sr = a->q.row_stride;
  p.timeout_ns = kTimeoutNs;
#ifdef FMLM_TRACE
  p.trace = g_trace_buffer;
#endif
  const long long items_bound = cap * (long long)a->num_heads * o_halves(D);
  return a->dtype == FMLM_DTYPE_BF16 ? dispatch<true>(D, m, p, items_bound, s, single)
                                     : dispatch<false>(D, m, p, items_bound, s, single);
}

#ifdef FMLM_TRACE
// Debug builds only: device buffer receiving the timeline of CTA 0.
extern "C" FMLM_API void fmlm_debug_set_trace(unsigned long long* buf) { fmlm::g_trace_buffer = buf; }
#endif

// ---------------------------------------------------------------------------
// Allocation-free variant of fmlm_attn_packed_fwd.
//
// Some callers cannot call cudaMalloc at all: code running inside a CUDA
// graph being captured, real-time or embedded hosts whose allocator is locked
// after start-up, and plugin hosts that hand a library only pre-allocated
// tensors.  For them the tile schedule lives in a fixed array in device
// memory that every GPU loading this library holds until the process exits
// (kNoAllocScheduleInts int32 = 256 KB).  The first call in a device's
// context looks the array's address up with cudaGetSymbolAddress (make that
// first call before any stream capture); later calls in that context reuse it.  Every call shares the array and
// the schedule kernel rewrites it completely on each call (nothing needs to
// start at zero), so calls that overlap on the GPU (different streams,
// different threads on one device) race and must be serialised by the caller.
namespace fmlm {
namespace {
constexpr int kNoAllocScheduleInts = 65536;
static __device__ __align__(256) int g_noalloc_schedule[kNoAllocScheduleInts];
std::mutex g_noalloc_mu;
// The array's device address belongs to the CUDA context that looked it up,
// so the cache is keyed by (device, context): a new primary context after
// cudaDeviceReset, or another context made current on the same device, looks
// the address up again.
struct NoAllocSlot {
  CUcontext ctx;
  void* ptr;
};
NoAllocSlot g_noalloc_slot[64] = {};

PFN_cuCtxGetCurrent_v4000 ctx_current_fn() {
  static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
  });
  return fn;
}

int noalloc_schedule_ptr(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(FMLM_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(FMLM_ERR_INVALID, "device index %d out of range", dev);
  auto get_ctx = ctx_current_fn();
  if (!get_ctx) return set_error(FMLM_ERR_CUDA, "cuCtxGetCurrent is unavailable");
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) return set_error(FMLM_ERR_CUDA, "cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  NoAllocSlot& slot = g_noalloc_slot[dev];
  if (ctx == nullptr || slot.ptr == nullptr || slot.ctx != ctx) {
    // The lookup also makes the device's primary context current when no
    // context is yet, so the context is read again after it.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_schedule);
    if (e != cudaSuccess || p == nullptr)
      return set_error(FMLM_ERR_CUDA, "cudaGetSymbolAddress(schedule scratch): %s", cudaGetErrorString(e));
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr)
      return set_error(FMLM_ERR_CUDA, "no current CUDA context on device %d", dev);
    slot.ctx = ctx;
    slot.ptr = p;
  }
  *out = slot.ptr;
  return FMLM_OK;
}
}  // namespace
}  // namespace fmlm

extern "C" int fmlm_attn_packed_fwd_noalloc(const fmlm_packed_args* a, void* stream) {
  if (!a) return set_error(FMLM_ERR_INVALID, "null args");
  if (a->batch <= 0 || a->total_q_len < 0)
    return set_error(FMLM_ERR_INVALID, "batch must be > 0 and total_q_len >= 0");
  const size_t have = sizeof(int) * (size_t)kNoAllocScheduleInts;
  const size_t need = fmlm_packed_workspace_bytes(a->batch, a->total_q_len, a->head_dim);
  if (need > have)
    return set_error(FMLM_ERR_INVALID,
                     "fmlm_attn_packed_fwd_noalloc: this problem needs a %zu-byte tile schedule but the built-in "
                     "scratch holds %zu bytes (batch + total_q_len / 128 must stay below about 65500); "
                     "use fmlm_attn_packed_fwd with a caller workspace",
                     need, have);
  void* ws = nullptr;
  int rc = noalloc_schedule_ptr(&ws);
  if (rc) return rc;
  fmlm_packed_args b = *a;
  b.workspace = ws;
  b.workspace_bytes = have;
  b.reuse_schedule = 0;
  return fmlm_attn_packed_fwd(&b, stream);
}

extern "C" const char* fmlm_last_error(void) { return last_error_slot().c_str(); }

namespace fmlm {
// One warp waits on a barrier whose phase never completes; the bounded wait
// must return false, and the kernel reports it like the attention kernel does.
__global__ void bounded_wait_probe_kernel(int* err, unsigned long long limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0, &abort_flag, limit_ns);
  if (!ok && threadIdx.x == 0) atomicExch(err, kErrTimeout);
}
}  // namespace fmlm

extern "C" int fmlm_selftest_bounded_wait(int32_t* error_word, uint64_t limit_ns, void* stream) {
  if (!error_word) return set_error(FMLM_ERR_INVALID, "error_word is required");
  if (limit_ns == 0 || limit_ns > 100000000ull) return set_error(FMLM_ERR_INVALID, "limit_ns must be in (0, 0.1 s]");
  fmlm::bounded_wait_probe_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(error_word, limit_ns);
  return check_launch("bounded_wait_probe_kernel");
}

extern "C" int fmlm_version(void) { return 100; }
