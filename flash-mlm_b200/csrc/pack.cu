// Pack metadata, pack (gather + pad), unpack (scatter + zero) and pad kernels.
//
// These restate the torch index arithmetic of the reference host utilities
// (src/flash_mlm/host/host_utils.py) as single-pass vectorised CUDA kernels:
//   build_pack_metadata / _build_query_tile_map_from_cu_seqlens  :27-107
//   pack_for_kernel / _pack_flatten_for_kernel_into              :266-289, :397-420
//   pad_packed_main_tensors_for_mlm_compressed                   :494-584
//   unpack_from_kernel                                           :587-615
// Copies move the widest naturally aligned unit (16/8/4/2/1 bytes) that the
// row size, pointers and strides allow, so every access is coalesced.
#include <algorithm>

#include "common.h"

namespace fmlm {
namespace {

// Device error word value of an append that would pass the cache capacity
// (numbered after the attention kernel's codes 1-4).
constexpr int kErrCacheFull = 5;

constexpr int kScanThreads = 1024;

__device__ int block_scan_excl(int v, int* warp_sums, int* total) {
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
    if (lane < nw) warp_sums[lane] = s;
    if (lane == nw - 1) *total = s;
  }
  __syncthreads();
  const int r = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  __syncthreads();
  return r;
}

// counters: [0] total tokens, [1] total tiles, [2] error, [3 .. 3+B] tile prefix.
__global__ void __launch_bounds__(kScanThreads) meta_scan_kernel(const int* __restrict__ lengths, int B, int N,
                                                                 int block_n, int* __restrict__ cu,
                                                                 int* __restrict__ counters) {
  __shared__ int ws[32];
  __shared__ int tot_l, tot_t, run_l, run_t;
  if (threadIdx.x == 0) { run_l = 0; run_t = 0; cu[0] = 0; }
  int bad = 0;
  for (int base = 0; base < B; base += blockDim.x) {
    const int b = base + threadIdx.x;
    const int L = b < B ? lengths[b] : 0;
    if (b < B && (L < 0 || L > N)) bad = 1;
    const int Lc = (L < 0) ? 0 : L;
    const int tiles = (Lc + block_n - 1) / block_n;
    __syncthreads();
    const int rl = run_l, rt = run_t;
    const int el = block_scan_excl(L, ws, &tot_l);
    const int et = block_scan_excl(tiles, ws, &tot_t);
    if (b < B) {
      cu[b + 1] = rl + el + L;
      counters[3 + b] = rt + et;
    }
    __syncthreads();
    if (threadIdx.x == 0) { run_l += tot_l; run_t += tot_t; }
  }
  bad = __syncthreads_or(bad);
  if (threadIdx.x == 0) {
    counters[0] = run_l;
    counters[1] = run_t;
    counters[2] = bad;
    counters[3 + B] = run_t;
  }
}

// One CTA per sequence: token indices b*N+t of its valid tokens and its query tiles.
__global__ void meta_fill_kernel(const int* __restrict__ cu, const int* __restrict__ counters, int N, int block_n,
                                 long long* __restrict__ token_indices, int* __restrict__ batch_ids,
                                 int* __restrict__ tile_starts) {
  const int b = blockIdx.x;
  if (counters[2]) return;
  const int s = cu[b], L = cu[b + 1] - s;
  const int base = b * N;  // int32 product, as the reference builds it
  if (token_indices)
    for (int t = threadIdx.x; t < L; t += blockDim.x) token_indices[s + t] = (long long)(base + t);
  const int tp = counters[3 + b];
  const int nt = (L + block_n - 1) / block_n;
  for (int i = threadIdx.x; i < nt; i += blockDim.x) {
    batch_ids[tp + i] = b;
    tile_starts[tp + i] = s + i * block_n;
  }
}

template <int V>
struct VecT;
template <> struct VecT<16> { using T = uint4; };
template <> struct VecT<8> { using T = uint2; };
template <> struct VecT<4> { using T = uint32_t; };
template <> struct VecT<2> { using T = uint16_t; };
template <> struct VecT<1> { using T = uint8_t; };

// Row copies are organised per (row chunk, head, sequence): grid
// (ceil(rows / kRowsPerCta), H, B [+1]), so a CTA copies up to kRowsPerCta
// consecutive rows of one sequence and head with no per-element search or
// 64-bit division, and each thread issues kUnroll loads before its stores.
constexpr int kRowsPerCta = 64;
constexpr int kCopyThreads = 256;
constexpr int kUnroll = 4;

// out[h][r] = x[b(r)][h][r - cu[b(r)]] for r < total_tokens, zero for r < total_padded.
// Sequence slice b = B of the grid writes the zero rows [total_tokens, total_padded).
template <int V>
__global__ void __launch_bounds__(kCopyThreads) pack_rows_kernel(const uint8_t* __restrict__ x, long long sb,
                                                                 long long sh, long long sr, int row_bytes,
                                                                 const int* __restrict__ cu, int B,
                                                                 long long total_tokens, long long total_padded,
                                                                 uint8_t* __restrict__ out) {
  using T = typename VecT<V>::T;
  const int nvec = row_bytes / V;
  const int h = blockIdx.y;
  const long long r0 = (long long)blockIdx.x * kRowsPerCta;
  for (int b = blockIdx.z; b <= B; b += gridDim.z) {
    long long len, dst0;
    const uint8_t* src = nullptr;
    if (b < B) {
      const int s0 = __ldg(cu + b);
      len = __ldg(cu + b + 1) - s0;
      dst0 = (long long)h * total_padded + s0;
      src = x + b * sb + h * sh;
    } else {
      len = total_padded - total_tokens;
      dst0 = (long long)h * total_padded + total_tokens;
    }
    if (r0 >= len) continue;
    const int nv = (int)(len - r0 < kRowsPerCta ? len - r0 : kRowsPerCta) * nvec;
    for (int base = 0; base < nv; base += kCopyThreads * kUnroll) {
      T val[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = base + u * kCopyThreads + threadIdx.x;
        val[u] = T{};
        if (i < nv && src) {
          const int t = i / nvec, v = i - t * nvec;
          val[u] = *reinterpret_cast<const T*>(src + (r0 + t) * sr + (long long)v * V);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = base + u * kCopyThreads + threadIdx.x;
        if (i < nv) {
          const int t = i / nvec, v = i - t * nvec;
          *reinterpret_cast<T*>(out + (dst0 + r0 + t) * row_bytes + (long long)v * V) = val[u];
        }
      }
    }
  }
}

// out[b][h][n] = packed[h][cu[b] + n] for n < len(b), zero otherwise.
template <int V>
__global__ void __launch_bounds__(kCopyThreads) unpack_rows_kernel(const uint8_t* __restrict__ packed,
                                                                   long long total_tokens, int H, int row_bytes,
                                                                   const int* __restrict__ cu, int B, int N,
                                                                   uint8_t* __restrict__ out) {
  using T = typename VecT<V>::T;
  const int nvec = row_bytes / V;
  const int h = blockIdx.y;
  const int r0 = blockIdx.x * kRowsPerCta;
  const int nv = min(kRowsPerCta, N - r0) * nvec;
  for (int b = blockIdx.z; b < B; b += gridDim.z) {
    const int s0 = __ldg(cu + b);
    const int len = __ldg(cu + b + 1) - s0;
    const uint8_t* src = packed + ((long long)h * total_tokens + s0) * row_bytes;
    uint8_t* dst = out + (((long long)b * H + h) * N + r0) * row_bytes;
    for (int base = 0; base < nv; base += kCopyThreads * kUnroll) {
      T val[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = base + u * kCopyThreads + threadIdx.x;
        val[u] = T{};
        const int t = i / nvec;
        if (i < nv && r0 + t < len) val[u] = *reinterpret_cast<const T*>(src + (long long)(r0 + t) * row_bytes + (long long)(i - t * nvec) * V);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = base + u * kCopyThreads + threadIdx.x;
        if (i < nv) *reinterpret_cast<T*>(dst + (long long)i * V) = val[u];
      }
    }
  }
}

// dst[h][r] = src[h][r] for r < old_len, zero for r < new_len.
template <int V>
__global__ void pad_rows_kernel(const uint8_t* __restrict__ src, long long old_len, long long new_len, int heads,
                                int row_bytes, uint8_t* __restrict__ dst) {
  using T = typename VecT<V>::T;
  const int nvec = row_bytes / V;
  const long long n = (long long)heads * new_len * nvec;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / nvec;
    const int v = (int)(i - row * nvec);
    const long long h = row / new_len;
    const long long r = row - h * new_len;
    T val{};
    if (r < old_len) val = *reinterpret_cast<const T*>(src + (h * old_len + r) * row_bytes + (long long)v * V);
    *reinterpret_cast<T*>(dst + row * row_bytes + (long long)v * V) = val;
  }
}

// Appends B sequences to a head-major context cache dst[h][cap] with spare
// room.  base = cu_kv[eb] (the rows the cache already holds, read on the
// device); sequence b lands at rows base + cu[b] - cu[0] ... of every head and
// its end offset is written to cu_kv[eb + 1 + b].  Source rows come from a
// padded [B][H][N] view (row t of batch b) or a packed [H][T] view (row
// cu[b] + t of batch 0).  grid.y covers the K heads then the V heads.  If the
// appended rows would pass `cap`, nothing is written and the error word is set.
template <int V>
__global__ void __launch_bounds__(kCopyThreads) cache_append_kernel(
    const uint8_t* __restrict__ src_k, const uint8_t* __restrict__ src_v, long long sb, long long sh, long long sr,
    int src_packed, int row_bytes, const int* __restrict__ cu, int B, int H, long long total_new,
    uint8_t* __restrict__ dst_k, uint8_t* __restrict__ dst_v, long long cap, int* cu_kv, int eb, int* err) {
  using T = typename VecT<V>::T;
  const int nvec = row_bytes / V;
  const bool is_v = blockIdx.y >= (unsigned)H;
  const int h = is_v ? blockIdx.y - H : blockIdx.y;
  const uint8_t* src_base = is_v ? src_v : src_k;
  uint8_t* dst = is_v ? dst_v : dst_k;
  const long long base = cu_kv[eb];
  if (base < 0 || base + total_new > cap) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && threadIdx.x == 0) atomicExch(err, kErrCacheFull);
    return;
  }
  const int c0 = __ldg(cu);
  const long long r0 = (long long)blockIdx.x * kRowsPerCta;
  for (int b = blockIdx.z; b < B; b += gridDim.z) {
    const int s0 = __ldg(cu + b);
    const long long len = __ldg(cu + b + 1) - s0;
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0)
      cu_kv[eb + 1 + b] = (int)(base + (s0 - c0) + len);
    if (r0 >= len) continue;
    const uint8_t* src = src_packed ? src_base + h * sh + (long long)s0 * sr : src_base + b * sb + h * sh;
    const long long dst0 = (long long)h * cap + base + (s0 - c0);
    const int nv = (int)(len - r0 < kRowsPerCta ? len - r0 : kRowsPerCta) * nvec;
    for (int i0 = 0; i0 < nv; i0 += kCopyThreads * kUnroll) {
      T val[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kCopyThreads + threadIdx.x;
        val[u] = T{};
        if (i < nv) {
          const int t = i / nvec, w = i - t * nvec;
          val[u] = *reinterpret_cast<const T*>(src + (r0 + t) * sr + (long long)w * V);
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = i0 + u * kCopyThreads + threadIdx.x;
        if (i < nv) {
          const int t = i / nvec, w = i - t * nvec;
          *reinterpret_cast<T*>(dst + (dst0 + r0 + t) * row_bytes + (long long)w * V) = val[u];
        }
      }
    }
  }
}

int pick_vec(long long a) {
  for (int v = 16; v > 1; v >>= 1)
    if (a % v == 0) return v;
  return 1;
}

int grid_for(long long n) {
  const long long blocks = (n + 255) / 256;
  return (int)std::max<long long>(1, std::min<long long>(blocks, (long long)device_sm_count() * 16));
}

}  // namespace
}  // namespace fmlm

using namespace fmlm;

extern "C" int fmlm_build_pack_metadata(const int32_t* lengths, int32_t B, int32_t N, int32_t block_n,
                                        int32_t* cu_seqlens, int64_t* token_indices, int32_t* batch_ids_q,
                                        int32_t* q_tile_starts_q, int32_t* counters, void* stream) {
  if (B < 0 || N < 0) return set_error(FMLM_ERR_INVALID, "N must be >= 0");
  if (block_n < 1) return set_error(FMLM_ERR_INVALID, "block_n must be >= 1");
  if (!cu_seqlens || !counters || (B > 0 && (!lengths || !batch_ids_q || !q_tile_starts_q)))
    return set_error(FMLM_ERR_INVALID, "null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  meta_scan_kernel<<<1, kScanThreads, 0, s>>>(lengths, B, N, block_n, cu_seqlens, counters);
  int rc = check_launch("meta_scan_kernel");
  if (rc || B == 0) return rc;
  meta_fill_kernel<<<B, 256, 0, s>>>(cu_seqlens, counters, N, block_n, reinterpret_cast<long long*>(token_indices),
                                     batch_ids_q, q_tile_starts_q);
  return check_launch("meta_fill_kernel");
}

extern "C" int fmlm_pack_rows(const fmlm_view4* x, int32_t elem_bytes, int32_t head_dim, const int32_t* cu_seqlens,
                              int32_t B, int64_t total_tokens, int64_t total_padded, void* out, void* stream) {
  if (!x || !out || !cu_seqlens) return set_error(FMLM_ERR_INVALID, "null pointer argument");
  if (elem_bytes <= 0 || head_dim <= 0 || B <= 0 || total_tokens < 0 || total_padded < total_tokens)
    return set_error(FMLM_ERR_INVALID, "bad pack sizes");
  const int H = (int)x->heads;
  const long long row_bytes = (long long)elem_bytes * head_dim;
  const long long n_rows = (long long)H * total_padded;
  if (n_rows == 0) return FMLM_OK;
  if (total_tokens > 0 && !x->data) return set_error(FMLM_ERR_INVALID, "x has no data");
  const long long sb = x->batch_stride * elem_bytes, sh = x->head_stride * elem_bytes, sr = x->row_stride * elem_bytes;
  long long g = row_bytes;
  for (long long a : {sb, sh, sr, (long long)reinterpret_cast<uintptr_t>(x->data),
                      (long long)reinterpret_cast<uintptr_t>(out)})
    g = std::__gcd(g, a == 0 ? g : a);
  const int V = pick_vec(g);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto px = reinterpret_cast<const uint8_t*>(x->data);
  auto po = reinterpret_cast<uint8_t*>(out);
  const long long max_rows = std::max<long long>(x->rows, total_padded - total_tokens);
  const dim3 pgrid((unsigned)((max_rows + kRowsPerCta - 1) / kRowsPerCta), (unsigned)H,
                   (unsigned)std::min<long long>((long long)B + 1, 65535));
  if (H > 65535 || pgrid.x == 0) return set_error(FMLM_ERR_INVALID, "bad pack sizes");
#define FMLM_PACK(VV) \
  pack_rows_kernel<VV><<<pgrid, kCopyThreads, 0, s>>>(px, sb, sh, sr, (int)row_bytes, cu_seqlens, B, total_tokens, \
                                                      total_padded, po)
  switch (V) {
    case 16: FMLM_PACK(16); break;
    case 8: FMLM_PACK(8); break;
    case 4: FMLM_PACK(4); break;
    case 2: FMLM_PACK(2); break;
    default: FMLM_PACK(1); break;
  }
#undef FMLM_PACK
  return check_launch("pack_rows_kernel");
}

extern "C" int fmlm_unpack_rows(const void* packed, int64_t total_tokens, int32_t H, int32_t head_dim,
                                int32_t elem_bytes, const int32_t* cu_seqlens, int32_t B, int32_t N, void* out,
                                void* stream) {
  if (!out || !cu_seqlens) return set_error(FMLM_ERR_INVALID, "null pointer argument");
  if (elem_bytes <= 0 || head_dim <= 0 || H < 0 || B < 0 || N < 0 || total_tokens < 0)
    return set_error(FMLM_ERR_INVALID, "bad unpack sizes");
  const long long row_bytes = (long long)elem_bytes * head_dim;
  const long long n_rows = (long long)B * H * N;
  if (n_rows == 0) return FMLM_OK;
  long long g = row_bytes;
  for (long long a : {(long long)reinterpret_cast<uintptr_t>(packed), (long long)reinterpret_cast<uintptr_t>(out)})
    g = std::__gcd(g, a == 0 ? g : a);
  const int V = pick_vec(g);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto pp = reinterpret_cast<const uint8_t*>(packed);
  auto po = reinterpret_cast<uint8_t*>(out);
  const dim3 ugrid((unsigned)((N + kRowsPerCta - 1) / kRowsPerCta), (unsigned)H, (unsigned)std::min(B, 65535));
  if (H > 65535) return set_error(FMLM_ERR_INVALID, "bad unpack sizes");
#define FMLM_UNPACK(VV) \
  unpack_rows_kernel<VV><<<ugrid, kCopyThreads, 0, s>>>(pp, total_tokens, H, (int)row_bytes, cu_seqlens, B, N, po)
  switch (V) {
    case 16: FMLM_UNPACK(16); break;
    case 8: FMLM_UNPACK(8); break;
    case 4: FMLM_UNPACK(4); break;
    case 2: FMLM_UNPACK(2); break;
    default: FMLM_UNPACK(1); break;
  }
#undef FMLM_UNPACK
  return check_launch("unpack_rows_kernel");
}

extern "C" int fmlm_pad_packed_rows(const void* src, int64_t old_len, int64_t new_len, int32_t heads,
                                    int32_t head_dim, int32_t elem_bytes, void* dst, void* stream) {
  if (!dst || (!src && old_len > 0)) return set_error(FMLM_ERR_INVALID, "null pointer argument");
  if (old_len < 0 || new_len < old_len || heads < 0 || head_dim <= 0 || elem_bytes <= 0)
    return set_error(FMLM_ERR_INVALID, "bad pad sizes");
  const long long row_bytes = (long long)elem_bytes * head_dim;
  const long long n_rows = (long long)heads * new_len;
  if (n_rows == 0) return FMLM_OK;
  long long g = row_bytes;
  for (long long a : {(long long)reinterpret_cast<uintptr_t>(src), (long long)reinterpret_cast<uintptr_t>(dst)})
    g = std::__gcd(g, a == 0 ? g : a);
  const int V = pick_vec(g);
  const long long n = n_rows * (row_bytes / V);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto ps = reinterpret_cast<const uint8_t*>(src);
  auto pd = reinterpret_cast<uint8_t*>(dst);
#define FMLM_PAD(VV) pad_rows_kernel<VV><<<grid_for(n), 256, 0, s>>>(ps, old_len, new_len, heads, (int)row_bytes, pd)
  switch (V) {
    case 16: FMLM_PAD(16); break;
    case 8: FMLM_PAD(8); break;
    case 4: FMLM_PAD(4); break;
    case 2: FMLM_PAD(2); break;
    default: FMLM_PAD(1); break;
  }
#undef FMLM_PAD
  return check_launch("pad_rows_kernel");
}

extern "C" int fmlm_cache_append(const fmlm_view4* k, const fmlm_view4* v, int32_t src_layout, int32_t elem_bytes,
                                 int32_t head_dim, const int32_t* cu_seqlens, int32_t B, int64_t total_tokens,
                                 void* k_cache, void* v_cache, int64_t capacity, int32_t* cu_seqlens_kv,
                                 int32_t entries_before, int32_t* error_word, void* stream) {
  if (!k || !k_cache || !cu_seqlens || !cu_seqlens_kv || !error_word)
    return set_error(FMLM_ERR_INVALID, "null pointer argument");
  if ((v == nullptr) != (v_cache == nullptr)) return set_error(FMLM_ERR_INVALID, "v and v_cache must be given together");
  if (elem_bytes <= 0 || head_dim <= 0 || B < 0 || total_tokens < 0 || capacity < 0 || entries_before < 0)
    return set_error(FMLM_ERR_INVALID, "bad cache-append sizes");
  if (src_layout != FMLM_LAYOUT_PADDED && src_layout != FMLM_LAYOUT_PACKED)
    return set_error(FMLM_ERR_INVALID, "src_layout must be FMLM_LAYOUT_PADDED or FMLM_LAYOUT_PACKED");
  if (total_tokens > capacity) return set_error(FMLM_ERR_INVALID, "appended rows exceed the cache capacity");
  if (v && (v->heads != k->heads || v->batch_stride != k->batch_stride || v->head_stride != k->head_stride ||
            v->row_stride != k->row_stride))
    return set_error(FMLM_ERR_INVALID, "k and v views must have the same shape and strides");
  if (B == 0) return FMLM_OK;
  const int H = (int)k->heads;
  if (H <= 0 || H * (v ? 2 : 1) > 65535) return set_error(FMLM_ERR_INVALID, "bad head count");
  if (total_tokens > 0 && (!k->data || (v && !v->data))) return set_error(FMLM_ERR_INVALID, "k/v have no data");
  const long long row_bytes = (long long)elem_bytes * head_dim;
  const long long sb = k->batch_stride * elem_bytes, sh = k->head_stride * elem_bytes, sr = k->row_stride * elem_bytes;
  long long g = row_bytes;
  for (long long a : {sb, sh, sr, (long long)reinterpret_cast<uintptr_t>(k->data),
                      (long long)reinterpret_cast<uintptr_t>(v ? v->data : k->data),
                      (long long)reinterpret_cast<uintptr_t>(k_cache),
                      (long long)reinterpret_cast<uintptr_t>(v_cache ? v_cache : k_cache)})
    g = std::__gcd(g, a == 0 ? g : a);
  const int V = pick_vec(g);
  // Rows per sequence are bounded by the source view (padded) or by the
  // appended total (packed).
  const long long max_rows = std::max<long long>(1, src_layout == FMLM_LAYOUT_PADDED ? k->rows : total_tokens);
  const dim3 grid((unsigned)((max_rows + kRowsPerCta - 1) / kRowsPerCta), (unsigned)(H * (v ? 2 : 1)),
                  (unsigned)std::min(B, 65535));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto sk = reinterpret_cast<const uint8_t*>(k->data);
  auto sv = reinterpret_cast<const uint8_t*>(v ? v->data : k->data);
  auto dk = reinterpret_cast<uint8_t*>(k_cache);
  auto dv = reinterpret_cast<uint8_t*>(v_cache ? v_cache : k_cache);
  const int packed = src_layout == FMLM_LAYOUT_PACKED;
#define FMLM_APPEND(VV)                                                                                           \
  cache_append_kernel<VV><<<grid, kCopyThreads, 0, s>>>(sk, sv, sb, sh, sr, packed, (int)row_bytes, cu_seqlens, B, \
                                                        H, total_tokens, dk, dv, capacity, cu_seqlens_kv,        \
                                                        entries_before, error_word)
  switch (V) {
    case 16: FMLM_APPEND(16); break;
    case 8: FMLM_APPEND(8); break;
    case 4: FMLM_APPEND(4); break;
    case 2: FMLM_APPEND(2); break;
    default: FMLM_APPEND(1); break;
  }
#undef FMLM_APPEND
  return check_launch("cache_append_kernel");
}
