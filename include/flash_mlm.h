/*
 * flash_mlm.h -- C ABI of the B200 (sm_100a) flash-mlm forward path.
 *
 * The reference implementation (vymao/flash-mlm 1.2.2) is Python + Triton and
 * has no foreign-function interface of its own: its host launchers call Triton
 * kernels and torch ops directly.  Each entry point below replaces one of those
 * device-side steps; the comment on each names the reference code it replaces
 * (paths relative to the reference project root).
 *
 * Conventions
 *   - All pointers are device pointers unless stated otherwise.  The caller
 *     owns every buffer; the library allocates no device memory at run time.
 *     One exception: fmlm_attn_packed_fwd_noalloc keeps its tile schedule in
 *     a statically sized 256 KB __device__ array owned by the library, held on
 *     every GPU that loads the library until exit.
 *   - `stream` is a cudaStream_t passed as void*.  Every call is asynchronous
 *     on that stream.
 *   - Return value: 0 on success, a negative FMLM_ERR_* code otherwise;
 *     fmlm_last_error() gives a message (thread-local).
 *   - Strides are in elements; the innermost (head_dim) dimension must be
 *     contiguous.
 */
#ifndef FLASH_MLM_H_
#define FLASH_MLM_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FMLM_API __attribute__((visibility("default")))
#else
#define FMLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FMLM_OK = 0,
  FMLM_ERR_INVALID = -1,     /* bad argument (shape, stride, alignment, size) */
  FMLM_ERR_UNSUPPORTED = -2, /* head_dim / dtype combination not built */
  FMLM_ERR_CUDA = -3         /* a CUDA runtime / driver call failed */
};

enum { FMLM_DTYPE_F16 = 0, FMLM_DTYPE_BF16 = 1 };

/* A [batch][heads][rows][head_dim] view of a tensor.  A packed rank-2 tensor
 * [heads * rows, head_dim] is batch = 1, head_stride = rows * head_dim,
 * row_stride = head_dim. */
typedef struct fmlm_view4 {
  const void* data;
  int64_t rows, heads, batch;
  int64_t row_stride, head_stride, batch_stride;
} fmlm_view4;

/* Arguments of the dense launcher.
 * Replaces the `_mlm_main_kernel` launch in flash_attn_mlm
 * (src/flash_mlm/host/host.py:164-204; kernel math src/flash_mlm/mlm_kernel_impl.py:65-216). */
typedef struct fmlm_dense_args {
  int32_t dtype;              /* FMLM_DTYPE_* */
  int32_t head_dim;           /* 16, 32, 64, 128, 256 */
  int32_t batch, num_heads, seq_len;
  int32_t is_mla;             /* V is K; context rows are not head-offset */
  int32_t prefill;            /* skip the context segment */
  int32_t context_batch_size; /* > 1: context batch b for query batch b; 1: shared */
  int32_t context_len;        /* uniform context length (0 = none) */
  float scale;
  fmlm_view4 q, k, v;         /* [B,H,N,D] */
  fmlm_view4 k_cache, v_cache;/* rows = context_len, heads = H (1 for MLA), batch = context_batch_size */
  void* out;                  /* [B,H,N,D] contiguous, dtype of q */
  int32_t* error_word;        /* device int32; kernels set 1 if a bounded wait gave up, 2 if shared memory was
                                 misaligned (the packed path also: 3 context_index out of range, 4 a sequence
                                 with more than 65536 work items) */
} fmlm_dense_args;

enum { FMLM_LAYOUT_PADDED = 0, FMLM_LAYOUT_PACKED = 1 };

/* Arguments of the packed (variable-length) launcher.
 * Replaces the `_mlm_compressed_kernel` launch of flash_attn_mlm_compressed and
 * flash_attn_mlm_precompressed (src/flash_mlm/host/host.py:471-521, :727-786;
 * kernel math src/flash_mlm/mlm_kernel_impl.py:219-390) together with the
 * pack/pad step in front of it (src/flash_mlm/host/host_utils.py:423-491) and the
 * trim behind it (host.py:523-528): q/k/v may be given padded [B,H,N,D] and are
 * read in place. */
typedef struct fmlm_packed_args {
  int32_t dtype, head_dim, num_heads, batch;
  int32_t is_mla, prefill, causal_query_seq_attn;
  int32_t context_batch_size;       /* > 1: context batch b for query batch b; 1: shared */
  float scale;
  int32_t q_layout;                 /* FMLM_LAYOUT_*; padded: q is [B,H,N,D] */
  int32_t kv_layout;                /* FMLM_LAYOUT_*; layout of the main k/v */
  int32_t seq_len;                  /* N of padded layouts */
  int64_t total_q_len;              /* packed layouts: rows per head of q/k/v (>= total tokens) */
  fmlm_view4 q, k, v;               /* MLA: k has heads = 1 (head 0 of the caller's k) and v is ignored */
  fmlm_view4 k_cache, v_cache;      /* [H][total_context_len] (MLA: heads = 1) */
  const int32_t* cu_seqlens_q;      /* [batch + 1] */
  const int32_t* cu_seqlens_kv;     /* [>= context_batch_size + 1], or NULL when there is no context */
  void* out;                        /* [H * out_rows_per_head, D], or [batch][H][seq_len][D] (out_padded) */
  int64_t out_rows_per_head;
  void* workspace;                  /* fmlm_packed_workspace_bytes() bytes, 16-byte aligned */
  size_t workspace_bytes;
  int32_t* error_word;
  int32_t reuse_schedule;           /* 1: the workspace already holds the tile schedule of an earlier call
                                       with the same cu_seqlens / context / flags; skip rebuilding it */
  const int32_t* context_index;     /* optional [batch] (device): query batch b attends context entry
                                       context_index[b] (0 <= index < context_batch_size); NULL: the
                                       context_batch_size rule.  An index out of range attends no context
                                       and sets the error word.  No counterpart in the reference, whose
                                       README lists index-mapped context batching as planned. */
  int32_t out_padded;               /* 0: out is packed [H * out_rows_per_head, D] (rows of no sequence are left
                                       unwritten).  1: out is padded [batch][H][seq_len][D], contiguous, with
                                       zero rows past each sequence's length: the unpack step
                                       (src/flash_mlm/host/host_utils.py:587-615) done by the attention epilogue. */
} fmlm_packed_args;

/* Dense bidirectional attention over [context ++ own sequence]. */
FMLM_API int fmlm_attn_dense_fwd(const fmlm_dense_args* args, void* stream);

/* Packed variable-length attention over [context segment ++ main segment]. */
FMLM_API int fmlm_attn_packed_fwd(const fmlm_packed_args* args, void* stream);

/* Same computation as fmlm_attn_packed_fwd, but allocation-free: `workspace`
 * and `workspace_bytes` are ignored and the tile schedule is kept in a fixed
 * 256 KB array in device memory that the library owns (held by every GPU that
 * loads the library until exit).  No counterpart in the reference: it exists
 * for callers that cannot allocate device memory (capture of a CUDA graph,
 * hosts whose allocator is locked after start-up, plugin hosts that only pass
 * pre-allocated buffers).  The first call in each CUDA context of a device
 * looks the array's address up (make it before any stream capture).  Problems whose schedule would exceed
 * the array (batch + total_q_len / 128 above about 65500) are rejected with
 * FMLM_ERR_INVALID.  All calls share the array: calls that overlap on the GPU
 * race, so serialise them. */
FMLM_API int fmlm_attn_packed_fwd_noalloc(const fmlm_packed_args* args, void* stream);

/* Workspace size for fmlm_attn_packed_fwd (on-device tile schedule). */
FMLM_API size_t fmlm_packed_workspace_bytes(int32_t batch, int64_t total_q_len, int32_t head_dim);

/* Pack metadata from per-sequence lengths.
 * Replaces build_pack_metadata + _build_query_tile_map_from_cu_seqlens
 * (src/flash_mlm/host/host_utils.py:27-107).
 *   lengths          [B] int32
 *   cu_seqlens       [B+1] int32 (out)
 *   token_indices    [B*N] int64 capacity (out; first total_tokens valid); may be NULL
 *   batch_ids_q      [B*ceil(N/block_n)] int32 capacity (out)
 *   q_tile_starts_q  [B*ceil(N/block_n)] int32 capacity (out)
 *   counters         [B + 5] int32 scratch (out): [0] total_tokens, [1] number of tiles,
 *                    [2] non-zero if some length is outside [0, N]. */
FMLM_API int fmlm_build_pack_metadata(const int32_t* lengths, int32_t B, int32_t N, int32_t block_n,
                             int32_t* cu_seqlens, int64_t* token_indices, int32_t* batch_ids_q,
                             int32_t* q_tile_starts_q, int32_t* counters, void* stream);

/* Gather the valid rows of x [B][H][N][D] into out [H * total_padded, D], zeroing
 * rows [total_tokens, total_padded) of every head.
 * Replaces _pack_flatten_for_kernel_into / pack_for_kernel
 * (src/flash_mlm/host/host_utils.py:266-289, :397-420). */
FMLM_API int fmlm_pack_rows(const fmlm_view4* x, int32_t elem_bytes, int32_t head_dim, const int32_t* cu_seqlens,
                   int32_t B, int64_t total_tokens, int64_t total_padded, void* out, void* stream);

/* Scatter packed [H * total_tokens, D] into out [B][H][N][D] (contiguous),
 * writing zeros at padding positions, in one pass.
 * Replaces unpack_from_kernel (src/flash_mlm/host/host_utils.py:587-615). */
FMLM_API int fmlm_unpack_rows(const void* packed, int64_t total_tokens, int32_t H, int32_t head_dim,
                     int32_t elem_bytes, const int32_t* cu_seqlens, int32_t B, int32_t N, void* out,
                     void* stream);

/* Append B sequences of K (and V) rows to a head-major context cache with spare
 * capacity: k_cache / v_cache are [H][capacity][D] (MLA: H = 1, v = v_cache =
 * NULL).  The cache already holds cu_seqlens_kv[entries_before] rows per head
 * (read on the device); sequence b (length cu_seqlens[b+1] - cu_seqlens[b]) is
 * written at row cu_seqlens_kv[entries_before] + cu_seqlens[b] - cu_seqlens[0]
 * of every head, and cu_seqlens_kv[entries_before + 1 + b] receives its end
 * offset, so cu_seqlens_kv[0 .. entries_before + B] describes every entry
 * without a host round trip.  src_layout FMLM_LAYOUT_PADDED: k / v are
 * [B][H][N][D] views (row t of batch b); FMLM_LAYOUT_PACKED: [H][T][D] views
 * (row cu_seqlens[b] + t, batch 1).  total_tokens = cu_seqlens[B] - cu_seqlens[0].
 * If the appended rows would pass `capacity`, nothing is written and
 * *error_word is set to 5.
 * Replaces the prefill store of flash_attn_mlm_compressed / precompressed
 * (src/flash_mlm/host/host.py:327-364, :775-787), which packs this call's K/V into a
 * new per-layer buffer, with an append into a preallocated one; with a padded
 * [B][H][ctx] source and uniform cu_seqlens it also converts the dense
 * prefill layout (src/flash_mlm/host/host.py:206-223) to the packed one. */
FMLM_API int fmlm_cache_append(const fmlm_view4* k, const fmlm_view4* v, int32_t src_layout, int32_t elem_bytes,
                               int32_t head_dim, const int32_t* cu_seqlens, int32_t B, int64_t total_tokens,
                               void* k_cache, void* v_cache, int64_t capacity, int32_t* cu_seqlens_kv,
                               int32_t entries_before, int32_t* error_word, void* stream);

/* Copy packed [H * old_len, D] into [H * new_len, D] with zero rows appended per head.
 * Replaces the pad step of pad_packed_main_tensors_for_mlm_compressed
 * (src/flash_mlm/host/host_utils.py:494-584). */
FMLM_API int fmlm_pad_packed_rows(const void* src, int64_t old_len, int64_t new_len, int32_t heads, int32_t head_dim,
                         int32_t elem_bytes, void* dst, void* stream);

/* Self-test of the kernels' bounded waits (no counterpart in the reference):
 * launches one CTA that waits on an mbarrier nobody arrives on, with the given
 * limit.  The wait must give up and write 1 to *error_word (device int32);
 * the GPU context stays usable.  Returns 0 if the launch succeeded. */
FMLM_API int fmlm_selftest_bounded_wait(int32_t* error_word, uint64_t limit_ns, void* stream);

/* Message of the last failed call on this thread ("" if none). */
FMLM_API const char* fmlm_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
FMLM_API int fmlm_version(void);

#ifdef __cplusplus
}
#endif
#endif /* FLASH_MLM_H_ */
