// Bidirectional MLM attention forward for sm_100a (B200).
//
// Semantics follow the reference Triton kernels:
//   * src/flash_mlm/mlm_kernel_impl.py:10-62   (_mlm_inner_attention: masked online softmax)
//   * src/flash_mlm/mlm_kernel_impl.py:65-216  (_mlm_main_kernel_impl: dense [B,H,N,D])
//   * src/flash_mlm/mlm_kernel_impl.py:219-390 (_mlm_compressed_kernel_impl: packed varlen,
//     context segment then main segment, causal_query_seq_attn prefix, MLA)
// Every query row attends to [context segment] ++ [main segment]; rows with no
// key at all produce zeros (l_safe, mlm_kernel_impl.py:381).
//
// Design (one persistent CTA per SM, warp specialised):
//   warps [0, 4*NQ)   softmax warpgroups, one per 128-row query tile; each
//                     thread owns one query row (one TMEM lane)
//   warp 4*NQ         TMA producer (Q tiles, K/V blocks through a STAGES ring)
//   warp 4*NQ+1       TMEM allocator + single-thread tcgen05.mma issuer
// A work item is NQ query tiles of 128 rows from the same (sequence, head);
// they share every K/V block.  S = Q K^T lands in TMEM (fp32), softmax reads
// it with tcgen05.ld, writes P (f16/bf16) back over S, and O += P V is issued
// with P as the TMEM operand.  The running max is only moved (and O rescaled
// in TMEM) when a new block raises it by more than 2^8, which keeps P <= 256.
// MMA order per block j is  PV_t(j), S_t(j+1)  for each tile t, so when the
// softmax sees S_t(j+1) complete, PV_t(j) is complete too (tcgen05 ops issued
// by one thread complete in order and a commit covers all earlier ops).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace fmlm {

// Error codes written to the device error word.
enum : int { kErrTimeout = 1, kErrSmemAlign = 2, kErrContextIndex = 3, kErrSeqTooLong = 4 };

// Packed-mode workspace (int32): [0] entry count, [1] next-item counter,
// [2] CTAs finished, [3] unused, then one (b << 16 | pair) entry per query
// pair.  The schedule kernel zeroes [1] and [2]; the last CTA of each
// attention launch zeroes them again, so a reused schedule starts clean.
constexpr int kWorkHeader = 4;

struct AttnParams {
  int mode;         // 0 = dense [B,H,N,D] rows; 1 = packed variable-length (cu_seqlens_q)
  int q_padded;     // packed: Q rows come from a padded [B,H,N,D] tensor (1) or packed [H*Tq,D] (0)
  int main_padded;  // packed: main K/V rows from padded [B,Hkv,N,D] (1) or packed [Hkv*Tk,D] (0)
  int causal;       // packed: main range is the prefix [0, cu_q[b+1]) (causal_query_seq_attn)
  int has_ctx;      // a context segment is attended (prefill=False and context rows exist)
  int is_mla;       // V is the K tile; K/V head coordinate is 0 (except dense main keys)
  int B, H, N;      // N: dense / padded sequence length
  int ctx_bs;       // context batch size
  int ctx_len;      // dense: uniform context length per context batch
  long long t_out;  // packed: rows per head in the output
  int out_padded;   // packed: output is [B, H, N, D] with zero rows past each sequence (else packed [H*t_out, D])
  int num_items;    // dense: number of work items
  float scale_log2; // scale * log2(e)
  const int* cu_q;  // [B+1] packed query offsets
  const int* cu_kv; // context offsets (packed)
  const int* ctx_index;  // packed, optional: context entry of each query batch
  int* work;        // packed: schedule workspace (layout at kWorkHeader)
  void* out;        // [rows, D]
  int* err;         // device error word
  const uint16_t* q_ptr;          // TQ: q itself (16-bit elements), read by the softmax warps
  long long q_sb, q_sh, q_sr;     // its batch / head / row strides in elements
  unsigned long long timeout_ns;
  unsigned long long* trace;  // optional timeline buffer (builds with FMLM_TRACE only)
};

// Opt-in timeline instrumentation (builds with -DFMLM_TRACE only): in CTA 0
// each recording thread (one per role) appends (event << 48 | clock) records
// to its own shared-memory slice; the slices are copied to p.trace at exit
// (p.trace[0..3] = record counts, role r's records from 4 + r * kTraceSlots).
#ifdef FMLM_TRACE
#ifndef FMLM_TRACE_SLOTS
#define FMLM_TRACE_SLOTS 1024
#endif
// FMLM_TRACE_SLOTS = 0 records only per-CTA entry/exit times (no static
// shared memory, so the occupancy is that of the product build).
// FMLM_TRACE_SLOTS < 0 writes the records straight to global memory (1024
// per role), also without static shared memory.
constexpr bool kTraceGlobal = FMLM_TRACE_SLOTS < 0;
constexpr int kTraceSlots = kTraceGlobal ? 1024 : FMLM_TRACE_SLOTS;
#define FMLM_TR(ev)                                                                                   \
  do {                                                                                                \
    if (tr_role >= 0 && tr_n < kTraceSlots)                                                           \
      tr_buf[tr_role * kTraceSlots + tr_n++] = ((unsigned long long)(ev) << 48) | (clock64() & 0xFFFFFFFFFFFFull); \
  } while (0)
#else
#define FMLM_TR(ev) \
  do {              \
  } while (0)
#endif

template <int D_, int NQ_>
struct AttnCfg {
  static constexpr int D = D_;
  static constexpr int NQ = NQ_;
  static constexpr int BM = 128;                   // query rows per tile (UMMA M)
  // D = 512 is the MLA latent width: O (128 x 512 fp32) alone would fill TMEM,
  // so a work item accumulates one 256-column half of O (DV) and S is
  // recomputed for the other half.  V is the K tile (MLA only).
  static constexpr int DV = (D == 512) ? 256 : D;  // O columns per work item
  static constexpr int NDH = D / DV;               // work items per (tile, head)
  static constexpr bool MLA_ONLY = (D == 512);
#ifndef FMLM_PINGPONG
#define FMLM_PINGPONG 1
#endif
#ifndef FMLM_BN_D128
#define FMLM_BN_D128 128
#endif
#ifndef FMLM_MLA_TQ
#define FMLM_MLA_TQ 1
#endif
  // D = 512: Q columns [QS, D) are kept in TMEM instead of shared memory and
  // that half of S = Q Kᵀ is issued with A from TMEM.  The 64 KB this frees
  // holds 64-key K tiles (S at N=64) instead of 32-key ones (N=32, a third of
  // the tensor rate).
  static constexpr bool TQ = FMLM_MLA_TQ && D == 512;
  static constexpr int QS = TQ ? D / 2 : D;        // Q columns staged in shared memory
#ifndef FMLM_MLA_BN
#define FMLM_MLA_BN 48
#endif
#ifndef FMLM_MLA_KSPLIT
#define FMLM_MLA_KSPLIT 1
#endif
  // KSPLIT (with TQ): the K tile is held as two 256-column halves in two
  // rings.  The half this item uses as V (columns dh*DV ...) stays until PV;
  // the other half is needed only by S and is released as soon as S has run,
  // so a shorter ring suffices and 64-key blocks fit in shared memory.
  static constexpr bool KSPLIT = TQ && FMLM_MLA_KSPLIT;
  static constexpr int BN = (D == 512) ? (KSPLIT ? 64 : TQ ? FMLM_MLA_BN : 32) : (D >= 256) ? 64 : (D == 128) ? FMLM_BN_D128 : 128;  // key rows per block
  static constexpr int PAIR = NQ * BM;             // query rows per work item
  static constexpr int SWB = (D * 2 >= 128) ? 128 : D * 2;  // swizzle span in bytes
  static constexpr int SLAB_COLS = SWB / 2;
  static constexpr int NSLAB = D / SLAB_COLS;
  static constexpr int Q_BYTES = BM * QS * 2;
  static constexpr int Q_NSLAB = QS / SLAB_COLS;
  static constexpr int KV_BYTES = KSPLIT ? BN * (D / 2) * 2 : BN * D * 2;  // KSPLIT: one half tile
  static constexpr int KNSLAB = KSPLIT ? NSLAB / 2 : NSLAB;  // swizzle slabs per K/V tile in shared memory
  static constexpr int SHORT_STAGES = KSPLIT ? 2 : 0;        // KSPLIT: ring of the halves used by S only
  // One tile per CTA at D <= 64 runs two CTAs per SM (TMEM 256 columns and
  // about 80 KB of shared memory each): the two CTAs work on independent items.
  static constexpr int CTAS_PER_SM = (NQ == 1 && D <= 64) ? 2 : 1;
#ifndef FMLM_STAGES_2CTA
#define FMLM_STAGES_2CTA 3
#endif
#ifndef FMLM_EARLY_O
#define FMLM_EARLY_O 1
#endif
#ifndef FMLM_QBUF_2CTA
#define FMLM_QBUF_2CTA 1
#endif
  // Q buffers: with two, the next item's Q is loaded while the current item
  // still computes, so its first S is ready when the softmax reaches it.
  static constexpr int QBUF = (CTAS_PER_SM == 2) ? FMLM_QBUF_2CTA : 1;
#ifndef FMLM_STAGES_D64_NQ2
#define FMLM_STAGES_D64_NQ2 3
#endif
  static constexpr int STAGES = (CTAS_PER_SM == 2) ? (QBUF == 2 ? 2 : FMLM_STAGES_2CTA) : (D <= 32) ? 4 : (D <= 64) ? FMLM_STAGES_D64_NQ2 : (D == 512) ? ((TQ && !KSPLIT) ? (BN <= 48 ? 3 : 2) : 3)
                              : (D == 128 && BN == 64) ? 4 : 2;
#ifndef FMLM_POLY_EXP
#define FMLM_POLY_EXP 0
#endif
#ifndef FMLM_POLY_EXP_D128
#define FMLM_POLY_EXP_D128 0
#endif
  // One pair of exponentials in POLY is evaluated on the FMA pipe (0: all on MUFU).
  static constexpr int POLY = (D <= 64) ? FMLM_POLY_EXP : (D == 128) ? FMLM_POLY_EXP_D128 : 0;
  static_assert(STAGES >= 1 && STAGES <= 4, "the barrier block holds four K/V stages");
#ifndef FMLM_SPLIT_KV
#define FMLM_SPLIT_KV 0
#endif
  // SPLIT_KV (separate K and V tiles): a K stage is released as soon as the S
  // that read it completes (k_empty) and a V stage when its P V completes
  // (kv_empty), and the producer requests V one block behind K, so K(j) is
  // requested about one block earlier than with a shared release after P V.
  // (With MLA at run time the K tile is also V: it is released after P V.)
  static constexpr bool SPLIT_KV = FMLM_SPLIT_KV && D != 512;
  static constexpr int NUM_SOFTMAX_WARPS = 4 * NQ;
  static constexpr int TMA_WARP = NUM_SOFTMAX_WARPS;
  static constexpr int MMA_WARP = NUM_SOFTMAX_WARPS + 1;  // one MMA-issuing warp per tile: MMA_WARP + t
  static constexpr int THREADS = 32 * (NUM_SOFTMAX_WARPS + 1 + NQ);
  // Each SM sub-partition owns a quarter of the register file; the warps of
  // all resident CTAs are spread over the four, so the budget is
  // 16384 / (32 * ceil(warps per SM / 4)).  (Measured: two 6-warp CTAs at 168
  // registers are resident together, although the occupancy API, which
  // assumes warp w of every CTA sits on sub-partition w % 4, reports one.)
  static constexpr int WARPS_PER_SMSP = (CTAS_PER_SM * (NUM_SOFTMAX_WARPS + 1 + NQ) + 3) / 4;
  static constexpr int MAX_REGS = (16384 / (32 * WARPS_PER_SMSP)) / 8 * 8 > 255 ? 255
                                : (16384 / (32 * WARPS_PER_SMSP)) / 8 * 8;
  // P gets its own TMEM columns when they fit (D <= 64 with two tiles, or one
  // tile): S_t(j+1) can then be issued as soon as the softmax has read S_t(j).
  // Otherwise P is written over the first BN/2 columns of S_t.
  // SDB (with TQ): two S buffers, P written over the first half of its own
  // S buffer, so S(j+1) is queued on the tensor pipe while the softmax works
  // on S(j); a buffer is reused only after the PV that read its P was issued
  // (tcgen05 ops of one thread run in order).
  static constexpr bool SDB = TQ;
  static constexpr bool SEP_P = !SDB && NQ * (BN + DV + BN / 2) <= 512;
#ifndef FMLM_SPLIT_PV
#define FMLM_SPLIT_PV 0
#endif
  // SPLIT_PV (separate P, one tile): P is written and consumed in two halves
  // of the key block.  The softmax stores half h of P(j) and signals it on
  // p_full[h]; the MMA warp issues the P V MMAs of that half at once and
  // commits pv_done[h].  Writing half h of P(j+1) then waits only for half h
  // of P V(j), which was issued half an exponential loop earlier, so the
  // P V latency leaves the softmax's critical path.
  static constexpr bool SPLIT_PV = SEP_P && NQ == 1 && FMLM_SPLIT_PV;
  static constexpr int TM_S = 0;                   // S_t at column t*BN (SDB: buffer b at b*BN)
  static constexpr int TM_O = SDB ? 2 * BN : NQ * BN;  // O_t at column TM_O + t*DV
  static constexpr int TM_P = SEP_P ? NQ * (BN + DV) : 0;  // P_t at TM_P + t*BN/2 (or over S_t)
  static constexpr int TM_Q1 = 384;                // TQ: Q columns [QS, D) as packed pairs, (D - QS) / 2 columns
  static constexpr int TMEM_USED = TQ ? TM_Q1 + (D - QS) / 2 : NQ * (BN + DV) + (SEP_P ? NQ * BN / 2 : 0);
  static_assert(!TQ || (NQ == 1 && SDB && 2 * BN + DV <= TM_Q1), "TQ TMEM layout");
  static constexpr int TMEM_COLS = TMEM_USED <= 32 ? 32 : TMEM_USED <= 64 ? 64 : TMEM_USED <= 128 ? 128
                                 : TMEM_USED <= 256 ? 256 : 512;
  static_assert(TMEM_USED <= 512, "TMEM budget");
  static constexpr int SMEM_TILES = QBUF * NQ * Q_BYTES + (MLA_ONLY ? 1 : 2) * STAGES * KV_BYTES + SHORT_STAGES * KV_BYTES;
  // Two CTAs with three K/V stages need all but 1.5 KB of the SM's 228 KB, so
  // they carry no alignment slack: the dynamic shared window of a kernel with
  // no static shared memory starts 1024-byte aligned, which the kernel checks.
#if defined(FMLM_TRACE) && FMLM_TRACE_SLOTS > 0
  static constexpr int ALIGN_PAD = 1024;
#else
  static constexpr int ALIGN_PAD = (CTAS_PER_SM == 2) ? 0 : 1024;
#endif
  static constexpr int ITEM_RING_BYTES = 4 * 96;  // decoded work items passed producer -> consumers
  static constexpr int SMEM_BYTES = SMEM_TILES + 512 /*barriers*/ + ITEM_RING_BYTES + ALIGN_PAD;
};

struct Seg {
  int map;  // 0 = context tensors, 1 = main tensors
  int h, b; // head / batch coordinates in that tensor map
  int row0, row1;
  int fix;  // rows past row1 inside the tensor are caller padding: zero them in V
  int nblk;
};

// One work item: up to two 128-row query tiles of one (sequence, head) and the
// two key segments they attend (context, then main).  Kept as scalars so no
// role needs dynamically indexed local memory.
struct Item {
  int qb, qh, qrow0;
  // Bit 0: which DV-wide column block of O this item produces (dh).  Bits
  // 1-31, padded output only: rows [0, zero_limit) from out_row0 are this
  // item's to write; rows at or past its valid query rows get zeros (the last
  // item of a sequence also owns the padding rows up to N); 0 otherwise.
  int dh_zl;
  int qrows0, qrows1;
  long long out_row0;
  Seg ctx, main;
  __device__ __forceinline__ int qrows(int t) const { return t == 0 ? qrows0 : qrows1; }
  __device__ __forceinline__ int dh() const { return dh_zl & 1; }
  __device__ __forceinline__ int zero_limit() const { return dh_zl >> 1; }
  __device__ __forceinline__ int nblocks() const { return ctx.nblk + main.nblk; }
  // Segment and first row of key block j (j counts context blocks first).
  __device__ __forceinline__ Seg block_seg(int j, int bn, int& row) const {
    const bool in_ctx = j < ctx.nblk;
    const Seg s = in_ctx ? ctx : main;
    row = s.row0 + (in_ctx ? j : j - ctx.nblk) * bn;
    return s;
  }
};

template <int PAIR, int BN, int NDH>
__device__ __forceinline__ Item decode_item(const AttnParams& p, int w) {
  Item it;
  it.dh_zl = w % NDH;
  w /= NDH;
  const int h = w % p.H;
  const int r = w / p.H;
  int b, pair, L, seq_start;
  if (p.mode == 0) {
    const int npairs = (p.N + PAIR - 1) / PAIR;
    pair = r % npairs;
    b = r / npairs;
    L = p.N;
    seq_start = 0;
  } else {
    const int e = __ldg(p.work + kWorkHeader + r);
    b = e >> 16;
    pair = e & 0xFFFF;
    seq_start = __ldg(p.cu_q + b);
    L = __ldg(p.cu_q + b + 1) - seq_start;
  }
  const int rel0 = pair * PAIR;
  it.qh = h;
  it.qrows0 = min(max(L - rel0, 0), 128);
  it.qrows1 = min(max(L - rel0 - 128, 0), 128);
  if (p.mode == 0) {
    it.qb = b;
    it.qrow0 = rel0;
    it.out_row0 = ((long long)b * p.H + h) * p.N + rel0;
  } else {
    it.qb = p.q_padded ? b : 0;
    it.qrow0 = p.q_padded ? rel0 : seq_start + rel0;
    if (p.out_padded) {
      it.out_row0 = ((long long)b * p.H + h) * p.N + rel0;
      it.dh_zl |= ((rel0 + PAIR >= L) ? p.N - rel0 : PAIR) << 1;
    } else {
      it.out_row0 = (long long)h * p.t_out + seq_start + rel0;
    }
  }
  const int kh = p.is_mla ? 0 : h;
  // context segment
  Seg& c = it.ctx;
  c.map = 0; c.h = kh; c.fix = 0;
  if (!p.has_ctx) {
    c.b = 0; c.row0 = 0; c.row1 = 0;
  } else if (p.mode == 0) {
    c.b = (p.ctx_bs > 1) ? b : 0; c.row0 = 0; c.row1 = p.ctx_len;
  } else {
    const int ci = p.ctx_index ? __ldg(p.ctx_index + b) : (p.ctx_bs > 1) ? b : 0;
    if (ci < 0 || ci >= p.ctx_bs) {
      atomicExch(p.err, kErrContextIndex);  // attend no context
      c.b = 0; c.row0 = 0; c.row1 = 0;
    } else {
      c.b = 0; c.row0 = __ldg(p.cu_kv + ci); c.row1 = __ldg(p.cu_kv + ci + 1);
    }
  }
  // main segment
  Seg& m = it.main;
  m.map = 1; m.fix = 0;
  if (p.mode == 0) {
    m.h = h;  // dense MLA attends the per-head keys (mlm_kernel_impl.py:124, :188-206)
    m.b = b; m.row0 = 0; m.row1 = p.N;
  } else if (p.main_padded) {
    m.h = kh; m.b = b; m.row0 = 0; m.row1 = L; m.fix = (L < p.N);
  } else {
    m.h = kh; m.b = 0; m.row0 = p.causal ? 0 : seq_start; m.row1 = seq_start + L;
  }
  c.nblk = c.row1 > c.row0 ? (c.row1 - c.row0 + BN - 1) / BN : 0;
  m.nblk = m.row1 > m.row0 ? (m.row1 - m.row0 + BN - 1) / BN : 0;
  if (L == 0) c.nblk = m.nblk = 0;  // an empty sequence's item only writes zero rows (padded output)
  return it;
}

static_assert(sizeof(Item) <= 96, "item ring slot");

struct __align__(8) AttnBarriers {
  uint64_t q_full[2], q_empty[2], fix;
  uint64_t k_full[4], v_full[4], kv_empty[4], k_empty[4];
  uint64_t s_full[2], p_full[2], o_full[2], o_empty[2];
  uint64_t s_free[2], pv_done[2];  // separate-P pipeline only
  uint64_t item_full[4], item_empty[4];  // ring of work-item indices, producer -> other roles
  int item_idx[4];
  uint64_t exp_tok[2];  // two-tile ping-pong: tile t may run its exp2 loop
  uint64_t q1_full;     // TQ: the softmax warps have written this item's Q columns [QS, D) to TMEM
  uint64_t ks_empty[2]; // KSPLIT: short-ring slot free (the S that read it has completed); v_full is its "full"
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(AttnBarriers) <= 512, "barrier block is reserved 512 bytes");

template <int D, int NQ, bool BF16>
__global__ void __launch_bounds__(AttnCfg<D, NQ>::THREADS) __maxnreg__((AttnCfg<D, NQ>::MAX_REGS))
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_kc,
                    const __grid_constant__ CUtensorMap tm_vc, const AttnParams p) {
  using C = AttnCfg<D, NQ>;
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  constexpr int BM = C::BM, BN = C::BN, SWB = C::SWB, STAGES = C::STAGES;
  constexpr int OC = (D >= 32) ? 32 : 16;  // O columns per TMEM transfer
  auto tmem_ld_chunk = [](uint32_t a, uint32_t(&o)[OC]) {
    if constexpr (OC == 32) tmem_ld_x32(a, o); else tmem_ld_x16(a, o);
  };
  auto tmem_st_chunk = [](uint32_t a, const uint32_t(&o)[OC]) {
    if constexpr (OC == 32) tmem_st_x32(a, o); else tmem_st_x16(a, o);
  };

  extern __shared__ uint8_t smem_raw[];
  if constexpr (C::ALIGN_PAD == 0) {
    if ((static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u) != 0) {
      if (threadIdx.x == 0) atomicExch(p.err, kErrSmemAlign);
      return;  // before any barrier, TMEM or TMA work
    }
  }
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::QBUF * NQ * C::Q_BYTES;
  uint8_t* sV = C::MLA_ONLY ? sK : sK + STAGES * C::KV_BYTES;
  uint8_t* sKs = sK + STAGES * C::KV_BYTES;  // KSPLIT short ring (SHORT_STAGES half tiles)
  AttnBarriers* bar = reinterpret_cast<AttnBarriers*>(sV + STAGES * C::KV_BYTES + C::SHORT_STAGES * C::KV_BYTES);
  volatile int* abort_flag = &bar->abort_flag;
  Item* item_ring = reinterpret_cast<Item*>(reinterpret_cast<uint8_t*>(bar) + 512);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool mla = p.is_mla != 0;
#ifdef FMLM_TRACE
#if FMLM_TRACE_SLOTS > 0
  __shared__ unsigned long long tr_buf[4 * kTraceSlots];
  __shared__ int tr_cnt[4];
#else
  unsigned long long* tr_buf = kTraceGlobal && p.trace ? p.trace + 4 : nullptr;
  int* tr_cnt = nullptr;
#endif
  int tr_n = 0;
  int tr_role = -1;
  if (kTraceSlots > 0 && p.trace && blockIdx.x == 0) {
    if (warp < C::NUM_SOFTMAX_WARPS && (threadIdx.x & 127) == 0) tr_role = warp >> 2;
    if (warp == C::TMA_WARP && lane == 0) tr_role = 2;
    if (warp == C::MMA_WARP && lane == 0) tr_role = 3;  // tile-0 MMA issuer
  }
  if (!kTraceGlobal && kTraceSlots > 0 && threadIdx.x < 4 && p.trace) tr_cnt[threadIdx.x] = 0;
  const uint64_t tr_entry_ns = global_timer_ns();
#endif

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar->q_full[i], 1);
      mbar_init(&bar->q_empty[i], NQ);
    }
    mbar_init(&bar->fix, 1);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->kv_empty[s], NQ);
      mbar_init(&bar->k_empty[s], NQ);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar->s_full[t], 1);
      mbar_init(&bar->p_full[t], 4);
      mbar_init(&bar->o_full[t], 1);
      mbar_init(&bar->o_empty[t], 4);
      mbar_init(&bar->s_free[t], 4);
      mbar_init(&bar->pv_done[t], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&bar->item_full[i], 1);
      mbar_init(&bar->item_empty[i], 5 * NQ);  // every MMA and softmax warp
    }
    mbar_init(&bar->q1_full, 4);
    mbar_init(&bar->ks_empty[0], 1);
    mbar_init(&bar->ks_empty[1], 1);
    mbar_init(&bar->exp_tok[0], 4);
    mbar_init(&bar->exp_tok[1], 4);
    bar->abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == C::MMA_WARP) {
    tmem_alloc(&bar->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == C::TMA_WARP && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_kc);
    tma_prefetch_desc(&tm_vc);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bar->tmem_base;

  const int num_items = (p.mode == 0) ? p.num_items : __ldg(p.work) * p.H * C::NDH;
  const uint64_t tmo = p.timeout_ns;
  bool failed = false;

  auto fail = [&]() {
    failed = true;
    *abort_flag = 1;
    atomicExch(p.err, kErrTimeout);
  };

  // Next work item for the MMA and softmax warps (whole warp): the index the
  // producer published in ring slot `ring`; num_items means no more work.
  // The producer also publishes the decoded item, so consumers do not repeat
  // decode_item's dependent global loads at every item start.
  auto take_item = [&](uint32_t ring, int& w, Item& it) -> bool {
    if (failed) return false;
    if (!mbar_wait(&bar->item_full[ring & 3], (ring >> 2) & 1u, abort_flag, tmo)) fail();
    failed = __any_sync(0xffffffffu, failed);
    if (failed) return false;
    w = *reinterpret_cast<volatile int*>(&bar->item_idx[ring & 3]);
    if (w < num_items) it = item_ring[ring & 3];
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar->item_empty[ring & 3]);
    return w < num_items;
  };

  if (warp == C::TMA_WARP) {
    // ------------------------------------------------------------ producer
    uint32_t fix_ph = 0;
    // A partial last block of a padded main segment: rows [valid, BN) of its V
    // tile (K for MLA) hold the caller's padding, which may be non-finite; P is
    // zero there but 0 * NaN is not, so they are cleared once the tile lands.
    // For a V tile the clearing is deferred to just before the producer's next
    // wait for a free K/V stage (the only wait that can depend on V), so the
    // next item's Q and first blocks are requested without waiting for it.
    uint8_t* pend_tile = nullptr;
    int pend_valid = 0;
    uint64_t* pend_bar = nullptr;
    auto resolve_fix = [&]() {
      if (pend_tile == nullptr || failed) return;
      if (!mbar_wait(&bar->fix, fix_ph, abort_flag, tmo)) fail();
      fix_ph ^= 1u;
      failed = __any_sync(0xffffffffu, failed);
      if (!failed) {
        const int nbytes = (BN - pend_valid) * SWB;
        for (int s = 0; s < C::KNSLAB; ++s) {
          uint4* z = reinterpret_cast<uint4*>(pend_tile + s * (BN * SWB) + pend_valid * SWB);
          for (int i = lane; i < nbytes / 16; i += 32) z[i] = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(pend_bar);
      }
      pend_tile = nullptr;
    };
    uint32_t fill = 0;
    // Work items are handed out dynamically: the first one is blockIdx.x, the
    // rest come from a global counter (packed mode; the schedule is sorted by
    // cost, so this is longest-first list scheduling), and each index is
    // passed to the other roles through the item ring.
    auto issue_q = [&](const Item& q_it, int qs) {
      if (lane == 0) {
        FMLM_TR(42);
        const uint32_t nq = (q_it.qrows0 > 0 ? 1u : 0u) + (NQ > 1 && q_it.qrows1 > 0 ? 1u : 0u);
        mbar_arrive_expect_tx(&bar->q_full[qs], nq * C::Q_BYTES);
#pragma unroll
        for (int t = 0; t < NQ; ++t) {
          if (q_it.qrows(t) == 0) continue;
          for (int s = 0; s < C::Q_NSLAB; ++s)
            tma_load_4d(sQ + (qs * NQ + t) * C::Q_BYTES + s * (BM * SWB), &tm_q, &bar->q_full[qs], s * C::SLAB_COLS,
                        q_it.qrow0 + t * BM, q_it.qh, q_it.qb);
        }
      }
      __syncwarp();
    };
    bool q_pre = false;
    Item cur;
    bool have_cur = false;  // cur holds the decoded item w (decoded during the previous item)
    int w = blockIdx.x;
    for (uint32_t ring = 0;; ++ring) {
      if (!mbar_wait(&bar->item_empty[ring & 3], ((ring >> 2) & 1u) ^ 1u, abort_flag, tmo)) fail();
      failed = __any_sync(0xffffffffu, failed);
      if (failed) break;
      const Item it = (w < num_items) ? (have_cur ? cur : decode_item<C::PAIR, BN, C::NDH>(p, w)) : Item{};
      if (lane == 0) {
        if (w < num_items) item_ring[ring & 3] = it;
        bar->item_idx[ring & 3] = w;
        mbar_arrive(&bar->item_full[ring & 3]);
      }
      if (w >= num_items) break;
      int next = 0;
      if (lane == 0) next = (p.mode == 0) ? w + (int)gridDim.x : (int)gridDim.x + atomicAdd(p.work + 1, 1);
      next = __shfl_sync(0xffffffffu, next, 0);
      // Q buffer ring % QBUF, used for the (ring / QBUF)-th time.  With two
      // buffers the next item's Q is requested during this item, as soon as
      // its buffer is free (q_pre), so it has landed when this item ends.
      if (!q_pre) {
        const int qs = ring % C::QBUF;
        if (!mbar_wait(&bar->q_empty[qs], ((ring / C::QBUF) & 1u) ^ 1u, abort_flag, tmo)) fail();
        failed = __any_sync(0xffffffffu, failed);
        if (!failed) issue_q(it, qs);
      }
      q_pre = false;
      const bool want_next = C::QBUF == 2 && next < num_items;
      const int qn = (ring + 1) % C::QBUF;
      const uint32_t qn_par = (((ring + 1) / C::QBUF) & 1u) ^ 1u;
      const Item itn = (next < num_items) ? decode_item<C::PAIR, BN, C::NDH>(p, next) : it;
      const int nb = it.nblocks();
      if constexpr (C::SPLIT_KV) {
        // K(j) is requested when its stage's previous K has been read by S;
        // V(j) one block later, when its stage's previous V has been read by
        // P V.  A partial padded tile is cleared before the next stage wait.
        struct VJob {
          int row, h, b, map, st, valid;
          uint32_t ph;
          bool fix;
        };
        VJob pv{};
        bool have_pv = false;
        auto issue_v = [&](const VJob& vj) {
          resolve_fix();
          if (!mbar_wait(&bar->kv_empty[vj.st], vj.ph ^ 1u, abort_flag, tmo)) fail();
          failed = __any_sync(0xffffffffu, failed);
          uint8_t* tv = sV + vj.st * C::KV_BYTES;
          if (lane == 0 && !failed) {
            const CUtensorMap* mv = vj.map == 0 ? &tm_vc : &tm_v;
            uint64_t* vb = vj.fix ? &bar->fix : &bar->v_full[vj.st];
            mbar_arrive_expect_tx(vb, C::KV_BYTES);
            for (int s = 0; s < C::NSLAB; ++s)
              tma_load_4d(tv + s * (BN * SWB), mv, vb, s * C::SLAB_COLS, vj.row, vj.h, vj.b);
          }
          failed = __shfl_sync(0xffffffffu, failed, 0);
          if (vj.fix && !failed) {
            pend_tile = tv;
            pend_valid = vj.valid;
            pend_bar = &bar->v_full[vj.st];
          }
        };
        for (int j = 0; j < nb && !failed; ++j, ++fill) {
          int row;
          const Seg sgm = it.block_seg(j, BN, row);
          const CUtensorMap* mk = sgm.map == 0 ? &tm_kc : &tm_k;
          const int st = fill % STAGES;
          const uint32_t ph = (fill / STAGES) & 1u;
          const int valid = min(BN, sgm.row1 - row);
          const bool fix = sgm.fix && valid < BN;
          uint8_t* tk = sK + st * C::KV_BYTES;
          resolve_fix();
          if (!mbar_wait(&bar->k_empty[st], ph ^ 1u, abort_flag, tmo)) fail();
          failed = __any_sync(0xffffffffu, failed);
          if (lane == 0 && !failed) {
            FMLM_TR(40);
            // with MLA the K tile is also V: a partial padded one is cleared
            uint64_t* kb = (fix && mla) ? &bar->fix : &bar->k_full[st];
            mbar_arrive_expect_tx(kb, C::KV_BYTES);
            for (int s = 0; s < C::NSLAB; ++s)
              tma_load_4d(tk + s * (BN * SWB), mk, kb, s * C::SLAB_COLS, row, sgm.h, sgm.b);
          }
          failed = __shfl_sync(0xffffffffu, failed, 0);
          if (fix && mla && !failed) {
            pend_tile = tk;
            pend_valid = valid;
            pend_bar = &bar->k_full[st];
            resolve_fix();
          }
          if (!mla && !failed) {
            if (have_pv) issue_v(pv);
            pv = VJob{row, sgm.h, sgm.b, sgm.map, st, valid, ph, fix};
            have_pv = true;
          }
          if (want_next && !q_pre && !failed) {
            bool ready = false;
            if (lane == 0) ready = mbar_test_wait(smem_u32(&bar->q_empty[qn]), qn_par);
            if (__shfl_sync(0xffffffffu, ready, 0)) {
              issue_q(itn, qn);
              q_pre = true;
            }
          }
        }
        if (have_pv && !failed) issue_v(pv);
      } else {
        for (int j = 0; j < nb && !failed; ++j, ++fill) {
          {
            int row;
            const Seg sgm = it.block_seg(j, BN, row);
            const CUtensorMap* mk = sgm.map == 0 ? &tm_kc : &tm_k;
            const CUtensorMap* mv = sgm.map == 0 ? &tm_vc : &tm_v;
            const int st = fill % STAGES;
            const uint32_t ph = (fill / STAGES) & 1u;
            const int valid = min(BN, sgm.row1 - row);
            const bool fix = sgm.fix && valid < BN;
            uint8_t* tk = sK + st * C::KV_BYTES;
            uint8_t* tv = sV + st * C::KV_BYTES;
            resolve_fix();
            if (!mbar_wait(&bar->kv_empty[st], ph ^ 1u, abort_flag, tmo)) fail();
            const int ss = fill % 2;
            if constexpr (C::KSPLIT) {
              if (!mbar_wait(&bar->ks_empty[ss], ((fill / 2) & 1u) ^ 1u, abort_flag, tmo)) fail();
            }
            failed = __any_sync(0xffffffffu, failed);
            if (lane == 0) {
              FMLM_TR(40);
              if (!failed && C::KSPLIT) {
                // long ring: the half this item uses as V (columns dh*256...);
                // short ring: the other half, read only by S.
                const int hl = it.dh(), hs = 1 - it.dh();
                uint64_t* lb = fix ? &bar->fix : &bar->k_full[st];
                mbar_arrive_expect_tx(lb, C::KV_BYTES);
                for (int s = 0; s < C::KNSLAB; ++s)
                  tma_load_4d(tk + s * (BN * SWB), mk, lb, (hl * C::KNSLAB + s) * C::SLAB_COLS, row, sgm.h, sgm.b);
                uint8_t* ts = sKs + ss * C::KV_BYTES;
                mbar_arrive_expect_tx(&bar->v_full[ss], C::KV_BYTES);
                for (int s = 0; s < C::KNSLAB; ++s)
                  tma_load_4d(ts + s * (BN * SWB), mk, &bar->v_full[ss], (hs * C::KNSLAB + s) * C::SLAB_COLS, row, sgm.h,
                              sgm.b);
              } else if (!failed) {
                if (!(fix && mla)) {
                  mbar_arrive_expect_tx(&bar->k_full[st], C::KV_BYTES);
                  for (int s = 0; s < C::NSLAB; ++s)
                    tma_load_4d(tk + s * (BN * SWB), mk, &bar->k_full[st], s * C::SLAB_COLS, row, sgm.h, sgm.b);
                }
                if (fix) {
                  uint8_t* tf = mla ? tk : tv;
                  const CUtensorMap* mf = mla ? mk : mv;
                  mbar_arrive_expect_tx(&bar->fix, C::KV_BYTES);
                  for (int s = 0; s < C::NSLAB; ++s)
                    tma_load_4d(tf + s * (BN * SWB), mf, &bar->fix, s * C::SLAB_COLS, row, sgm.h, sgm.b);
                } else if (!mla) {
                  mbar_arrive_expect_tx(&bar->v_full[st], C::KV_BYTES);
                  for (int s = 0; s < C::NSLAB; ++s)
                    tma_load_4d(tv + s * (BN * SWB), mv, &bar->v_full[st], s * C::SLAB_COLS, row, sgm.h, sgm.b);
                }
              }
            }
            failed = __shfl_sync(0xffffffffu, failed, 0);
            if (want_next && !q_pre && !failed) {
              bool ready = false;
              if (lane == 0) ready = mbar_test_wait(smem_u32(&bar->q_empty[qn]), qn_par);
              if (__shfl_sync(0xffffffffu, ready, 0)) {
                issue_q(itn, qn);
                q_pre = true;
              }
            }
            if (fix && !failed) {
              pend_tile = mla ? tk : tv;
              pend_valid = valid;
              pend_bar = mla ? &bar->k_full[st] : &bar->v_full[st];
              // With MLA the cleared tile is K, which this item's last S (and so
              // the release of the Q buffer the next item waits for) needs.
              if (mla) resolve_fix();
            }
          }
        }
      }
      w = next;
      cur = itn;
      have_cur = next < num_items;
    }
    resolve_fix();
  } else if (warp >= C::MMA_WARP) {
    // ------------------------------------------------------------ MMA issuers
    // Warp MMA_WARP + t issues every tcgen05.mma of query tile t, so the two
    // tiles' dependency chains (waits, issue back-pressure) run side by side.
    // The whole warp waits (converged polling is several times cheaper than a
    // lone lane's); one elected lane issues.
    const int t = warp - C::MMA_WARP;
    constexpr uint32_t fmt = BF16 ? 1u : 0u;
    constexpr uint32_t idesc_qk = make_idesc_f16(fmt, 0, 0, BM, BN);
    constexpr uint32_t idesc_pv = make_idesc_f16(fmt, 0, 1, BM, C::DV);
    constexpr uint32_t layout = swizzle_code(SWB);
    const uint32_t sQ0 = smem_u32(sQ) + t * C::Q_BYTES, sKa = smem_u32(sK), sVa = smem_u32(sV), sKsa = smem_u32(sKs);
    uint32_t sQa = sQ0;  // this item's Q buffer
    const uint32_t tS_d = tmem_base + C::TM_S + t * BN;
    const uint32_t tO_d = tmem_base + C::TM_O + t * C::DV;
    const uint32_t tP_a = tmem_base + (C::SEP_P ? C::TM_P + t * (BN / 2) : C::TM_S + t * BN);
    const bool leader = elect_one();
    uint32_t p_ph = 0, o_empty_ph = 1, s_free_ph = 0, q1_ph = 0;
    uint32_t gb = 0;  // SDB: key blocks issued so far (S buffer gb & 1, its (gb >> 1)-th use)
    bool first_item = true;
    uint32_t fill = 0;

    // KSPLIT: K columns [0, 256) come from the long ring when dh == 0 and from
    // the short ring (slot ss) otherwise, columns [256, 512) the other way round.
    auto issue_s = [&](int st, uint32_t d_col = 0, int ss = 0, int dh = 0) {
      if (leader) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t slab = (kk * 32) / SWB, inrow = (kk * 32) % SWB;
          uint32_t kbase = sKa + st * C::KV_BYTES + slab * (BN * SWB);
          if constexpr (C::KSPLIT) {
            const int half = kk / (D / 32);
            const uint32_t kslab = slab - half * C::KNSLAB;
            kbase = (half == dh ? sKa + st * C::KV_BYTES : sKsa + ss * C::KV_BYTES) + kslab * (BN * SWB);
          }
          const uint64_t b = make_smem_desc(kbase + inrow, 16, 8 * SWB, layout);
          if (C::TQ && kk >= C::QS / 16) {
            umma_ts(tS_d + d_col, tmem_base + C::TM_Q1 + (kk - C::QS / 16) * 8, b, idesc_qk, 1u);
          } else {
            const uint64_t a = make_smem_desc(sQa + slab * (BM * SWB) + inrow, 16, 8 * SWB, layout);
            umma_ss(tS_d + d_col, a, b, idesc_qk, kk > 0 ? 1u : 0u);
          }
        }
      }
    };
    auto issue_pv = [&](int st, bool acc, int dh, uint32_t p_col = 0, int k_lo = 0, int k_hi = -1) {
      if (k_hi < 0) k_hi = BN / 16;
      if (leader) {
        // V columns [dh*DV, dh*DV + DV) start at slab dh*DV/SLAB_COLS of the tile.
        const uint32_t vbase = C::KSPLIT ? sKa + st * C::KV_BYTES  // the long ring holds exactly the V half
                               : (mla ? sKa : sVa) + st * C::KV_BYTES + (dh * C::DV / C::SLAB_COLS) * (BN * SWB);
#pragma unroll
        for (int kk = k_lo; kk < k_hi; ++kk) {
          const uint64_t b = make_smem_desc(vbase + kk * 16 * SWB, BN * SWB, 8 * SWB, layout);
          umma_ts(tO_d, tP_a + p_col + kk * 8, b, idesc_pv, (acc || kk > 0) ? 1u : 0u);
        }
      }
    };
    auto commit = [&](uint64_t* b) {
      if (leader) umma_commit(b);
      __syncwarp();
    };
    auto wait = [&](uint64_t* b, uint32_t ph) -> bool {
      if (!mbar_wait(b, ph, abort_flag, tmo)) fail();
      failed = __any_sync(0xffffffffu, failed);
      return !failed;
    };

    int w;
    Item it;
    for (uint32_t ring = 0; take_item(ring, w, it); ++ring) {
      const int nb = it.nblocks();
      const int qs = ring % C::QBUF;
      uint64_t* q_empty = &bar->q_empty[qs];
      sQa = sQ0 + qs * NQ * C::Q_BYTES;
      if (!wait(&bar->q_full[qs], (ring / C::QBUF) & 1u)) break;
      if (t == 0) FMLM_TR(34);
      if (it.qrows(t) == 0) {
        // This tile is empty for the item: release Q and every K/V stage in
        // order (after each fill has landed, so no release runs ahead).
        if (leader) mbar_arrive(q_empty);
        for (int j = 0; j < nb; ++j) {
          const int st = (fill + j) % STAGES;
          const uint32_t ph = ((fill + j) / STAGES) & 1u;
          if (!wait(&bar->k_full[st], ph)) break;
          if constexpr (C::SPLIT_KV) {
            if (leader) mbar_arrive(&bar->k_empty[st]);
            // the V stage is released only once this block's V has landed, so
            // the release cannot count toward the stage's previous use
            if (!mla && !wait(&bar->v_full[st], ph)) break;
          }
          if (leader) mbar_arrive(&bar->kv_empty[st]);
        }
        fill += nb;
        continue;
      }
      if constexpr (C::SDB) {
        // Order on the tensor pipe: S(0), S(1), PV(0), S(2), PV(1), ...
        // S(g+1) overwrites buffer (g+1) & 1, whose P(g-1) was read by PV(g-1),
        // issued in the previous iteration.  MLA only: V is the K tile.
        bool ok = true;
        for (int j = -1; j < nb && ok; ++j) {
          if (j + 1 < nb) {
            const uint32_t g1 = gb + j + 1;
            const int st1 = (fill + j + 1) % STAGES;
            if (!wait(&bar->k_full[st1], ((fill + j + 1) / STAGES) & 1u)) { ok = false; break; }
            const int ss1 = (fill + j + 1) % 2;
            if constexpr (C::KSPLIT) {
              if (!wait(&bar->v_full[ss1], ((fill + j + 1) / 2) & 1u)) { ok = false; break; }
            }
            if (j < 0) {
              // the softmax warps' copy of this item's Q columns [QS, D) into TMEM
              if (!wait(&bar->q1_full, q1_ph)) { ok = false; break; }
              q1_ph ^= 1u;
            }
            tc_fence_after();
            issue_s(st1, (g1 & 1u) * BN, ss1, it.dh());
            commit(&bar->s_full[g1 & 1u]);
            if constexpr (C::KSPLIT) commit(&bar->ks_empty[ss1]);
            FMLM_TR(32);
            if (j + 2 == nb) commit(q_empty);
          }
          if (j < 0) continue;
          const uint32_t g = gb + j, b = g & 1u;
          const int st = (fill + j) % STAGES;
          if (!wait(&bar->p_full[b], (g >> 1) & 1u)) { ok = false; break; }
          FMLM_TR(30);
          if (j == 0) {
            if (!wait(&bar->o_empty[0], o_empty_ph)) { ok = false; break; }
            o_empty_ph ^= 1u;
          }
          tc_fence_after();
          issue_pv(st, j > 0, it.dh(), b * BN);
          commit(&bar->pv_done[0]);
          commit(&bar->kv_empty[st]);
        }
        if (!ok) break;
        gb += nb;
        fill += nb;
        continue;
      }
      {
        const int st = fill % STAGES;
        if (!wait(&bar->k_full[st], (fill / STAGES) & 1u)) break;
        if (C::SEP_P && !first_item) {
          // the softmax's read of the previous item's last S (done long ago)
          if (!wait(&bar->s_free[t], s_free_ph)) break;
          s_free_ph ^= 1u;
        }
        first_item = false;
        if constexpr (C::TQ) {
          // the softmax warps' copy of this item's Q columns [QS, D) into TMEM
          if (!wait(&bar->q1_full, q1_ph)) break;
          q1_ph ^= 1u;
        }
        tc_fence_after();
        issue_s(st);
        commit(&bar->s_full[t]);
        if (C::SPLIT_KV && !mla) commit(&bar->k_empty[st]);
        if (nb == 1) commit(q_empty);
      }
      for (int j = 0; j < nb && !failed; ++j) {
        const int st = (fill + j) % STAGES;
        const int st1 = (fill + j + 1) % STAGES;
        const uint32_t ph = ((fill + j) / STAGES) & 1u;
        const uint32_t ph1 = ((fill + j + 1) / STAGES) & 1u;
        if constexpr (C::SEP_P) {
          // S_t(j+1) as soon as the softmax has read S_t(j) ...
          if (j + 1 < nb) {
            if (!wait(&bar->k_full[st1], ph1)) break;
            if (t == 0) FMLM_TR(36);
            if (!wait(&bar->s_free[t], s_free_ph)) break;
            if (t == 0) FMLM_TR(38);
            s_free_ph ^= 1u;
            tc_fence_after();
            issue_s(st1);
            commit(&bar->s_full[t]);
            if (C::SPLIT_KV && !mla) commit(&bar->k_empty[st1]);
            if (t == 0) FMLM_TR(32);
            if (j + 2 == nb) commit(q_empty);
          }
          // ... then O_t += P_t(j) V(j) once P_t(j) is in TMEM.
          if (!mla && !wait(&bar->v_full[st], ph)) break;
          if constexpr (C::SPLIT_PV) {
            // each half of P as soon as the softmax has stored it
            bool ok = true;
#pragma unroll
            for (int h = 0; h < 2 && ok; ++h) {
              if (!wait(&bar->p_full[h], p_ph)) { ok = false; break; }
              if (h == 0) FMLM_TR(30);
              if (h == 0 && j == 0) {
                if (!wait(&bar->o_empty[t], o_empty_ph)) { ok = false; break; }
                o_empty_ph ^= 1u;
              }
              tc_fence_after();
              issue_pv(st, j > 0, it.dh(), 0, h * (BN / 32), (h + 1) * (BN / 32));
              commit(&bar->pv_done[h]);
            }
            if (!ok) break;
            p_ph ^= 1u;
            commit(&bar->kv_empty[st]);
            if (C::SPLIT_KV && mla) commit(&bar->k_empty[st]);  // MLA: the K tile was also V
            continue;
          }
          if (!wait(&bar->p_full[t], p_ph)) break;
          p_ph ^= 1u;
          if (t == 0) FMLM_TR(30);
          if (j == 0) {
            if (!wait(&bar->o_empty[t], o_empty_ph)) break;
            o_empty_ph ^= 1u;
          }
          tc_fence_after();
          issue_pv(st, j > 0, it.dh());
          commit(&bar->pv_done[t]);
          commit(&bar->kv_empty[st]);
          if (C::SPLIT_KV && mla) commit(&bar->k_empty[st]);  // MLA: the K tile was also V
          if (t == 0) FMLM_TR(44);
        } else {
          if (!mla && !wait(&bar->v_full[st], ph)) break;
          if (!wait(&bar->p_full[t], p_ph)) break;
          p_ph ^= 1u;
          if (t == 0) FMLM_TR(30);
          if (j == 0) {
            if (!wait(&bar->o_empty[t], o_empty_ph)) break;
            o_empty_ph ^= 1u;
          }
          tc_fence_after();
          issue_pv(st, j > 0, it.dh());
          if (j + 1 < nb) {
            if (!wait(&bar->k_full[st1], ph1)) break;
            tc_fence_after();
            issue_s(st1);
            commit(&bar->s_full[t]);
            if (C::SPLIT_KV && !mla) commit(&bar->k_empty[st1]);
            if (t == 0) FMLM_TR(32);
          } else {
            commit(&bar->o_full[t]);
          }
          if (j + 2 == nb) commit(q_empty);
          commit(&bar->kv_empty[st]);
          if (C::SPLIT_KV && mla) commit(&bar->k_empty[st]);  // MLA: the K tile was also V
        }
      }
      fill += nb;
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int t = warp >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + C::TM_S + t * BN;
    const uint32_t tO = tmem_base + lane_off + C::TM_O + t * C::DV;
    const uint32_t tP = C::SEP_P ? tmem_base + lane_off + C::TM_P + t * (BN / 2) : tS;
    const float sl2 = p.scale_log2;
    const bool pos_scale = sl2 > 0.f;
    const float fac = pos_scale ? sl2 : 1.0f;
    uint32_t s_ph = 0, o_ph = 0, pv_ph = 0, tok_ph = 0;
    uint32_t pvh_ph0 = 0, pvh_ph1 = 0;  // SPLIT_PV: phases of pv_done[0] / pv_done[1]
    uint32_t gblk = 0;  // SDB: key blocks processed so far (same count as the MMA warp's)
    T* out = reinterpret_cast<T*>(p.out);
    // With two tiles the exp2 loops of the tiles alternate (a token passed
    // through exp_tok), so one tile's MUFU-bound loop overlaps the other's
    // max / TMEM / barrier latency instead of contending with it.  Measured:
    // 17% faster at head_dim 128; slower at 64, where one tile per CTA and
    // two CTAs per SM is used instead.
#ifndef FMLM_PINGPONG_D64
#define FMLM_PINGPONG_D64 0
#endif
    constexpr bool kPingPong = NQ == 2 && ((D >= 128 && FMLM_PINGPONG) || (D == 64 && FMLM_PINGPONG_D64));
    if (kPingPong && t == 1 && lane == 0) mbar_arrive(&bar->exp_tok[0]);

    int w;
    Item it;
    for (uint32_t ring = 0; take_item(ring, w, it); ++ring) {
      const int nrows = it.qrows(t);
      // Padded output: zero the rows of this tile past the sequence's valid
      // rows, and (tile NQ-1 of a sequence's last item) the padding rows after
      // the item, up to N.  Each row of [B, H, N, D] is written exactly once.
      auto zero_pad_rows = [&]() {
        if (it.zero_limit() == 0) return;
        T* obase = out + it.out_row0 * (long long)D + it.dh() * C::DV;
        auto zero_row = [&](int i) {
          uint4* dst = reinterpret_cast<uint4*>(obase + (long long)i * D);
#pragma unroll 4
          for (int q = 0; q < C::DV * 2 / 16; ++q) dst[q] = make_uint4(0, 0, 0, 0);
        };
        const int i0 = t * BM + row;
        if (row >= nrows && i0 < it.zero_limit()) zero_row(i0);
        if (t == NQ - 1)
          for (int i = NQ * BM + row; i < it.zero_limit(); i += BM) zero_row(i);
      };
      // (before the key loop, so nothing it needs stays live through it)
      zero_pad_rows();
      if (nrows == 0) continue;
      const bool row_valid = row < nrows;
      const bool pp = kPingPong && it.qrows0 > 0 && it.qrows1 > 0;
      float m = -INFINITY, l = 0.f;
      const int nb = it.nblocks();
      if constexpr (C::TQ) {
        // Q columns [QS, D) of this thread's row go to TMEM lane `row` as
        // packed pairs (the layout of a TMEM A operand).  Every MMA of the
        // previous item has completed (its epilogue waited for the last PV).
        constexpr int NW = (D - C::QS) / 2;  // 32-bit words per row
        const uint16_t* qrow = p.q_ptr + (long long)it.qb * p.q_sb + (long long)it.qh * p.q_sh +
                               (long long)(it.qrow0 + row) * p.q_sr + C::QS;
        const uint32_t tQ1 = tmem_base + lane_off + C::TM_Q1;
#pragma unroll
        for (int c0 = 0; c0 < NW; c0 += 64) {
          uint32_t qv[64];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint4 u = row_valid ? __ldg(reinterpret_cast<const uint4*>(qrow) + c0 / 4 + q) : make_uint4(0, 0, 0, 0);
            qv[4 * q] = u.x; qv[4 * q + 1] = u.y; qv[4 * q + 2] = u.z; qv[4 * q + 3] = u.w;
          }
          tmem_st_x64(tQ1 + c0, qv);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->q1_full);
      }
      {
        for (int j = 0; j < nb; ++j) {
          int brow;
          const Seg sgm = it.block_seg(j, BN, brow);
          int kvv = min(BN, sgm.row1 - brow);
          if (!row_valid) kvv = 0;
          const uint32_t g = gblk + j, sb = C::SDB ? (g & 1u) : 0u;
          const uint32_t tSb = tS + sb * BN, tPb = tP + sb * BN;  // SDB: S buffer g & 1, P over it
          if (!mbar_wait(&bar->s_full[C::SDB ? sb : t], C::SDB ? ((g >> 1) & 1u) : s_ph, abort_flag, tmo)) { fail(); }
          failed = __any_sync(0xffffffffu, failed);
          if (failed) break;
          FMLM_TR(10 + t);
          s_ph ^= 1u;
          tc_fence_after();
          uint32_t r[BN];
          if constexpr (BN == 128) tmem_ld_x128(tSb, r);
          else if constexpr (BN == 64) tmem_ld_x64(tSb, r);
          else if constexpr (BN == 48) tmem_ld_x48(tSb, r);
          else tmem_ld_x32(tSb, r);
          FMLM_TR(12 + t);
#ifndef FMLM_LATE_SFREE
#define FMLM_LATE_SFREE 0
#endif
          // S_t is in registers: the MMA warp may overwrite it with S_t(j+1).
          // (LATE_SFREE: signalled after the row max instead, so the signal's
          // latency overlaps the exponentials rather than preceding the max.)
          auto release_s = [&]() {
            if constexpr (C::SEP_P) {
#if !defined(FMLM_SFREE_NOFENCE)
              tc_fence_before();
#endif
              __syncwarp();
              if (lane == 0) mbar_arrive(&bar->s_free[t]);
            }
          };
          if (!FMLM_LATE_SFREE) release_s();
          // With a positive scale the row max is taken on raw scores and the
          // scale is folded into the exp2 argument (one FFMA per element);
          // otherwise scores are scaled first.
          if (!pos_scale) {
#pragma unroll
            for (int c = 0; c < BN; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * sl2);
          }
          if (kvv < BN) {
#pragma unroll
            for (int c = 0; c < BN; ++c)
              if (c >= kvv) r[c] = 0xff800000u;  // -inf
          }
          FMLM_TR(26 + t);
          float mx;
#if defined(FMLM_MAXMODE) && FMLM_MAXMODE == 2
          mx = (j == 0) ? 0.f : m / fac;  // timing experiment only: no max
          mx *= fac;
#elif defined(FMLM_MAXMODE) && FMLM_MAXMODE == 1
          {
            float m16[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) m16[i] = __uint_as_float(r[i]);
#pragma unroll
            for (int c = 16; c < BN; ++c) m16[c & 15] = fmaxf(m16[c & 15], __uint_as_float(r[c]));
#pragma unroll
            for (int w2 = 8; w2 > 0; w2 >>= 1)
#pragma unroll
              for (int i = 0; i < w2; ++i) m16[i] = fmaxf(m16[i], m16[i + w2]);
            mx = m16[0] * fac;
          }
#else
          {
            // 3-input max tree: BN/2 instructions in 8 independent chains.
            float m8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) m8[i] = __uint_as_float(r[i]);
#pragma unroll
            for (int c = 8; c + 1 < BN; c += 2) {
              const int k = (c >> 1) & 7;
              m8[k] = fmax3(m8[k], __uint_as_float(r[c]), __uint_as_float(r[c + 1]));
            }
            mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
            mx *= fac;  // -inf stays -inf (fac > 0)
          }
#endif
          // Move the reference max only when this block raises it by more than 2^8.
          bool need = false;
          float alpha = 1.0f;
          if (j == 0) {
            m = mx;
          } else if (mx > m + 8.0f) {
            need = true;
            alpha = ex2_approx(m - mx);
            l *= alpha;
            m = mx;
          }
          const float neg_mu = (m == -INFINITY) ? 0.f : -m;
          if (FMLM_LATE_SFREE) release_s();
          FMLM_TR(22 + t);
          if constexpr (C::SPLIT_PV) {
            // Half h of P(j) may be written once half h of P V(j-1) has read
            // P(j-1).  A rescale of O needs all of P V(j-1) first, and must
            // land before P V(j) starts (its first half is issued as soon as
            // half 0 of P(j) is stored), so it comes before the exponentials.
            bool waited0 = j == 0, waited1 = j == 0;
            auto wait_half = [&](int h) -> bool {
              uint32_t& ph = h == 0 ? pvh_ph0 : pvh_ph1;
              if (!mbar_wait(&bar->pv_done[h], ph, abort_flag, tmo)) fail();
              failed = __any_sync(0xffffffffu, failed);
              ph ^= 1u;
              tc_fence_after();
              return !failed;
            };
            const bool rescale = __any_sync(0xffffffffu, need);
            FMLM_TR(24 + t);
            float sums[4] = {0.f, 0.f, 0.f, 0.f};
            constexpr int HC = BN / 4;  // packed P columns per half
            bool ok = true;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (!(h == 0 ? waited0 : waited1) && !wait_half(h)) { ok = false; break; }
              if (h == 1) waited1 = true;
              uint32_t pk[HC];
#pragma unroll
              for (int cc = 0; cc < HC; ++cc) {
                const int c = h * HC + cc;
                const float x0 = fmaf(__uint_as_float(r[2 * c]), fac, neg_mu);
                const float x1 = fmaf(__uint_as_float(r[2 * c + 1]), fac, neg_mu);
                const float p0 = ex2_approx(x0);
                const float p1 = ex2_approx(x1);
                sums[(2 * c) & 3] += p0;
                sums[(2 * c + 1) & 3] += p1;
                if constexpr (BF16) {
                  __nv_bfloat162 v2 = __floats2bfloat162_rn(p0, p1);
                  pk[cc] = *reinterpret_cast<uint32_t*>(&v2);
                } else {
                  __half2 v2 = __floats2half2_rn(p0, p1);
                  pk[cc] = *reinterpret_cast<uint32_t*>(&v2);
                }
              }
              static_assert(HC == 32 || HC == 16, "SPLIT_PV half width");
              if constexpr (HC == 32) tmem_st_x32_nowait(tP + h * HC, pk);
              else tmem_st_x16_nowait(tP + h * HC, pk);
              if (h == 0 && rescale) {
                // O holds P V(0..j-1) once both halves of P V(j-1) are done;
                // it is rescaled before P V(j) (released by p_full[0]) starts.
                if (!waited1 && !wait_half(1)) { ok = false; break; }
                waited1 = true;
#pragma unroll
                for (int c0 = 0; c0 < C::DV; c0 += 16) {
                  uint32_t o[16];
                  tmem_ld_x16(tO + c0, o);
#pragma unroll
                  for (int c = 0; c < 16; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
                  tmem_st_x16(tO + c0, o);
                }
              }
              tmem_wait_st();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bar->p_full[h]);
            }
            if (!ok) break;
            l += (sums[0] + sums[1]) + (sums[2] + sums[3]);
            FMLM_TR(14 + t);
            FMLM_TR(16 + t);
            continue;
          }
          if constexpr (C::SEP_P) {
            // P_t and O_t are free once PV_t(j-1) has completed (almost always
            // by now); waiting first lets each half of P be stored as soon as
            // it is packed.
            if (j > 0) {
              if (!mbar_wait(&bar->pv_done[t], pv_ph, abort_flag, tmo)) fail();
              failed = __any_sync(0xffffffffu, failed);
              if (failed) break;
              pv_ph ^= 1u;
              tc_fence_after();
            }
          }
          FMLM_TR(24 + t);
          if (pp) {
            if (!mbar_wait(&bar->exp_tok[t], tok_ph, abort_flag, tmo)) fail();
            failed = __any_sync(0xffffffffu, failed);
            if (failed) break;
            tok_ph ^= 1u;
          }
          float sums[4] = {0.f, 0.f, 0.f, 0.f};
          // P in chunks of up to 32 packed columns (64 scores), each stored to
          // TMEM as soon as it is ready, so at most one chunk of packed P is live.
#ifndef FMLM_PCHUNK
#define FMLM_PCHUNK 32
#endif
          constexpr int PC = BN / 2 < FMLM_PCHUNK ? BN / 2 : FMLM_PCHUNK;
#pragma unroll
          for (int h0 = 0; h0 < BN / 2; h0 += PC) {
            uint32_t pk[PC];
#pragma unroll
            for (int cc = 0; cc < PC; ++cc) {
              const int c = h0 + cc;
              const float x0 = fmaf(__uint_as_float(r[2 * c]), fac, neg_mu);
              const float x1 = fmaf(__uint_as_float(r[2 * c + 1]), fac, neg_mu);
              // A share of the exponentials (pairs with cc % FMLM_POLY_EXP ==
              // FMLM_POLY_EXP - 1) runs on the FMA pipe, the rest on MUFU.
              const bool poly = C::POLY > 0 && (cc % (C::POLY > 0 ? C::POLY : 1)) == (C::POLY > 0 ? C::POLY : 1) - 1;
#if defined(FMLM_EXPMODE) && FMLM_EXPMODE == 1
              const float p0 = x0 * 1e-3f, p1 = x1 * 1e-3f;  // timing experiment only: no exponentials
#else
              const float p0 = poly ? ex2_poly(x0) : ex2_approx(x0);
              const float p1 = poly ? ex2_poly(x1) : ex2_approx(x1);
#endif
              sums[(2 * c) & 3] += p0;
              sums[(2 * c + 1) & 3] += p1;
              if constexpr (BF16) {
                __nv_bfloat162 v2 = __floats2bfloat162_rn(p0, p1);
                pk[cc] = *reinterpret_cast<uint32_t*>(&v2);
              } else {
                __half2 v2 = __floats2half2_rn(p0, p1);
                pk[cc] = *reinterpret_cast<uint32_t*>(&v2);
              }
            }
            if constexpr (PC == 32) tmem_st_x32_nowait(tPb + h0, pk);
            else if constexpr (PC == 24) tmem_st_x24_nowait(tPb + h0, pk);
            else if constexpr (PC == 16) tmem_st_x16_nowait(tPb + h0, pk);
            else tmem_st_x8_nowait(tPb + h0, pk);
          }
          if (pp) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar->exp_tok[t ^ 1]);
          }
          l += (sums[0] + sums[1]) + (sums[2] + sums[3]);
          FMLM_TR(14 + t);
          if (__any_sync(0xffffffffu, need)) {
            // O holds PV(0..j-1), all complete (aliased P: PV_t(j-1) was issued
            // before S_t(j); separate P: waited above; SDB: S(j) was issued
            // before PV(j-1), so PV(j-1) is waited for here); PV_t(j) waits
            // for p_full.
            if constexpr (C::SDB) {
              if (!mbar_wait(&bar->pv_done[0], (g - 1) & 1u, abort_flag, tmo)) fail();
              failed = __any_sync(0xffffffffu, failed);
              if (failed) break;
              tc_fence_after();
            }
#pragma unroll
            for (int c0 = 0; c0 < C::DV; c0 += OC) {
              uint32_t o[OC];
              tmem_ld_chunk(tO + c0, o);
#pragma unroll
              for (int c = 0; c < OC; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
              tmem_st_chunk(tO + c0, o);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bar->p_full[C::SDB ? sb : t]);
          FMLM_TR(16 + t);
        }
        if (failed) break;
      }
      if (failed) break;
      // epilogue: O / l  ->  global
      if constexpr (C::SDB) {
        const uint32_t gl = gblk + nb - 1;
        gblk += nb;
        if (!mbar_wait(&bar->pv_done[0], gl & 1u, abort_flag, tmo)) fail();
      } else if constexpr (C::SPLIT_PV) {
        if (!mbar_wait(&bar->pv_done[0], pvh_ph0, abort_flag, tmo)) fail();
        if (!mbar_wait(&bar->pv_done[1], pvh_ph1, abort_flag, tmo)) fail();
        pvh_ph0 ^= 1u;
        pvh_ph1 ^= 1u;
      } else if constexpr (C::SEP_P) {
        if (!mbar_wait(&bar->pv_done[t], pv_ph, abort_flag, tmo)) fail();
        pv_ph ^= 1u;
      } else {
        if (!mbar_wait(&bar->o_full[t], o_ph, abort_flag, tmo)) fail();
        o_ph ^= 1u;
      }
      failed = __any_sync(0xffffffffu, failed);
      if (failed) break;
      FMLM_TR(18 + t);
      tc_fence_after();
      const float inv = (l > 0.f) ? 1.0f / l : 1.0f;
      T* orow = out + (it.out_row0 + t * BM + row) * (long long)D + it.dh() * C::DV;
      auto store_chunk = [&](const uint32_t(&o)[OC], int c0) {
        if (!row_valid) return;
        uint32_t v[OC / 2];
#pragma unroll
        for (int c = 0; c < OC / 2; ++c) {
          const float a = __uint_as_float(o[2 * c]) * inv, b = __uint_as_float(o[2 * c + 1]) * inv;
          if constexpr (BF16) {
            __nv_bfloat162 v2 = __floats2bfloat162_rn(a, b);
            v[c] = *reinterpret_cast<uint32_t*>(&v2);
          } else {
            __half2 v2 = __floats2half2_rn(a, b);
            v[c] = *reinterpret_cast<uint32_t*>(&v2);
          }
        }
        uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
        for (int q = 0; q < OC / 8; ++q) dst[q] = make_uint4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      };
      if constexpr (C::DV <= 64 && FMLM_EARLY_O) {
        // Small O: read all of it, hand TMEM back to the MMA warp (the next
        // item's first PV may start), then normalise and store.
        uint32_t o[C::DV / OC][OC];
#pragma unroll
        for (int k = 0; k < C::DV / OC; ++k) tmem_ld_chunk(tO + k * OC, o[k]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->o_empty[t]);
#pragma unroll
        for (int k = 0; k < C::DV / OC; ++k) store_chunk(o[k], k * OC);
      } else {
#pragma unroll 4
        for (int c0 = 0; c0 < C::DV; c0 += OC) {
          uint32_t o[OC];
          tmem_ld_chunk(tO + c0, o);
          store_chunk(o, c0);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bar->o_empty[t]);
      }
      FMLM_TR(20 + t);
    }
  }

  // ------------------------------------------------------------ teardown
#ifdef FMLM_TRACE
  if (tr_role >= 0) {
    if (kTraceGlobal) p.trace[tr_role] = tr_n;
    else tr_cnt[tr_role] = tr_n;
  }
#endif
  tc_fence_before();
  __syncthreads();
#ifdef FMLM_TRACE
  if (p.trace && threadIdx.x == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    p.trace[8192 + 3 * blockIdx.x] = tr_entry_ns;
    p.trace[8192 + 3 * blockIdx.x + 1] = global_timer_ns();
    p.trace[8192 + 3 * blockIdx.x + 2] = smid;
  }
  if (!kTraceGlobal && kTraceSlots > 0 && p.trace && blockIdx.x == 0) {
    for (int r = 0; r < 4; ++r) {
      const int n = tr_cnt[r];
      if (threadIdx.x == 0) p.trace[r] = (unsigned long long)n;
      for (int i = threadIdx.x; i < n; i += blockDim.x) p.trace[4 + r * kTraceSlots + i] = tr_buf[r * kTraceSlots + i];
    }
  }
#endif
  if (p.mode == 1 && threadIdx.x == 0) {
    // The last CTA to finish re-arms the item counter for the next launch.
    __threadfence();
    if (atomicAdd(p.work + 2, 1) == (int)gridDim.x - 1) {
      atomicExch(p.work + 1, 0);
      atomicExch(p.work + 2, 0);
    }
  }
  tc_fence_after();
  if (warp == C::MMA_WARP) {
    if (*abort_flag) {
      // Give in-flight MMAs a bounded chance to retire before freeing TMEM.
      const uint64_t t0 = global_timer_ns();
      while (global_timer_ns() - t0 < 1000000ull) {}
    }
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace fmlm
