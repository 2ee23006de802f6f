// sm_100a forward attention with additive relative-position terms.
//
// One kernel template serves both reference operators:
//   * kT5      — kernels/flash_attention_rpb.py:62-230 (_flash_attn_rpb_fwd_kernel_final):
//                s = scale * q.k + rpb_table[bucket(n - m), h] + padding_mask[b, h, n]
//   * kDeberta — kernels/flash_deberta_attention.py:145-299 (_flash_deberta_fwd_kernel):
//                s = sm_scale * (q.k + pos_key[m, idx(m - n)] + pos_query[n, idx(m - n)])
//     kT5 also runs over a packed batch (KParams::cu_seqlens set): sequence b is rows
//     [cu_seqlens[b], cu_seqlens[b+1]) of q/k/v/out and attends only within itself (no
//     counterpart in the reference, which pads; no mask)
//
// Persistent launch: one CTA per SM walks a list of work units; a unit is 256 query rows
// of one (batch, head) as two 128-row tiles, against that batch's live 128-key tiles.
// Warp roles (384 threads = 3 warpgroups):
//   warps 0-3  softmax group 0 (query tile 0), one thread per query row
//   warps 4-7  softmax group 1 (query tile 1)
//   warp  8    TMA producer (Q per unit and a K/V ring across units; depths per variant, Smem<>)
//   warp  9    UMMA issuer (one elected lane) + TMEM allocation
//   warp  10   unit preparation (schedule, live key span, per-head bias table), one unit ahead
//   warp  11   UMMA issuer for group 1 (warp 9 then serves group 0)
// Register split after the prologue: kRegsSoftmax / kRegsProducer (T5), kRegsSoftmaxDeberta /
// kRegsProducerDeberta.
// TMEM (512 columns, fp32): per query tile g, S at 256g, P (bf16 pairs) at 256g+128,
// O at 256g+192.  S = Q K^T and O += P V run on tcgen05.mma (kind::f16, fp32 accumulate);
// softmax threads read S with tcgen05.ld, write P back with tcgen05.st, and the PV MMA
// takes P straight from TMEM.  O leaves through a shared-memory staging tile and a TMA
// bulk store.  All waits are bounded (see vf_ptx.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <type_traits>
#include <vector>

#include "vf_ptx.cuh"
#include "vf_internal.h"
#include "../../include/vf_b200.h"

namespace vf {

constexpr int kBM = 128;          // query rows per tile
constexpr int kNQ = 2;            // query tiles per work unit (softmax groups per CTA)
constexpr int kBN = 128;          // keys per tile
constexpr int kHeadDim = 64;
constexpr int kTileBytes = kBM * kHeadDim * 2;   // 16 KB for a 128 x 64 16-bit tile
constexpr int kSoftmaxWarps = 4 * kNQ;
constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
constexpr int kThreads = kSoftmaxThreads + 128;
// Launched at 168 registers/thread; after the prologue the producer warpgroup drops to
// 88 and the softmax warpgroups rise to 208 (2*128*208 + 128*88 = 384*168).  The softmax
// path fits in 208 without spills; the producer roles (loader, UMMA issuer, unit
// preparation) are latency-critical and get the rest.
constexpr uint32_t kRegsSoftmax = 208;
constexpr uint32_t kRegsProducer = 88;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsProducer == 384 * 168, "setmaxnreg split must use the launch budget");
// DeBERTa: its softmax warps hold the gathers in flight, its producer warps do little
// (measured on C1 / a C3-sized packed layer: 232/40 is 3-5 % faster than 208/88).
constexpr uint32_t kRegsSoftmaxDeberta = 232;
constexpr uint32_t kRegsProducerDeberta = 40;
static_assert(2 * 128 * kRegsSoftmaxDeberta + 128 * kRegsProducerDeberta == 384 * 168,
              "setmaxnreg split must use the launch budget");
constexpr int kLoadWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;
constexpr int kPrepWarp = kSoftmaxWarps + 2;
constexpr int kMmaWarp2 = kSoftmaxWarps + 3;
#ifndef VF_MMA_ISSUERS
#define VF_MMA_ISSUERS 2
#endif
// UMMA issuing warps: 2 = one per softmax group (warps 9 and 11), so neither group's
// MMAs wait behind the other's in one instruction stream; 1 = warp 9 issues for both.
constexpr int kMmaIssuers = VF_MMA_ISSUERS;
constexpr uint32_t kTmemCols = 256 * kNQ;
constexpr int kMaxRel = 1024;               // relative-position table radius limit
constexpr int kMaxLut = 2 * kMaxRel + 1;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kDeadMask = -1.0e4f;        // additive mask at/below this kills a key
constexpr float kMaskFloor = -1.0e30f;      // masks are clamped here before scaling
#ifndef VF_RESCALE_BF16
#define VF_RESCALE_BF16 32.0f
#endif
constexpr int kPolyEvery = 3;               // every 3rd exponential pair on the FMA pipe

enum Variant : int { kT5 = 0, kDeberta = 1 };

struct __align__(64) KParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_o;
  void* out;
  long long o_sb, o_sh, o_sm;
  int B, H, M, N;
  float scale_log2;      // softmax scale * log2(e)
  int causal;
  int rel_R;             // lut covers relative positions [-rel_R, rel_R]
  // T5 bias
  const void* table;
  long long tb_srow, tb_scol;
  int table_dtype;
  const void* mask;
  long long mk_sb, mk_sh, mk_sn;
  int mask_dtype;
  // T5 mask that varies over query rows (additive, [B|1, H|1, M, N]; the kernel instance
  // with kQMask reads it per score; `mask` is then null and mask_dtype gives its type)
  const void* qmask;
  long long qm_sb, qm_sh, qm_sm, qm_sn;
  int qmask_vec;         // 16-bit, unit column stride, 16-byte aligned rows: 16-byte loads
  // DeBERTa positions
  const void* pos_key;
  long long pk_sb, pk_sh, pk_sm, pk_sk;
  const void* pos_query;
  long long pq_sb, pq_sh, pq_sn, pq_sk;
  const int* seq_lengths;
  // Packed variable-length batch (T5): sequence b is rows [cu_seqlens[b], cu_seqlens[b+1])
  // of the single packed "batch" of the q/k/v/out views; B = number of sequences and
  // M = N = the longest sequence.  nullptr: padded (B, H, L, D) layout.
  const int* cu_seqlens;
  int packed_rows;       // rows of the packed views (bound of every cu_seqlens entry)
  int p_seq;             // N - M (causal offset)
  int span2;             // 2 * ATT_SPAN, bound of the position index
  short lut[kMaxLut];    // T5: bucket of r = n - m;  DeBERTa: idx of r = m - n
};

constexpr int kRPad = 160;                  // bias-table padding: a warp's window never clamps
constexpr int kRBiasLen = (kMaxLut + 2 * kRPad + 3) & ~3;
constexpr int kMaxLptPairs = 1024;          // (batch, query block) pairs ordered by cost
constexpr int kMaxLptSamples = 2048;        // T5 mask samples (batch x key tile) for the costs

// Pipeline depths and shared-memory carve-up (offsets from a 1024-aligned base) per variant.
// T5: Q double-buffered by unit, a 3-stage K/V ring across units, the bias table by unit.
// DeBERTa: one Q buffer and a 2-stage ring.  Its time goes to the position-term gathers,
// which are served by the L1 cache that shares the SM's 256 KB with shared memory: this
// carve-up (~139 KB with the static part) leaves ~92 KB of L1 where the T5 depths
// (~203 KB) left ~28 KB.  Each group stages its O tile for the bulk store.
template <int kVariant>
struct Smem {
  static constexpr int kQBuf = kVariant == kDeberta ? 1 : 2;   // Q buffers (units)
  static constexpr int kKV = kVariant == kDeberta ? 2 : 3;     // K/V ring stages (>= 2)
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBuf * kNQ * kTileBytes;
  static constexpr int kOffV = kOffK + kKV * kTileBytes;
  static constexpr int kOffOStage = kOffV + kKV * kTileBytes;
  static constexpr int kOffKBias = kOffOStage + kNQ * kTileBytes;
  static constexpr int kOffKZero = kOffKBias + kKV * kBN * 4;    // per stage: key mask all zero
  static constexpr int kOffZeroRow = kOffKZero + 16;             // kBN zero floats
  static constexpr int kOffLut = kOffZeroRow + kBN * 4;
  static constexpr int kOffBar = (kOffLut + kMaxLut * 2 + 15) & ~15;
  // barriers: q_full[2], q_empty[2], s_full[2], p_full[2], s_consumed[2], pv_done[2],
  // info_full[2], info_empty[2], stage_free[2], stage_full[2], k_full/v_full/kv_empty[kKV],
  // drain
  static constexpr int kNumBars = 20 + 3 * kKV + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kOffInfo = kOffMisc + 16;
  static constexpr int kOffOrder = kOffInfo + 2 * 64;              // uint16_t[kMaxLptPairs]
  static constexpr int kOffCost = kOffOrder + 2 * kMaxLptPairs;    // uint8_t[kMaxLptPairs]
  // T5-only tables last: the DeBERTa kernel requests shared memory up to kOffLive only.
  static constexpr int kOffLive = kOffCost + kMaxLptPairs;                 // uint8_t[kMaxLptSamples]
  static constexpr int kOffRBias = (kOffLive + kMaxLptSamples + 15) & ~15;  // float[2][kRBiasLen]
  static constexpr int kBytes = kVariant == kDeberta ? kOffLive : kOffRBias + 2 * kRBiasLen * 4;
  static constexpr int kAlloc = kBytes + 1024;
};
template <int kVariant> constexpr int smem_alloc() { return Smem<kVariant>::kAlloc; }

// Slot and phase parity of use i of an N-deep ring of buffers and barriers.
template <int N> __device__ __forceinline__ int ring_slot(int i) { return N == 1 ? 0 : (N == 2 ? (i & 1) : i % N); }
template <int N> __device__ __forceinline__ uint32_t ring_parity(int i) {
  return N == 1 ? (i & 1) : (N == 2 ? ((i >> 1) & 1) : (i / N) & 1);
}

struct SmemMisc {
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(Smem<kT5>::kAlloc <= 227 * 1024 && Smem<kDeberta>::kAlloc <= 227 * 1024,
              "shared memory over the per-CTA limit");

// One zero position value: the gather of a missing DeBERTa position term reads it with
// stride 0 (read-only; never written).
__device__ const uint16_t g_zero_pos = 0;

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

__device__ __forceinline__ float load_any(const void* p, long long off, int dtype) {
  if (dtype == VF_DTYPE_F32) return __ldg(reinterpret_cast<const float*>(p) + off);
  if (dtype == VF_DTYPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[off]);
  return __half2float(reinterpret_cast<const __half*>(p)[off]);
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <> __device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }

// Lazy-rescale threshold (log2 units): P = 2^(x - m_run) stays below 2^(threshold + 1).
// bf16 has the fp32 exponent range; fp16 P must stay well inside 65504.
template <typename T> struct RescaleThreshold;
template <> struct RescaleThreshold<__nv_bfloat16> { static constexpr float value = VF_RESCALE_BF16; };
template <> struct RescaleThreshold<__half> { static constexpr float value = 8.0f; };
template <typename T> struct AbFormat;
template <> struct AbFormat<__nv_bfloat16> { static constexpr uint32_t value = 1u; };
template <> struct AbFormat<__half> { static constexpr uint32_t value = 0u; };

template <typename M> __device__ __forceinline__ float ld_f(const M* p) { return to_f<M>(p[0]); }
template <> __device__ __forceinline__ float ld_f<float>(const float* p) { return __ldg(p); }

// Live span of one mask row (additive mask > kDeadMask), per lane; eight loads in flight.
template <typename M>
__device__ __forceinline__ void live_span(const void* mask, long long base, long long stride, int N, int lane,
                                          int& lo, int& hi) {
  const M* row = reinterpret_cast<const M*>(mask) + base;
  for (int n0 = 0; n0 < N; n0 += 8 * 32) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = n0 + lane + 32 * j;
      v[j] = n < N ? ld_f<M>(row + n * stride) : -INFINITY;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (v[j] > kDeadMask) {
        const int n = n0 + lane + 32 * j;
        lo = min(lo, n);
        hi = max(hi, n);
      }
    }
  }
}

__device__ __forceinline__ float half_bits_to_f(uint32_t u, bool is_bf16) {
  return is_bf16 ? __uint_as_float(u << 16) : __half2float(__ushort_as_half(static_cast<unsigned short>(u)));
}

// Same for a contiguous 16-bit mask row starting on a 16-byte boundary: 8 values per
// 16-byte load, four loads in flight per lane.
__device__ __forceinline__ void live_span_vec16(const void* mask, long long base, int N, bool is_bf16, int lane,
                                                int& lo, int& hi) {
  const uint16_t* row = reinterpret_cast<const uint16_t*>(mask) + base;
  const uint4* vrow = reinterpret_cast<const uint4*>(row);
  const int nvec = N / 8;
  for (int c0 = 0; c0 < nvec; c0 += 4 * 32) {
    uint4 w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + lane + 32 * j;
      w[j] = c < nvec ? __ldg(vrow + c) : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + lane + 32 * j;
      if (c >= nvec) continue;
      const uint32_t ws[4] = {w[j].x, w[j].y, w[j].z, w[j].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int n = 8 * c + 2 * q;
        if (half_bits_to_f(ws[q] & 0xffffu, is_bf16) > kDeadMask) { lo = min(lo, n); hi = max(hi, n); }
        if (half_bits_to_f(ws[q] >> 16, is_bf16) > kDeadMask) { lo = min(lo, n + 1); hi = max(hi, n + 1); }
      }
    }
  }
  for (int n = 8 * nvec + lane; n < N; n += 32) {
    if (half_bits_to_f(row[n], is_bf16) > kDeadMask) { lo = min(lo, n); hi = max(hi, n); }
  }
}

// rbias[r + R + kRPad] = table[bucket(r), h] * log2(e) for r in [-R - kRPad, R + kRPad];
// beyond +-R the bucket is saturated, so the padding repeats the end values.
template <typename M>
__device__ __forceinline__ void fill_bias(const KParams& p, const short* lut_s, float* rb, int h, int lane) {
  const M* tab = reinterpret_cast<const M*>(p.table) + (long long)h * p.tb_scol;
  const int n = 2 * (p.rel_R + kRPad) + 1;
  for (int e0 = 0; e0 < n; e0 += 8 * 32) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + lane + 32 * j;
      const int rc = min(max(e - kRPad, 0), 2 * p.rel_R);
      v[j] = e < n ? ld_f<M>(tab + (long long)lut_s[rc] * p.tb_srow) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + lane + 32 * j;
      if (e < n) rb[e] = v[j] * kLog2e;
    }
  }
}

// One work unit: kNQ * kBM query rows of one (batch, head) against that batch's live key
// tiles.  Units are ordered by estimated cost, longest first, and dealt to the CTAs in
// snake order (c, 2G-1-c, 2G+c, ...), so every CTA ends up with a similar amount of work.
struct UnitInfo {
  int valid;             // 0: the CTA's work list has ended
  int b, h, q0;
  int t_begin, nkv;      // key tiles [t_begin, t_begin + nkv)
  int klen, qlen;        // valid keys / rows (DeBERTa seq_len; T5: N and M, or the sequence)
};
// The packed layout's first row of the unit's sequence sits beside the slots, in its own
// int[2] (a larger UnitInfo costs the softmax warps registers).
constexpr int kOffInfoRow0 = 96;
static_assert(2 * sizeof(UnitInfo) <= kOffInfoRow0, "unit slots");

// Rows of sequence b: valid keys / query rows and the first row in the tensor views.
// Padded layout: every row of batch b (DeBERTa: up to seq_len), from row 0.  Packed layout:
// the cu_seqlens range of the views' single batch.
struct SeqGeo {
  int klen, qlen, row0;
};
template <int kVariant>
__device__ __forceinline__ SeqGeo seq_geo(const KParams& p, int b) {
  SeqGeo s{p.N, p.M, 0};
  if (kVariant == kDeberta && p.seq_lengths != nullptr) {
    const int L = __ldg(p.seq_lengths + b);
    s.klen = min(max(L, 0), p.N);
    s.qlen = min(max(L, 0), p.M);
  }
  if (p.cu_seqlens != nullptr) {
    // Offsets outside [0, packed_rows], decreasing offsets or a sequence longer than
    // max_seqlen set the error word; the rows used are clamped into the views either way.
    const int r0 = __ldg(p.cu_seqlens + b), r1 = __ldg(p.cu_seqlens + b + 1);
    if (r0 < 0 || r1 < r0 || r1 > p.packed_rows || r1 - r0 > p.M) atomicOr(&g_vf_error, kErrBadInput);
    const int lo = min(max(r0, 0), p.packed_rows);
    const int L = min(min(max(r1, lo), p.packed_rows) - lo, p.M);
    s.klen = s.qlen = L;
    s.row0 = lo;
  }
  return s;
}

// Whether the CTA orders its units by cost: the (batch, query block) pairs and, for a
// T5 mask, the (batch, key tile) mask samples must fit the shared-memory tables.
template <int kVariant>
__device__ __forceinline__ bool lpt_enabled(const KParams& p) {
  const int nqb = (p.M + kNQ * kBM - 1) / (kNQ * kBM);
  const int ntile = (p.N + kBN - 1) / kBN;
  if ((long long)p.B * nqb > kMaxLptPairs) return false;
  if (kVariant == kT5 && p.mask != nullptr && (long long)p.B * ntile > kMaxLptSamples) return false;
  return true;
}

// Estimated key tiles of the units of (batch b, query block qb): seq_len for DeBERTa, the
// mask sampled at each tile's first key for T5 (`live`, exact for contiguous padding;
// only the schedule depends on it), trimmed by causality.
template <int kVariant>
__device__ int pair_cost(const KParams& p, const uint8_t* live, int b, int qb) {
  const int q0 = qb * (kNQ * kBM);
  const SeqGeo sg = seq_geo<kVariant>(p, b);
  const int klen = sg.klen, qlen = sg.qlen;
  if ((kVariant == kDeberta || p.cu_seqlens != nullptr) && q0 >= qlen) return 0;
  int t_end = (klen + kBN - 1) / kBN;
  if (p.causal) {
    const int last_key = min(q0 + kNQ * kBM, qlen) - 1 + p.p_seq;
    t_end = min(t_end, last_key < 0 ? 0 : last_key / kBN + 1);
  }
  int n = t_end;
  if (kVariant == kT5 && p.mask != nullptr) {
    const int ntile = (p.N + kBN - 1) / kBN;
    n = 0;
    for (int kt = 0; kt < t_end; ++kt) n += live[b * ntile + kt];
    if (n == 0) n = t_end;   // every key dead: every tile is visited
  }
  return n;
}

// Unit i of this CTA.  `order` lists the (batch, query block) pairs by cost, longest
// first (nullptr: natural order); each pair stands for H units, one per head.
__device__ __forceinline__ bool unit_coords(const KParams& p, const uint16_t* order, int i, int& b, int& h,
                                            int& q0) {
  const int nqb = (p.M + kNQ * kBM - 1) / (kNQ * kBM);
  const long long G = gridDim.x;
  const long long k = (long long)i * G + ((i & 1) ? G - 1 - blockIdx.x : blockIdx.x);
  if (k >= (long long)p.H * nqb * p.B) return false;
  const int pair_rank = static_cast<int>(k / p.H);
  h = static_cast<int>(k % p.H);
  const int pair = order != nullptr ? order[pair_rank] : pair_rank;
  b = pair / nqb;
  q0 = (pair % nqb) * (kNQ * kBM);
  return true;
}

template <int kVariant, typename T, bool kQMask = false>
__global__ void __launch_bounds__(kThreads, 1) attn_fwd_kernel(const __grid_constant__ KParams p) {
  using S = Smem<kVariant>;
  constexpr int KV = S::kKV, QB = S::kQBuf;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* kbias = reinterpret_cast<float*>(smem + S::kOffKBias);
  float* rbias_buf = reinterpret_cast<float*>(smem + S::kOffRBias);   // [2][kRBiasLen], index r + R + kRPad
  int* kzero = reinterpret_cast<int*>(smem + S::kOffKZero);
  float* zero_row = reinterpret_cast<float*>(smem + S::kOffZeroRow);
  short* lut_s = reinterpret_cast<short*>(smem + S::kOffLut);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kOffBar);
  uint64_t* q_full = bars + 0;        // [2] Q tiles of a unit are in shared memory
  uint64_t* q_empty = bars + 2;       // [2] every QK reading that Q buffer has completed
  uint64_t* s_full = bars + 4;        // [2] S = Q K^T of the tile is in TMEM
  uint64_t* p_full = bars + 6;        // [2] P of the tile is in TMEM
  uint64_t* s_consumed = bars + 8;    // [2] softmax has read S into registers
  uint64_t* pv_done = bars + 10;      // [2] O += P V of the tile has completed
  uint64_t* info_full = bars + 12;    // [2] unit description and bias table published
  uint64_t* info_empty = bars + 14;   // [2] every role is done with that unit slot
  uint64_t* stage_free = bars + 16;   // [2] the group's previous O store has read its staging tile
  uint64_t* stage_full = bars + 18;   // [2] the group's O rows are staged for the store
  uint64_t* k_full = bars + 20;       // [KV]
  uint64_t* v_full = k_full + KV;
  uint64_t* kv_empty = v_full + KV;
  uint64_t* drain = kv_empty + KV;
  SmemMisc* misc = reinterpret_cast<SmemMisc*>(smem + S::kOffMisc);
  UnitInfo* info = reinterpret_cast<UnitInfo*>(smem + S::kOffInfo);   // [2]
  int* info_row0 = reinterpret_cast<int*>(smem + S::kOffInfo + kOffInfoRow0);   // [2]
  volatile int* abort_flag = &misc->abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int R = p.rel_R;
  const bool has_mask = (kVariant == kT5) && (p.mask != nullptr);

  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], kMmaIssuers);
      mbar_init(&info_full[s], 32);
      mbar_init(&info_empty[s], kSoftmaxThreads + 1 + kMmaIssuers);
      mbar_init(&stage_free[s], 1);
      mbar_init(&stage_full[s], kBM);
    }
    for (int g = 0; g < kNQ; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], kBM);
      mbar_init(&s_consumed[g], kBM);
      mbar_init(&pv_done[g], 1);
    }
    for (int s = 0; s < KV; ++s) {
      mbar_init(&k_full[s], has_mask ? 2 : 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], kMmaIssuers);
    }
    mbar_init(drain, kMmaIssuers);
    misc->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&misc->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kLoadWarp && lane == 0) {
    tma_prefetch_desc(&p.tm_q);
    tma_prefetch_desc(&p.tm_k);
    tma_prefetch_desc(&p.tm_v);
    tma_prefetch_desc(&p.tm_o);
  }
  // Relative-position lookup table (the same for every unit).
  for (int i = tid; i <= 2 * R; i += kThreads) lut_s[i] = p.lut[i];
  if (tid < kBN) zero_row[tid] = 0.f;
  // T5 mask samples for the unit costs (one load per thread for typical sizes).
  if (has_mask && lpt_enabled<kVariant>(p)) {
    uint8_t* live = smem + S::kOffLive;
    const int ntile = (p.N + kBN - 1) / kBN;
    for (int it = tid; it < p.B * ntile; it += kThreads) {
      const int b = it / ntile, kt = it % ntile;
      live[it] = load_any(p.mask, b * p.mk_sb + (long long)kt * kBN * p.mk_sn, p.mask_dtype) > kDeadMask ? 1 : 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc->tmem_base;

  if (warp >= kSoftmaxWarps) {
  reg_dealloc<kVariant == kDeberta ? kRegsProducerDeberta : kRegsProducer>();
  if (warp == kPrepWarp) {
    // ------------------------------------------------------------ unit preparation
    // Describes unit i in slot i & 1: live key range (mask scan), and for T5 the bias
    // table of the unit's head.  Runs one unit ahead of the other roles.
    uint16_t* order = reinterpret_cast<uint16_t*>(smem + S::kOffOrder);
    uint8_t* cost = smem + S::kOffCost;
    const int nqb = (p.M + kNQ * kBM - 1) / (kNQ * kBM);
    const bool lpt = lpt_enabled<kVariant>(p);
    if (lpt) {
      // Stable counting sort of the pairs by estimated cost, descending.
      const int P = p.B * nqb;
      const uint8_t* live = smem + S::kOffLive;
      int maxc = 0;
      for (int pi = lane; pi < P; pi += 32) {
        const int c = min(pair_cost<kVariant>(p, live, pi / nqb, pi % nqb), 255);
        cost[pi] = static_cast<uint8_t>(c);
        maxc = max(maxc, c);
      }
      maxc = __reduce_max_sync(0xffffffffu, maxc);
      __syncwarp();
      int pos = 0;
      for (int c = maxc; c >= 0; --c) {
        for (int base = 0; base < P; base += 32) {
          const int pi = base + lane;
          const bool match = pi < P && cost[pi] == c;
          const uint32_t ballot = __ballot_sync(0xffffffffu, match);
          if (match) order[pos + __popc(ballot & ((1u << lane) - 1u))] = static_cast<uint16_t>(pi);
          pos += __popc(ballot);
        }
      }
      __syncwarp();
    }
    for (int i = 0;; ++i) {
      const int slot = i & 1;
      if (i >= 2) {
        const bool ok = mbar_wait(&info_empty[slot], ((i - 2) >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      int b = 0, h = 0, q0 = 0;
      const bool valid = unit_coords(p, lpt ? order : nullptr, i, b, h, q0);
      int klen = p.N, qlen = p.M, t_begin = 0, t_end = 0, row0 = 0;
      if (valid) {
        const SeqGeo sg = seq_geo<kVariant>(p, b);
        klen = sg.klen;
        qlen = sg.qlen;
        row0 = sg.row0;
        t_end = (klen + kBN - 1) / kBN;
        if (has_mask) {
          // The span of keys whose mask is alive bounds the key tiles worth visiting.
          int lo = 0x7fffffff, hi = -1;
          const long long base = b * p.mk_sb + h * p.mk_sh;
          const bool vec16 = p.mask_dtype != VF_DTYPE_F32 && p.mk_sn == 1 &&
                             ((reinterpret_cast<uintptr_t>(p.mask) + base * 2) & 15) == 0;
          if (vec16)
            live_span_vec16(p.mask, base, p.N, p.mask_dtype == VF_DTYPE_BF16, lane, lo, hi);
          else if (p.mask_dtype == VF_DTYPE_BF16)
            live_span<__nv_bfloat16>(p.mask, base, p.mk_sn, p.N, lane, lo, hi);
          else if (p.mask_dtype == VF_DTYPE_F16)
            live_span<__half>(p.mask, base, p.mk_sn, p.N, lane, lo, hi);
          else
            live_span<float>(p.mask, base, p.mk_sn, p.N, lane, lo, hi);
          lo = __reduce_min_sync(0xffffffffu, lo);
          hi = __reduce_max_sync(0xffffffffu, hi);
          if (hi >= 0) { t_begin = lo / kBN; t_end = hi / kBN + 1; }   // else every key is dead: visit all
        }
        if (p.causal) {
          // Keys a row may see: n <= m + p_seq, m < q0 + kNQ * kBM.
          const int last_key = min(q0 + kNQ * kBM, qlen) - 1 + p.p_seq;
          t_end = min(t_end, last_key < 0 ? 0 : last_key / kBN + 1);
        }
        if (kVariant == kDeberta && q0 >= qlen) t_end = t_begin;   // rows all padded: zeros only
        if (p.cu_seqlens != nullptr && q0 >= qlen) t_end = t_begin;   // packed: no rows here at all
        if (kVariant == kT5) {
          float* rb = rbias_buf + slot * kRBiasLen;
          if (p.table == nullptr) {
            for (int e = lane; e <= 2 * (R + kRPad); e += 32) rb[e] = 0.f;
          } else if (p.table_dtype == VF_DTYPE_BF16) {
            fill_bias<__nv_bfloat16>(p, lut_s, rb, h, lane);
          } else if (p.table_dtype == VF_DTYPE_F16) {
            fill_bias<__half>(p, lut_s, rb, h, lane);
          } else {
            fill_bias<float>(p, lut_s, rb, h, lane);
          }
        }
      }
      if (lane == 0) {
        UnitInfo& u = info[slot];
        u.valid = valid ? 1 : 0;
        u.b = b;
        u.h = h;
        u.q0 = q0;
        u.t_begin = t_begin;
        u.nkv = max(t_end - t_begin, 0);
        u.klen = klen;
        u.qlen = qlen;
        info_row0[slot] = row0;
      }
      __syncwarp();
      mbar_arrive(&info_full[slot]);
      if (!valid) break;
    }
  } else if (warp == kLoadWarp) {
    // ------------------------------------------------------------ TMA producer
    int gt = 0;          // key tiles issued so far (ring position)
    int qi = 0;          // units with key tiles so far (Q buffer index)
    for (int i = 0;; ++i) {
      const int slot = i & 1;
      const bool oki = mbar_wait(&info_full[slot], (i >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, oki)) break;
      const UnitInfo u = info[slot];
      const int row0 = info_row0[slot];
      const int bc = p.cu_seqlens != nullptr ? 0 : u.b;   // batch coordinate in the views
      __syncwarp();
      if (lane == 0) mbar_arrive(&info_empty[slot]);
      if (!u.valid) break;
      if (u.nkv == 0) continue;
      const int qs = ring_slot<QB>(qi);
      if (qi >= QB) {
        const bool ok = mbar_wait(&q_empty[qs], ring_parity<QB>(qi - QB), abort_flag);
        if (!__all_sync(0xffffffffu, ok)) break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&q_full[qs], kNQ * kTileBytes);
        for (int g = 0; g < kNQ; ++g)
          tma_load_4d(smem + S::kOffQ + (qs * kNQ + g) * kTileBytes, &p.tm_q, &q_full[qs], 0, row0 + u.q0 + g * kBM, u.h, bc);
      }
      ++qi;
      bool stop = false;
      for (int t = 0; t < u.nkv; ++t, ++gt) {
        const int s = gt % KV;
        const int round = gt / KV;
        if (round > 0) {
          const bool ok = mbar_wait(&kv_empty[s], (round - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) { stop = true; break; }
        }
        const int k0 = (u.t_begin + t) * kBN;
        if (lane == 0) {
          mbar_arrive_expect_tx(&k_full[s], kTileBytes);
          tma_load_4d(smem + S::kOffK + s * kTileBytes, &p.tm_k, &k_full[s], 0, row0 + k0, u.h, bc);
          mbar_arrive_expect_tx(&v_full[s], kTileBytes);
          tma_load_4d(smem + S::kOffV + s * kTileBytes, &p.tm_v, &v_full[s], 0, row0 + k0, u.h, bc);
        }
        if (has_mask) {
          bool zero = true;
          const long long base = u.b * p.mk_sb + u.h * p.mk_sh;
#pragma unroll
          for (int i2 = 0; i2 < kBN / 32; ++i2) {
            const int c = lane + 32 * i2;
            const int n = k0 + c;
            float mv = 0.f;
            if (n < p.N) mv = load_any(p.mask, base + n * p.mk_sn, p.mask_dtype);
            zero = zero && (mv == 0.f);
            kbias[s * kBN + c] = fmaxf(mv, kMaskFloor) * kLog2e;
          }
          zero = __all_sync(0xffffffffu, zero);
          if (lane == 0) kzero[s] = zero ? 1 : 0;
          __syncwarp();
          if (lane == 0) mbar_arrive(&k_full[s]);
        }
      }
      if (stop) break;
    }
    // No TMA write may land after this CTA exits: wait for the last fills (already
    // complete on the normal path), ignoring the abort flag but still time-bounded.
    if (lane == 0) {
      for (int j = max(qi - QB, 0); j < qi; ++j) mbar_wait_bounded(&q_full[ring_slot<QB>(j)], ring_parity<QB>(j));
      for (int t = max(gt - KV, 0); t < gt; ++t) {
        mbar_wait_bounded(&k_full[t % KV], (t / KV) & 1);
        mbar_wait_bounded(&v_full[t % KV], (t / KV) & 1);
      }
    }
  } else if (warp == kMmaWarp || (kMmaIssuers == 2 && warp == kMmaWarp2)) {
    // ------------------------------------------------------------ UMMA issuer
    // Serves softmax groups [g_lo, g_hi).
    const int g_lo = (kMmaIssuers == 2 && warp == kMmaWarp2) ? 1 : 0;
    const int g_hi = kMmaIssuers == 2 ? g_lo + 1 : kNQ;
    if (lane == 0) {
      constexpr uint32_t fmt = AbFormat<T>::value;
      constexpr uint32_t idesc_qk = idesc_f16(fmt, kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = idesc_f16(fmt, kBM, kHeadDim, 0, 1);
      const uint32_t sQ = smem_u32(smem + S::kOffQ);
      const uint32_t sK = smem_u32(smem + S::kOffK);
      const uint32_t sV = smem_u32(smem + S::kOffV);
      auto issue_qk = [&](int g, int qs, int s) {
#pragma unroll
        for (int kk = 0; kk < kHeadDim / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(sQ + (qs * kNQ + g) * kTileBytes + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(sK + s * kTileBytes + kk * 32, 16, 1024);
          umma_ss(tmem + 256 * g, ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int g, int s, bool acc) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bd = smem_desc_sw128(sV + s * kTileBytes + kk * 2048, 0, 1024);
          umma_ts(tmem + 256 * g + 192, tmem + 256 * g + 128 + kk * 8, bd, idesc_pv,
                  (acc || kk > 0) ? 1u : 0u);
        }
      };
      // Cursor over this CTA's key tiles in order (units with no tiles are skipped).
      int ui = 0;          // next unit slot to read
      int qi = -1;         // Q buffer index of the cursor's unit
      bool ok = true;
      auto next_unit = [&](int& nkv) -> bool {   // advances to the next unit with tiles
        for (;;) {
          const int slot = ui & 1;
          if (!mbar_wait(&info_full[slot], (ui >> 1) & 1, abort_flag)) { ok = false; return false; }
          const int valid = info[slot].valid;
          nkv = info[slot].nkv;
          mbar_arrive(&info_empty[slot]);
          ++ui;
          if (!valid) return false;
          if (nkv > 0) { ++qi; return true; }
        }
      };
      int cur_nkv = 0, cur_t = 0;
      int G = 0;           // global tile index of the cursor
      // First tile of a unit: S = Q K^T for both groups (the S columns are free).
      auto start_unit = [&]() -> bool {
        if (!mbar_wait(&q_full[ring_slot<QB>(qi)], ring_parity<QB>(qi), abort_flag) ||
            !mbar_wait(&k_full[G % KV], (G / KV) & 1, abort_flag))
          return false;
        tc_fence_after();
        for (int g = g_lo; g < g_hi; ++g) {
          issue_qk(g, ring_slot<QB>(qi), G % KV);
          umma_commit(&s_full[g]);
        }
        if (cur_nkv == 1) umma_commit(&q_empty[ring_slot<QB>(qi)]);
        return true;
      };
      bool have = next_unit(cur_nkv);
      if (have && ok) ok = start_unit();
      // Order per key tile G: as soon as a group has read S(G) into registers, its
      // S(G+1) = Q K(G+1)^T of the same unit is issued (it overlaps that group's
      // exponentials); PV(G) is issued when the group's P(G) is in TMEM.  The next unit
      // is looked up only after the last PV of the current one, so a run of units with
      // no key tiles never waits on a unit slot that this unit still holds; its first QK
      // is not needed earlier anyway (the softmax threads read O first).  The first PV of
      // a unit overwrites O: the softmax threads have read the previous unit's O before
      // they publish that P.
      while (have && ok) {
        const int s = G % KV;
        const bool more = cur_t + 1 < cur_nkv;
        const int s2 = (G + 1) % KV;
        if (more && !mbar_wait(&k_full[s2], ((G + 1) / KV) & 1, abort_flag)) break;
        for (int g = g_lo; g < g_hi && ok; ++g) {
          if (!mbar_wait(&s_consumed[g], G & 1, abort_flag)) { ok = false; break; }
          if (more) {
            tc_fence_after();
            issue_qk(g, ring_slot<QB>(qi), s2);
            umma_commit(&s_full[g]);
          }
        }
        if (!ok) break;
        if (more && cur_t + 2 == cur_nkv) umma_commit(&q_empty[ring_slot<QB>(qi)]);
        if (!mbar_wait(&v_full[s], (G / KV) & 1, abort_flag)) break;
        for (int g = g_lo; g < g_hi && ok; ++g) {
          if (!mbar_wait(&p_full[g], G & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
          issue_pv(g, s, cur_t > 0);
          umma_commit(&pv_done[g]);
        }
        if (!ok) break;
        umma_commit(&kv_empty[s]);
        ++G;
        if (more) {
          ++cur_t;
        } else {
          cur_t = 0;
          have = next_unit(cur_nkv);
          if (have && ok) ok = start_unit();
        }
      }
      // Drain: every MMA issued above has completed before TMEM is released.
      umma_commit(drain);
      {
        const uint32_t a = smem_u32(drain);
        const long long t0 = clock64();
        while (!mbar_try_wait(a, 0) && clock64() - t0 < kWaitCycles) {}
      }
    }
    __syncwarp();
    // TMEM is released once every softmax group and issuer is done with it.
    tc_fence_before();
    named_bar_sync(1, kSoftmaxThreads + 32 * kMmaIssuers);
    tc_fence_after();
    if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
  }
  return;
  }

  reg_alloc<kVariant == kDeberta ? kRegsSoftmaxDeberta : kRegsSoftmax>();
  {
    // ------------------------------------------------------------ softmax groups
    const int g = warp >> 2;                  // query tile
    const int row = (warp & 3) * 32 + lane;   // row inside the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + lane_off + 256 * g;
    const uint32_t tP = tS + 128;
    const uint32_t tO = tS + 192;
    const float scale_log2 = p.scale_log2;
    int G = 0;                                // global tile index
    bool aborted = false;

    for (int i = 0; !aborted; ++i) {
      const int slot = i & 1;
      {
        const bool oki = mbar_wait(&info_full[slot], (i >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, oki)) break;
      }
      // Unit fields are re-read from shared memory where they are used, which keeps
      // them out of the registers held across the tile loop.
      const volatile UnitInfo* vu = info + slot;
      if (!vu->valid) break;
      const int nkv = vu->nkv;
      const int m = vu->q0 + g * kBM + row;

      float m_run = -INFINITY;
      float l_run = 0.f;
      int k0 = vu->t_begin * kBN;
      for (int t = 0; t < nkv; ++t, ++G, k0 += kBN) {
        const int st = G % KV;
        const float* rbias = rbias_buf + slot * kRBiasLen;
        bool ok = mbar_wait(&s_full[g], G & 1, abort_flag);
        if (has_mask) ok = ok && mbar_wait(&k_full[st], (G / KV) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
        tc_fence_after();
        // Scores in log2 units.  TMEM is read 32 columns at a time (bounded register
        // pressure; the asm's memory clobber also keeps each chunk's loads behind its TMEM
        // load).  x2[j] holds columns 2j, 2j+1.
        float2 x2[kBN / 2];
        bool const_bias = false;   // x2 holds raw S; bias `cbias` and scale still to apply
        float cbias = 0.f;
        if constexpr (kVariant == kT5) {
          // Warp-uniform tile class over the warp's 32 rows: r = n - m in [r_lo, r_hi].
          const int m0 = m - lane;
          const int r_lo = k0 - (m0 + 31);
          const int r_hi = k0 + kBN - 1 - m0;
          const float2 sc2 = make_float2(scale_log2, scale_log2);
          const bool saturated = (r_lo >= R) || (r_hi <= -R);
          tmem_ld_2x64_f2(tS, x2);
          tc_fence_before();
          mbar_arrive(&s_consumed[g]);
          // The key mask (additive, per key) joins the bias operand of the single FMA pass;
          // tiles whose mask is all zero skip it.
          const bool kadd = has_mask && !kzero[st];
          const float2* kb2 = reinterpret_cast<const float2*>(kbias + st * kBN);
          const int klen = vu->klen;
          const bool edge = (k0 + kBN > klen) || (p.causal && r_hi > 0);
          if (!kQMask && saturated && !kadd && !edge && scale_log2 > 0.f) {
            // Constant bias: keep raw S; max(s * sc + cb) = max(s) * sc + cb, and the
            // exponent pass computes s * sc + (cb - m) in one FMA.
            const_bias = true;
            cbias = rbias[(r_lo >= R ? 2 * R : 0) + kRPad];
          } else {
            // One FMA pass: x = s * scale + (bias[c] + key mask[c]).  rb[c] is the bias of
            // column c; a saturated window reads a constant run of the table's padding.
            // Tiles whose key mask is all zero read a zero row instead of the mask.
            const float* rb = saturated ? rbias + (r_lo >= R ? 2 * R + kRPad : 0)
                                        : rbias + (k0 - m + R + kRPad);
            if (kadd) {
#pragma unroll
              for (int j = 0; j < kBN / 2; ++j)
                x2[j] = __ffma2_rn(x2[j], sc2, __fadd2_rn(make_float2(rb[2 * j], rb[2 * j + 1]), kb2[j]));
            } else {
#pragma unroll
              for (int j = 0; j < kBN / 2; ++j) x2[j] = __ffma2_rn(x2[j], sc2, make_float2(rb[2 * j], rb[2 * j + 1]));
            }
          }
          if constexpr (kQMask) {
            // The caller's mask row m (rows past M read row M - 1; their output is not
            // stored), clamped like the key mask, in log2 units.
            const long long rowbase = vu->b * p.qm_sb + vu->h * p.qm_sh + (long long)min(m, p.M - 1) * p.qm_sm;
            if (p.qmask_vec && k0 + kBN <= p.N) {
              const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.qmask) + rowbase + k0);
              const bool bf = p.mask_dtype == VF_DTYPE_BF16;
#pragma unroll
              for (int q8 = 0; q8 < kBN / 8; ++q8) {
                const uint4 w = __ldg(src + q8);
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const uint16_t lo = static_cast<uint16_t>(ws[e] & 0xffffu), hi = static_cast<uint16_t>(ws[e] >> 16);
                  const float flo = bf ? __uint_as_float(static_cast<uint32_t>(lo) << 16) : __half2float(__ushort_as_half(lo));
                  const float fhi = bf ? __uint_as_float(static_cast<uint32_t>(hi) << 16) : __half2float(__ushort_as_half(hi));
                  x2[4 * q8 + e] = __ffma2_rn(make_float2(fmaxf(flo, kMaskFloor), fmaxf(fhi, kMaskFloor)),
                                              make_float2(kLog2e, kLog2e), x2[4 * q8 + e]);
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < kBN / 2; ++j) {   // fully unrolled: x2 stays in registers
                const int n = k0 + 2 * j;
                const float a0 = n < p.N ? load_any(p.qmask, rowbase + n * p.qm_sn, p.mask_dtype) : 0.f;
                const float a1 = n + 1 < p.N ? load_any(p.qmask, rowbase + (n + 1) * p.qm_sn, p.mask_dtype) : 0.f;
                x2[j] = __ffma2_rn(make_float2(fmaxf(a0, kMaskFloor), fmaxf(a1, kMaskFloor)),
                                   make_float2(kLog2e, kLog2e), x2[j]);
              }
            }
          }
          if (edge) {
#pragma unroll
            for (int j = 0; j < kBN / 2; ++j) {
              const int n = k0 + 2 * j;
              if (n >= klen || (p.causal && n > m)) x2[j].x = -INFINITY;
              if (n + 1 >= klen || (p.causal && n + 1 > m)) x2[j].y = -INFINITY;
            }
          }
        } else {
          // Position rows are rows row0 + m / row0 + n of the views (row0 = 0 unless the batch
          // is packed, whose single-batch views have their batch strides set to 0 by the host).
          const int row0 = reinterpret_cast<const volatile int*>(smem + S::kOffInfo + kOffInfoRow0)[slot];
          const int b = vu->b, h = vu->h, klen = vu->klen;
          // Position terms.  A missing term (or a row past the sequence, whose output is zero
          // or not written) reads one zero element with stride 0, so the gather loop has no
          // branches and its loads can be in flight together (a per-column branch around
          // each gather serialised them: ~1.9x slower).
          const T* zero = reinterpret_cast<const T*>(&g_zero_pos);
          const bool pk_on = p.pos_key != nullptr && m < vu->qlen;
          const T* pk_row = pk_on ? reinterpret_cast<const T*>(p.pos_key) + b * p.pk_sb + h * p.pk_sh +
                                        (long long)(row0 + m) * p.pk_sm
                                  : zero;
          const long long pk_sk = pk_on ? p.pk_sk : 0;
          const bool pq_on = p.pos_query != nullptr;
          const T* pq_bh = pq_on ? reinterpret_cast<const T*>(p.pos_query) + b * p.pq_sb + h * p.pq_sh +
                                       (long long)row0 * p.pq_sn
                                 : zero;
          const long long pq_sn = pq_on ? p.pq_sn : 0, pq_sk = pq_on ? p.pq_sk : 0;
          // Offsets inside the tile are 32-bit (the host bounds them): a 64-bit address per
          // column was 16-23 % slower.  Per column only nn = min(c, klen - 1 - k0) varies
          // (k0 < klen for every visited tile); the row and tile constants are hoisted, which
          // took C1 from 84 to 72 us.
          const T* pq_tile = pq_bh + (long long)k0 * pq_sn;
          const int nlim = klen - 1 - k0, mk = m - k0;
          const int pq_sn32 = static_cast<int>(pq_sn), pq_sk32 = static_cast<int>(pq_sk), pk_sk32 = static_cast<int>(pk_sk);
          // S first (one TMEM read, so QK of the next tile can start), then the terms.
          tmem_ld_2x64_f2(tS, x2);
          tc_fence_before();
          mbar_arrive(&s_consumed[g]);
          // Every index comes from the shared-memory LUT.  (A warp-uniform arithmetic path
          // for windows inside the exact bucket range, idx = r + const, was 11-13 % slower:
          // the select kept both paths in the unrolled loop.)
#pragma unroll
          for (int c = 0; c < kBN; ++c) {
            const int nn = min(c, nlim);            // key n = k0 + nn; keys past klen are masked below
            const int idx = lut_s[min(max(mk - nn, -R), R) + R];
            const float add = to_f<T>(pk_row[idx * pk_sk32]) + to_f<T>(pq_tile[nn * pq_sn32 + idx * pq_sk32]);
            if (c & 1) x2[c >> 1].y = (x2[c >> 1].y + add) * scale_log2;
            else x2[c >> 1].x = (x2[c >> 1].x + add) * scale_log2;
          }
          if (k0 + kBN > klen || p.causal) {
#pragma unroll
            for (int j = 0; j < kBN / 2; ++j) {
              const int n = k0 + 2 * j;
              if (n >= klen || (p.causal && n > m + p.p_seq)) x2[j].x = -INFINITY;
              if (n + 1 >= klen || (p.causal && n + 1 > m + p.p_seq)) x2[j].y = -INFINITY;
            }
          }
        }
        // Row max: eight independent 3-input max chains.
        float mx;
        {
          float a[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) a[i] = fmaxf(x2[i].x, x2[i].y);
#pragma unroll
          for (int j = 8; j < kBN / 2; j += 8) {
#pragma unroll
            for (int i = 0; i < 8; ++i) a[i] = fmax3(a[i], x2[j + i].x, x2[j + i].y);
          }
          mx = fmaxf(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], fmax3(a[5], a[6], a[7])));
          if (const_bias) mx = fmaf(mx, scale_log2, cbias);
        }

        // Online softmax with lazy rescaling: the running max only moves (and O, l are
        // rescaled) when a row's max grows by more than the threshold.
        const float m_new = fmaxf(m_run, mx);
        const bool need = m_new > m_run + RescaleThreshold<T>::value;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2_approx(m_run - m_new) : 1.f;
          if (t > 0) {
            // O holds PV(t-1) only once that MMA has completed.
            const bool okp = mbar_wait(&pv_done[g], (G - 1) & 1, abort_flag);
            if (!__all_sync(0xffffffffu, okp)) { aborted = true; break; }
            tc_fence_after();
#pragma unroll
            for (int ch = 0; ch < kHeadDim / 16; ++ch) {
              uint32_t o[16];
              tmem_ld_x16(tO + 16 * ch, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st_x16(tO + 16 * ch, o);
            }
          }
          l_run *= alpha;
          if (need) m_run = m_new;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        // y = x * mul + add: (1, -m) for finished scores, (scale, cbias - m) for raw S.
        const float2 mul2 = const_bias ? make_float2(scale_log2, scale_log2) : make_float2(1.f, 1.f);
        const float2 add2 = const_bias ? make_float2(cbias - m_use, cbias - m_use) : make_float2(-m_use, -m_use);
          float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
        uint32_t pk[kBN / 2];
#pragma unroll
        for (int j = 0; j < kBN / 2; ++j) {
          const float2 y = __ffma2_rn(x2[j], mul2, add2);
          // One pair in kPolyEvery goes to the FMA pipe, the rest to the MUFU unit.
          const float2 e = (j % kPolyEvery == kPolyEvery - 1) ? exp2_poly2(y)
                                                              : make_float2(ex2_approx(y.x), ex2_approx(y.y));
          if (j & 1) ls1 = __fadd2_rn(ls1, e); else ls0 = __fadd2_rn(ls0, e);
          pk[j] = pack2<T>(e.x, e.y);
        }
          const float2 ls = __fadd2_rn(ls0, ls1);
        l_run += ls.x + ls.y;
        if (G > 0) {
          // P(G-1) is read by PV(G-1): the P columns are free once it has completed.  The
          // wait sits after the exponentials, so the PV round trip overlaps them.
          const bool okp = mbar_wait(&pv_done[g], (G - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, okp)) { aborted = true; break; }
          tc_fence_after();
        }
        tmem_st_x64(tP, pk);
        tc_fence_before();
        mbar_arrive(&p_full[g]);
      }

      // Epilogue: O / l, rows past the valid length written as zeros (DeBERTa).  The wait
      // and the TMEM loads are warp-collective and run on every lane (`aborted` and `nkv`
      // are warp-uniform).  O has been read out of TMEM before this group's first P of the
      // next unit is published, so the next unit's first PV (which overwrites O) cannot
      // start early.
      bool have = false;
      if (nkv > 0 && !aborted) {
        const bool ok = mbar_wait(&pv_done[g], (G - 1) & 1, abort_flag);
        if (__all_sync(0xffffffffu, ok)) {
          tc_fence_after();
          have = true;
        } else {
          aborted = true;
        }
      }
      if (p.cu_seqlens != nullptr) {
        // Packed batch: the next sequence's rows follow this one's, so a 128-row tile store
        // could overwrite them.  Each thread stages its own row (unswizzled) and copies it
        // with one 128-byte bulk copy if the row belongs to the sequence.
        const bool mine = m < vu->qlen;     // units past the sequence's end write nothing
        const bool use = have && mine && l_run > 0.f;
        const float inv_l = use ? 1.f / l_run : 0.f;
        bulk_wait_read_all();                // this thread's previous row copy has read its row
        uint8_t* srow = smem + S::kOffOStage + g * kTileBytes + row * 128;
        // The row's eight 16-byte chunks, packed.  Written in natural order, the 8 lanes of
        // one store phase (rows r..r+7, 128 bytes apart) would all hit the same four banks;
        // instead step s writes chunk s ^ (row & 7), so those lanes write 8 different
        // chunks.  pk[s] is brought to hold chunk s ^ (row & 7) by three conditional swaps.
        uint4 pk[kHeadDim / 8];
#pragma unroll
        for (int ch = 0; ch < kHeadDim / 16; ++ch) {
          uint32_t o[16];
          if (have) {
            tmem_ld_x16(tO + 16 * ch, o);    // collective: every lane, whatever its row
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = 0u;
          }
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float f[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] = use ? __uint_as_float(o[8 * hf + j]) * inv_l : 0.f;
            uint4& v = pk[2 * ch + hf];
            v.x = pack2<T>(f[0], f[1]);
            v.y = pack2<T>(f[2], f[3]);
            v.z = pack2<T>(f[4], f[5]);
            v.w = pack2<T>(f[6], f[7]);
          }
        }
        const int rx = row & 7;
#pragma unroll
        for (int bit = 1; bit < 8; bit <<= 1) {
          const bool sw = (rx & bit) != 0;
#pragma unroll
          for (int s = 0; s < 8; ++s) {
            if ((s & bit) != 0) continue;
            const uint4 a = pk[s], b = pk[s | bit];
            pk[s] = sw ? b : a;
            pk[s | bit] = sw ? a : b;
          }
        }
        if (mine) {
#pragma unroll
          for (int s = 0; s < 8; ++s) *reinterpret_cast<uint4*>(srow + ((s ^ rx) * 16)) = pk[s];
        }
        if (mine) {
          fence_proxy_async_smem();
          T* dst = reinterpret_cast<T*>(p.out) + vu->h * p.o_sh +
                   (long long)(reinterpret_cast<const volatile int*>(smem + S::kOffInfo + kOffInfoRow0)[slot] + m) * p.o_sm;
          bulk_copy_s2g(dst, srow, kHeadDim * 2);
          bulk_commit();
        }
      } else
      // O rows go to the group's staging tile (128-byte rows, 16-byte chunks XOR-swizzled
      // by row as the store's SWIZZLE_128B map expects) and leave in one bulk store, so
      // no generic global store stands in front of this thread's later barrier releases.
      {
        const bool row_valid = (kVariant != kDeberta) || (m < vu->qlen);
        const bool use = have && row_valid && l_run > 0.f;
        const float inv_l = use ? 1.f / l_run : 0.f;
        if (row == 0) {
          bulk_wait_read_all();              // this group's previous store has read the tile
          mbar_arrive(&stage_free[g]);
        }
        const bool okf = mbar_wait(&stage_free[g], i & 1, abort_flag);
        uint8_t* stg = smem + S::kOffOStage + g * kTileBytes + row * 128;
        if (okf) {
          // O is read 16 columns at a time (`have` is warp-uniform: the load is collective).
#pragma unroll
          for (int ch = 0; ch < kHeadDim / 16; ++ch) {
            uint32_t o[16];
            if (have) {
              tmem_ld_x16(tO + 16 * ch, o);
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) o[j] = 0u;
            }
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = use ? __uint_as_float(o[8 * hf + j]) * inv_l : 0.f;
              uint4 v;
              v.x = pack2<T>(f[0], f[1]);
              v.y = pack2<T>(f[2], f[3]);
              v.z = pack2<T>(f[4], f[5]);
              v.w = pack2<T>(f[6], f[7]);
              *reinterpret_cast<uint4*>(stg + (((2 * ch + hf) ^ (row & 7)) * 16)) = v;
            }
          }
          fence_proxy_async_smem();
        }
        mbar_arrive(&stage_full[g]);
        if (row == 0 && mbar_wait(&stage_full[g], i & 1, abort_flag)) {
          tma_store_4d(&p.tm_o, smem + S::kOffOStage + g * kTileBytes, 0, vu->q0 + g * kBM, vu->h, vu->b);
          bulk_commit();
        }
        if (!__all_sync(0xffffffffu, okf)) aborted = true;
      }
      tc_fence_before();
      mbar_arrive(&info_empty[slot]);
    }
  }

  // This thread's O stores have landed (tile stores: one thread per group; packed rows:
  // every thread).
  if (p.cu_seqlens != nullptr || (threadIdx.x & (kBM - 1)) == 0) bulk_wait_all();
  tc_fence_before();
  named_bar_sync(1, kSoftmaxThreads + 32 * kMmaIssuers);
}

// Failure-detection self-test: one CTA waits on an mbarrier that nothing ever arrives
// at.  The bounded wait must give up after `limit_cycles`, set the abort flag and the
// device error word, and return; the kernel then exits normally.
__global__ void selftest_wait_timeout_kernel(long long limit_cycles, int* result) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0, &abort_flag, limit_cycles);
  if (threadIdx.x == 0 && result != nullptr) *result = ok ? 1 : 0;
}

}  // namespace vf

// =====================================================================================
// Host side: validation, bucket tables, tensor maps, launch, C ABI.
// =====================================================================================
namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int elem_size(vf_dtype_t d) { return d == VF_DTYPE_F32 ? 4 : 2; }

// T5 relative bucket, float32 arithmetic in the reference's order of operations
// (models/mt5/mt5_encoder.py:125-148).
int t5_bucket_one(int rp, int num_buckets, int max_distance, bool bidirectional) {
  int ret = 0;
  int nb = num_buckets;
  if (bidirectional) {
    nb /= 2;
    if (rp > 0) ret += nb;
    rp = rp < 0 ? -rp : rp;
  } else {
    rp = rp < 0 ? -rp : 0;
  }
  const int max_exact = nb / 2;
  if (rp < max_exact) return ret + rp;
  const float num = logf(static_cast<float>(rp) / static_cast<float>(max_exact));
  const float den = logf(static_cast<float>(static_cast<double>(max_distance) / static_cast<double>(max_exact)));
  const float v = num / den * static_cast<float>(nb - max_exact);
  long long large = max_exact + static_cast<long long>(v);   // .to(torch.long): truncation
  if (large > nb - 1) large = nb - 1;
  return ret + static_cast<int>(large);
}

// DeBERTa log bucket, float32 arithmetic in the reference's order of operations
// (models/deberta_v2/deberta_v2_encoder.py:70-89).
int deberta_bucket_one(int r, int bucket_size, int max_position) {
  const int mid = bucket_size / 2;
  const int sign = (r > 0) - (r < 0);
  const int abs_pos = (r < mid && r > -mid) ? mid - 1 : (r < 0 ? -r : r);
  if (abs_pos <= mid) return r;
  const float num = logf(static_cast<float>(abs_pos) / static_cast<float>(mid));
  const float den = logf(static_cast<float>(static_cast<double>(max_position - 1) / static_cast<double>(mid)));
  const float lp = ceilf(num / den * static_cast<float>(mid - 1)) + static_cast<float>(mid);
  return static_cast<int>(lp * static_cast<float>(sign));
}

// Cached relative-position tables.  `lut[i]` is the value for relative position i - R.
struct RelTable {
  int R = 0;
  std::vector<short> lut;
};
std::mutex g_table_mu;
std::map<std::tuple<int, int, int, int, int, int>, RelTable> g_tables;

// Smallest radius R (<= rmax) such that f(r) == f(+-R) for every |r| in [R, rmax].
template <class F>
int saturation_radius(F f, int rmax) {
  int R = rmax;
  const int vpos = f(rmax), vneg = f(-rmax);
  while (R > 0 && f(R - 1) == vpos && f(-(R - 1)) == vneg) --R;
  return R;
}

const RelTable& t5_table(int nb, int maxd, bool bidir, int L) {
  std::lock_guard<std::mutex> lk(g_table_mu);
  auto key = std::make_tuple(0, nb, maxd, bidir ? 1 : 0, L, 0);
  auto it = g_tables.find(key);
  if (it != g_tables.end()) return it->second;
  auto f = [&](int r) { return t5_bucket_one(r, nb, maxd, bidir); };
  RelTable t;
  t.R = saturation_radius(f, std::max(L - 1, 0));
  t.lut.resize(2 * t.R + 1);
  for (int i = 0; i <= 2 * t.R; ++i) t.lut[i] = static_cast<short>(f(i - t.R));
  return g_tables.emplace(key, std::move(t)).first->second;
}

const RelTable& deberta_table(int span, int nbuckets, int maxd, bool log_bucket, int L) {
  std::lock_guard<std::mutex> lk(g_table_mu);
  auto key = std::make_tuple(1, span, nbuckets, maxd, log_bucket ? 1 : 0, L);
  auto it = g_tables.find(key);
  if (it != g_tables.end()) return it->second;
  auto f = [&](int r) {
    const int bucket = log_bucket ? deberta_bucket_one(r, nbuckets, maxd) : r;
    long long idx = static_cast<long long>(bucket) + span;
    if (idx < 0) idx = 0;
    if (idx > 2LL * span - 1) idx = 2LL * span - 1;
    return static_cast<int>(idx);
  };
  RelTable t;
  t.R = saturation_radius(f, std::max(L - 1, 0));
  t.lut.resize(2 * t.R + 1);
  for (int i = 0; i <= 2 * t.R; ++i) t.lut[i] = static_cast<short>(f(i - t.R));
  return g_tables.emplace(key, std::move(t)).first->second;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// (B, H, L, 64) strided view -> 4-D tensor map with a 64 x 128 box, 128-byte swizzle.
int make_tile_map(CUtensorMap* map, const vf_tensor4d_t& t, vf_dtype_t dt, const char* name) {
  auto enc = get_encode_fn();
  if (enc == nullptr) return fail(VF_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const int es = elem_size(dt);
  if (t.stride[3] != 1) return fail(VF_EINVAL, std::string(name) + ": innermost (head_dim) stride must be 1");
  if ((reinterpret_cast<uintptr_t>(t.data) & 15) != 0) return fail(VF_EINVAL, std::string(name) + ": base pointer must be 16-byte aligned");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(t.size[3]), static_cast<cuuint64_t>(t.size[2]),
                        static_cast<cuuint64_t>(t.size[1]), static_cast<cuuint64_t>(t.size[0])};
  cuuint64_t strides[3];
  for (int i = 0; i < 3; ++i) {
    const long long s = t.stride[2 - i] * es;
    if (s <= 0 || (s % 16) != 0) return fail(VF_EINVAL, std::string(name) + ": strides must be positive multiples of 16 bytes");
    strides[i] = static_cast<cuuint64_t>(s);
  }
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType ty = dt == VF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, ty, 4, const_cast<void*>(t.data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VF_ECUDA, std::string(name) + ": cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return VF_OK;
}

int check_qkv(const vf_tensor4d_t& q, const vf_tensor4d_t& k, const vf_tensor4d_t& v, const vf_tensor4d_t& o) {
  if (!q.data || !k.data || !v.data || !o.data) return fail(VF_EINVAL, "q, k, v and out must be non-null");
  for (int i = 0; i < 4; ++i)
    if (q.size[i] <= 0 || k.size[i] <= 0 || v.size[i] <= 0) return fail(VF_EINVAL, "q, k, v must have positive sizes");
  if (q.size[3] != vf::kHeadDim || k.size[3] != vf::kHeadDim || v.size[3] != vf::kHeadDim)
    return fail(VF_EUNSUPPORTED, "head_dim must be 64");
  if (k.size[0] != q.size[0] || v.size[0] != q.size[0] || k.size[1] != q.size[1] || v.size[1] != q.size[1])
    return fail(VF_EINVAL, "q, k, v must agree on batch and heads");
  if (v.size[2] != k.size[2]) return fail(VF_EINVAL, "k and v must have the same length");
  for (int i = 0; i < 4; ++i)
    if (o.size[i] != q.size[i]) return fail(VF_EINVAL, "out must have the shape of q");
  if (o.stride[3] != 1 || (o.stride[2] % 8) != 0 || (reinterpret_cast<uintptr_t>(o.data) & 15) != 0)
    return fail(VF_EINVAL, "out rows must be contiguous and 16-byte aligned");
  if (q.size[0] > 65535 || q.size[1] > 65535) return fail(VF_EUNSUPPORTED, "batch and heads must be < 65536");
  if (q.size[2] > (1 << 30) || k.size[2] > (1 << 30)) return fail(VF_EUNSUPPORTED, "sequence too long");
  return VF_OK;
}

template <int kVariant, typename T, bool kQMask = false>
int launch(vf::KParams* kp, cudaStream_t stream) {
  auto kern = vf::attn_fwd_kernel<kVariant, T, kQMask>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::once_flag flags[64];
  static cudaError_t attr_err[64];
  static int sm_count[64];
  if (dev < 0 || dev >= 64) return fail(VF_ECUDA, "device ordinal out of range");
  std::call_once(flags[dev], [&] {
    attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, vf::smem_alloc<kVariant>());
    if (attr_err[dev] == cudaSuccess)
      attr_err[dev] = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
  });
  if (attr_err[dev] != cudaSuccess) return fail(VF_ECUDA, std::string("kernel set-up: ") + cudaGetErrorString(attr_err[dev]));
  // Persistent launch: one CTA per SM (at most one per unit); each walks its units.
  const long long units = (long long)((kp->M + vf::kNQ * vf::kBM - 1) / (vf::kNQ * vf::kBM)) * kp->H * kp->B;
  if (units == 0) return VF_OK;
  const dim3 grid(static_cast<unsigned>(std::min<long long>(units, std::max(sm_count[dev], 1))));
  kern<<<grid, vf::kThreads, vf::smem_alloc<kVariant>(), stream>>>(*kp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return VF_OK;
}

void fill_common(vf::KParams* kp, const vf_tensor4d_t& q, const vf_tensor4d_t& k, const vf_tensor4d_t& o) {
  kp->out = const_cast<void*>(o.data);
  kp->o_sb = o.stride[0];
  kp->o_sh = o.stride[1];
  kp->o_sm = o.stride[2];
  kp->B = static_cast<int>(q.size[0]);
  kp->H = static_cast<int>(q.size[1]);
  kp->M = static_cast<int>(q.size[2]);
  kp->N = static_cast<int>(k.size[2]);
}

// Shared set-up of the two T5 entry points: operand checks, tensor maps, scale, table
// pointer.  Leaves the mask, the bucket table and (packed layout) the geometry to the caller.
int rpb_prepare(const vf_rpb_attention_args_t* a, vf::KParams* kp) {
  if (a->dtype != VF_DTYPE_BF16 && a->dtype != VF_DTYPE_F16)
    return fail(VF_EUNSUPPORTED, "rpb attention: q/k/v dtype must be float16 or bfloat16");
  int rc = check_qkv(a->q, a->k, a->v, a->out);
  if (rc) return rc;
  if (a->dropout_p != 0.0f) return fail(VF_EUNSUPPORTED, "rpb attention: dropout_p must be 0 (inference path)");
  const int H = static_cast<int>(a->q.size[1]);
  std::memset(kp, 0, offsetof(vf::KParams, lut));
  if ((rc = make_tile_map(&kp->tm_q, a->q, a->dtype, "q"))) return rc;
  if ((rc = make_tile_map(&kp->tm_k, a->k, a->dtype, "k"))) return rc;
  if ((rc = make_tile_map(&kp->tm_v, a->v, a->dtype, "v"))) return rc;
  if ((rc = make_tile_map(&kp->tm_o, a->out, a->dtype, "out"))) return rc;
  fill_common(kp, a->q, a->k, a->out);
  kp->scale_log2 = a->softmax_scale * vf::kLog2e;
  kp->causal = a->is_decoder ? 1 : 0;
  kp->p_seq = 0;
  if (a->rpb_table != nullptr) {
    if (a->table_cols != H) return fail(VF_EINVAL, "rpb_table must be [num_buckets, heads]");
    if (a->table_rows <= 0) return fail(VF_EINVAL, "rpb_table has no rows");
    kp->table = a->rpb_table;
    kp->tb_srow = a->table_stride_row;
    kp->tb_scol = a->table_stride_col;
    kp->table_dtype = a->table_dtype;
  }
  const int half = a->is_decoder ? a->num_buckets : a->num_buckets / 2;
  if (half / 2 < 1 || a->max_distance <= half / 2)
    return fail(VF_EUNSUPPORTED, "rpb attention: bucket configuration outside the T5 formula's domain");
  return VF_OK;
}

// Bucket lookup table for relative positions |n - m| < span, clamped to the table's rows.
int finish_rpb_table(const vf_rpb_attention_args_t* a, int span, vf::KParams* kp) {
  const int nb = static_cast<int>(a->rpb_table ? a->table_rows : a->num_buckets);
  const RelTable& tab = t5_table(a->num_buckets, a->max_distance, !a->is_decoder, span);
  if (tab.R > vf::kMaxRel) return fail(VF_EUNSUPPORTED, "rpb attention: relative-position table too large");
  kp->rel_R = tab.R;
  for (int i = 0; i <= 2 * tab.R; ++i) {
    int v = tab.lut[i];
    v = std::min(std::max(v, 0), nb - 1);   // kernels/flash_attention_rpb.py:162 clamp to the table
    kp->lut[i] = static_cast<short>(v);
  }
  return VF_OK;
}

// Checks shared by the packed-batch entry points (the views and the offsets array).
int check_packed(const vf_tensor4d_t& q, const vf_tensor4d_t& k, const int32_t* cu_seqlens, int32_t num_seqs,
                 int32_t max_seqlen, const char* what) {
  const std::string w(what);
  if (cu_seqlens == nullptr || (reinterpret_cast<uintptr_t>(cu_seqlens) & 3) != 0)
    return fail(VF_EINVAL, w + ": cu_seqlens must be a non-null, 4-byte aligned device int32 array");
  if (num_seqs <= 0 || num_seqs > 65535) return fail(VF_EINVAL, w + ": num_seqs must be in [1, 65535]");
  if (q.size[0] != 1) return fail(VF_EINVAL, w + ": q/k/v/out must be packed views of size (1, H, total, 64)");
  if (k.size[2] != q.size[2]) return fail(VF_EINVAL, w + ": k and q must have the same packed rows");
  if (max_seqlen <= 0 || max_seqlen > q.size[2]) return fail(VF_EINVAL, w + ": max_seqlen must be in [1, total rows]");
  return VF_OK;
}

// Shared set-up of the two DeBERTa entry points: operand checks, tensor maps, scale and the
// position tensors (batch extent `batch`: B, or 1 for a packed batch).  Leaves the causal
// offset, seq_lengths, the index table and (packed layout) the geometry to the caller.
int deberta_prepare(const vf_deberta_attention_args_t* a, int64_t batch, vf::KParams* kp) {
  if (a->dtype != VF_DTYPE_BF16 && a->dtype != VF_DTYPE_F16)
    return fail(VF_EUNSUPPORTED, "deberta attention: q/k/v dtype must be float16 or bfloat16");
  int rc = check_qkv(a->q, a->k, a->v, a->out);
  if (rc) return rc;
  const int64_t H = a->q.size[1], M = a->q.size[2], N = a->k.size[2];
  const int span = a->position_buckets > 0 ? a->position_buckets : a->max_relative_distance;
  const bool has_pos = a->pos_key.data != nullptr || a->pos_query.data != nullptr;
  if (has_pos && span <= 0) return fail(VF_EINVAL, "deberta attention: position terms need position_buckets or max_relative_distance > 0");
  // The kernel gathers a pos_key row with 32-bit offsets idx * stride (idx < 2 * span) and a
  // key tile of pos_query with (n - k0) * row stride + idx * stride.
  if (a->pos_key.data != nullptr &&
      (a->pos_key.stride[3] < 0 || (2LL * span - 1) * a->pos_key.stride[3] >= (1LL << 31)))
    return fail(VF_EUNSUPPORTED, "deberta attention: pos_key index stride too large for 32-bit offsets");
  if (a->pos_query.data != nullptr &&
      (a->pos_query.stride[2] < 0 || a->pos_query.stride[3] < 0 ||
       (vf::kBN - 1LL) * a->pos_query.stride[2] + (2LL * span - 1) * a->pos_query.stride[3] >= (1LL << 31)))
    return fail(VF_EUNSUPPORTED, "deberta attention: pos_query strides too large for 32-bit in-tile offsets");
  std::memset(kp, 0, offsetof(vf::KParams, lut));
  if ((rc = make_tile_map(&kp->tm_q, a->q, a->dtype, "q"))) return rc;
  if ((rc = make_tile_map(&kp->tm_k, a->k, a->dtype, "k"))) return rc;
  if ((rc = make_tile_map(&kp->tm_v, a->v, a->dtype, "v"))) return rc;
  if ((rc = make_tile_map(&kp->tm_o, a->out, a->dtype, "out"))) return rc;
  fill_common(kp, a->q, a->k, a->out);
  const float sm_scale = a->has_sm_scale ? a->sm_scale : 1.0f / std::sqrt(static_cast<float>(vf::kHeadDim));
  kp->scale_log2 = sm_scale * vf::kLog2e;
  kp->causal = a->causal ? 1 : 0;
  kp->span2 = 2 * span;
  if (a->pos_key.data != nullptr) {
    const vf_tensor4d_t& t = a->pos_key;
    if (t.size[0] != batch || t.size[1] != H || t.size[2] != M || t.size[3] < 2 * span)
      return fail(VF_EINVAL, "deberta attention: pos_key must be (B, H, M, 2*ATT_SPAN)");
    kp->pos_key = t.data;
    kp->pk_sb = t.stride[0]; kp->pk_sh = t.stride[1]; kp->pk_sm = t.stride[2]; kp->pk_sk = t.stride[3];
  }
  if (a->pos_query.data != nullptr) {
    const vf_tensor4d_t& t = a->pos_query;
    if (t.size[0] != batch || t.size[1] != H || t.size[2] != N || t.size[3] < 2 * span)
      return fail(VF_EINVAL, "deberta attention: pos_query must be (B, H, N, 2*ATT_SPAN)");
    kp->pos_query = t.data;
    kp->pq_sb = t.stride[0]; kp->pq_sh = t.stride[1]; kp->pq_sn = t.stride[2]; kp->pq_sk = t.stride[3];
  }
  // Log buckets exactly when the reference's torch path uses them
  // (kernels/flash_deberta_attention.py:400).
  const bool log_bucket = a->use_log_bucket && a->position_buckets > 0 && a->max_relative_distance > 0;
  if (log_bucket && (a->position_buckets < 4 || a->max_relative_distance - 1 <= a->position_buckets / 2))
    return fail(VF_EUNSUPPORTED, "deberta attention: log-bucket configuration outside the formula's domain");
  return VF_OK;
}

// Position-index table for relative positions |m - n| < span.
int finish_deberta_table(const vf_deberta_attention_args_t* a, int span_rows, vf::KParams* kp) {
  const int span = a->position_buckets > 0 ? a->position_buckets : a->max_relative_distance;
  const bool has_pos = a->pos_key.data != nullptr || a->pos_query.data != nullptr;
  const bool log_bucket = a->use_log_bucket && a->position_buckets > 0 && a->max_relative_distance > 0;
  if (has_pos) {
    const RelTable& tab = deberta_table(span, a->position_buckets, a->max_relative_distance, log_bucket, span_rows);
    if (tab.R > vf::kMaxRel) return fail(VF_EUNSUPPORTED, "deberta attention: relative-position table too large");
    kp->rel_R = tab.R;
    std::memcpy(kp->lut, tab.lut.data(), tab.lut.size() * sizeof(short));
  } else {
    kp->rel_R = 0;
    kp->lut[0] = 0;
  }
  return VF_OK;
}

}  // namespace

namespace vf {
// Host helpers for the other kernel files of the library (vf_internal.h).
int set_last_error(int code, const std::string& msg) { return fail(code, msg); }
int host_make_tile_map(CUtensorMap* map, const vf_tensor4d_t& t, vf_dtype_t dt, const char* name) {
  return make_tile_map(map, t, dt, name);
}
int host_check_qkv(const vf_tensor4d_t& q, const vf_tensor4d_t& k, const vf_tensor4d_t& v, const vf_tensor4d_t& o) {
  return check_qkv(q, k, v, o);
}
int host_check_packed(const vf_tensor4d_t& q, const vf_tensor4d_t& k, const int32_t* cu_seqlens, int32_t num_seqs,
                      int32_t max_seqlen, const char* what) {
  return check_packed(q, k, cu_seqlens, num_seqs, max_seqlen, what);
}
int host_deberta_index_table(int span, int position_buckets, int max_relative_distance, bool log_bucket, int L,
                             int max_radius, short* lut_out) {
  const RelTable& tab = deberta_table(span, position_buckets, max_relative_distance, log_bucket, L);
  if (tab.R > max_radius) return -1;
  std::memcpy(lut_out, tab.lut.data(), tab.lut.size() * sizeof(short));
  return tab.R;
}
PFN_cuTensorMapEncodeTiled_v12000 host_encode_fn() { return get_encode_fn(); }
}  // namespace vf

extern "C" {

const char* vf_last_error(void) { return g_last_error.c_str(); }

int vf_abi_version(void) { return VF_ABI_VERSION; }

int vf_device_error(int32_t clear) {
  unsigned int word = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("cudaDeviceSynchronize: ") + cudaGetErrorString(e));
  e = vf::take_error_word(clear != 0, &word);
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("reading the device error word: ") + cudaGetErrorString(e));
  unsigned int fused_word = 0;
  e = vf::fused_take_error_word(clear != 0, &fused_word);
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("reading the device error word: ") + cudaGetErrorString(e));
  unsigned int span_word = 0;
  e = vf::span_take_error_word(clear != 0, &span_word);
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("reading the device error word: ") + cudaGetErrorString(e));
  unsigned int gemm_word = 0;
  e = vf::gemm_take_error_word(clear != 0, &gemm_word);
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("reading the device error word: ") + cudaGetErrorString(e));
  return static_cast<int>((word | fused_word | span_word | gemm_word) & 0x7fffffff);
}

int vf_selftest_wait_timeout(int64_t limit_cycles, void* stream) {
  if (limit_cycles <= 0) return fail(VF_EINVAL, "limit_cycles must be positive");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  vf::selftest_wait_timeout_kernel<<<1, 32, 0, s>>>(static_cast<long long>(limit_cycles), nullptr);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("selftest launch: ") + cudaGetErrorString(e));
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("selftest: ") + cudaGetErrorString(e));
  return VF_OK;
}

int vf_t5_relative_bucket(int32_t num_buckets, int32_t max_distance, int32_t bidirectional, int32_t rmin,
                          int32_t rmax, int32_t* out) {
  if (out == nullptr || rmax < rmin) return fail(VF_EINVAL, "bad output range");
  const int half = bidirectional ? num_buckets / 2 : num_buckets;
  if (half / 2 < 1) return fail(VF_EUNSUPPORTED, "num_buckets too small for the T5 bucket formula");
  if (max_distance <= half / 2) return fail(VF_EUNSUPPORTED, "max_distance must exceed num_buckets/4 (bidirectional) or num_buckets/2");
  for (int r = rmin; r <= rmax; ++r) out[r - rmin] = t5_bucket_one(r, num_buckets, max_distance, bidirectional != 0);
  return VF_OK;
}

int vf_deberta_log_bucket(int32_t bucket_size, int32_t max_position, int32_t rmin, int32_t rmax, int32_t* out) {
  if (out == nullptr || rmax < rmin) return fail(VF_EINVAL, "bad output range");
  if (bucket_size < 4 || max_position - 1 <= bucket_size / 2)
    return fail(VF_EUNSUPPORTED, "log buckets need bucket_size >= 4 and max_position - 1 > bucket_size / 2");
  for (int r = rmin; r <= rmax; ++r) out[r - rmin] = deberta_bucket_one(r, bucket_size, max_position);
  return VF_OK;
}

int vf_rpb_attention_fwd(const vf_rpb_attention_args_t* a, void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  // The mask's shape is checked first (before any driver call).
  const vf_tensor4d_t& mk = a->padding_mask;
  const bool query_mask = mk.data != nullptr && mk.size[2] != 1 && mk.stride[2] != 0;
  if (mk.data != nullptr) {
    if (query_mask && mk.size[2] != a->q.size[2])
      return fail(VF_EINVAL, "rpb attention: padding_mask query dim must be 1 or the query length");
    if (mk.size[3] != a->k.size[2]) return fail(VF_EINVAL, "rpb attention: padding_mask last dim must equal key length");
    if (mk.size[0] != 1 && mk.size[0] != a->q.size[0]) return fail(VF_EINVAL, "rpb attention: padding_mask batch dim");
    if (mk.size[1] != 1 && mk.size[1] != a->q.size[1]) return fail(VF_EINVAL, "rpb attention: padding_mask head dim");
  }
  static thread_local vf::KParams kp;
  int rc = rpb_prepare(a, &kp);
  if (rc) return rc;
  kp.qmask = nullptr;
  if (mk.data != nullptr) {
    kp.mask_dtype = a->mask_dtype;
    const long long sb = mk.size[0] > 1 ? mk.stride[0] : 0, sh = mk.size[1] > 1 ? mk.stride[1] : 0;
    const long long sn = mk.size[3] > 1 ? mk.stride[3] : 0;
    if (query_mask) {
      // A mask that varies over query rows: a kernel instance that adds mask[b, h, m, n] to
      // each score (every key tile of a row visited); the per-key mask path stays off.
      kp.mask = nullptr;
      kp.qmask = mk.data;
      kp.qm_sb = sb;
      kp.qm_sh = sh;
      kp.qm_sm = mk.stride[2];
      kp.qm_sn = sn;
      kp.qmask_vec = a->mask_dtype != VF_DTYPE_F32 && sn == 1 && sb % 8 == 0 && sh % 8 == 0 &&
                     kp.qm_sm % 8 == 0 && (reinterpret_cast<uintptr_t>(mk.data) & 15) == 0;
    } else {
      kp.mask = mk.data;
      kp.mk_sb = sb;
      kp.mk_sh = sh;
      kp.mk_sn = sn;
    }
  }
  if ((rc = finish_rpb_table(a, std::max(kp.M, kp.N), &kp))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (query_mask)
    return a->dtype == VF_DTYPE_BF16 ? launch<vf::kT5, __nv_bfloat16, true>(&kp, s) : launch<vf::kT5, __half, true>(&kp, s);
  return a->dtype == VF_DTYPE_BF16 ? launch<vf::kT5, __nv_bfloat16>(&kp, s) : launch<vf::kT5, __half>(&kp, s);
}

int vf_rpb_attention_varlen_fwd(const vf_rpb_attention_args_t* a, const int32_t* cu_seqlens, int32_t num_seqs,
                                int32_t max_seqlen, void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  int rc = check_packed(a->q, a->k, cu_seqlens, num_seqs, max_seqlen, "rpb varlen");
  if (rc) return rc;
  if (a->padding_mask.data != nullptr)
    return fail(VF_EUNSUPPORTED, "rpb varlen: the packed layout takes no padding_mask (sequences are exact)");
  static thread_local vf::KParams kp;
  rc = rpb_prepare(a, &kp);
  if (rc) return rc;
  kp.cu_seqlens = cu_seqlens;
  kp.packed_rows = kp.M;
  kp.B = num_seqs;
  kp.M = kp.N = max_seqlen;
  if ((rc = finish_rpb_table(a, max_seqlen, &kp))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return a->dtype == VF_DTYPE_BF16 ? launch<vf::kT5, __nv_bfloat16>(&kp, s) : launch<vf::kT5, __half>(&kp, s);
}

int vf_deberta_attention_fwd(const vf_deberta_attention_args_t* a, void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  static thread_local vf::KParams kp;
  int rc = deberta_prepare(a, a->q.size[0], &kp);
  if (rc) return rc;
  const int M = kp.M, N = kp.N;
  kp.p_seq = N - M;
  kp.seq_lengths = a->seq_lengths;
  if ((rc = finish_deberta_table(a, std::max(M, N), &kp))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return a->dtype == VF_DTYPE_BF16 ? launch<vf::kDeberta, __nv_bfloat16>(&kp, s) : launch<vf::kDeberta, __half>(&kp, s);
}

int vf_deberta_attention_varlen_fwd(const vf_deberta_attention_args_t* a, const int32_t* cu_seqlens,
                                    int32_t num_seqs, int32_t max_seqlen, void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  int rc = check_packed(a->q, a->k, cu_seqlens, num_seqs, max_seqlen, "deberta varlen");
  if (rc) return rc;
  if (a->seq_lengths != nullptr)
    return fail(VF_EUNSUPPORTED, "deberta varlen: seq_lengths must be NULL (cu_seqlens gives the lengths)");
  static thread_local vf::KParams kp;
  if ((rc = deberta_prepare(a, 1, &kp))) return rc;
  kp.cu_seqlens = cu_seqlens;
  kp.packed_rows = kp.M;
  kp.B = num_seqs;
  kp.M = kp.N = max_seqlen;
  kp.p_seq = 0;
  kp.pk_sb = kp.pq_sb = 0;   // one packed batch: the kernel's batch coordinate is 0
  if ((rc = finish_deberta_table(a, max_seqlen, &kp))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return a->dtype == VF_DTYPE_BF16 ? launch<vf::kDeberta, __nv_bfloat16>(&kp, s) : launch<vf::kDeberta, __half>(&kp, s);
}

}  // extern "C"
