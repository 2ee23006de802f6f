// sm_100a DeBERTa disentangled attention with the position contractions inside the kernel.
//
// The reference's caller (models/deberta_v2/deberta_v2_encoder.py:275-286) forms
//   pos_key   = Q . Kr^T   (Kr = key_proj(rel),   (1, H, 2S, D))
//   pos_query = K . Qr^T   (Qr = query_proj(rel), (1, H, 2S, D))
// as two (B, H, L, 2S) products in HBM, and the attention kernel
// (kernels/flash_deberta_attention.py:145-299) gathers them per score:
//   s[m, n] = sm_scale * (q_m . k_n + pos_key[m, idx(m - n)] + pos_query[n, idx(m - n)]).
// Here the kernel takes Kr and Qr themselves.  Per 128 x 128 tile (query rows m0.., keys
// k0..) the relative positions r = m - n span 255 consecutive values r_lo .. r_lo + 254,
// r_lo = m0 - k0 - 127, so both terms come from two tensor-core products against a
// 256-row window of "expanded" tables KrE[e] = Kr[idx(e - e0)], QrE[e] = Qr[idx(e - e0)]:
//   Pc[i, c] = q_{m0+i} . KrE[e_lo + c],   P2[j, c] = k_{k0+j} . QrE[e_lo + c],
//   c2p(m0+i, k0+j) = Pc[i, i - j + 127],  p2c(m0+i, k0+j) = P2[j, i - j + 127].
// Four position warps read Pc / P2 out of TMEM and store the skewed tiles (fp16) in shared
// memory in the canonical 64-byte-swizzled operand layouts (c2p K-major by query row, p2c
// MN-major by key row); sixteen small tensor-core products against a 16 x 16 identity then
// add both tiles to S = Q K^T in TMEM.  The softmax warps see the finished score sum and
// run a plain online softmax.  No (B, H, L, 2S) tensor exists anywhere.
//
// Warps (512 threads, 4 warpgroups):
//   0-3   softmax, one thread per query row (TMEM lane)
//   4-11  position warps: warp w reads TMEM lanes 32 (w % 4) .. + 31; warps 4-7 take the
//         first half of each product's columns, warps 8-11 the second half
//   12    TMA producer: Q per unit; K / V (2-stage rings), KrE / QrE windows per key tile
//   13    UMMA issuer (one elected lane) and TMEM owner
//   14    unit preparation (one unit ahead, two-slot ring)
//   15    idle
// TMEM (512 columns): S [0, 128), P (bf16 / fp16 pairs) [128, 192), O [192, 256),
// X [256, 512) = the current position product (Pc, then P2).
// Work units: 128 query rows of one (batch, head); pairs (batch, query block) are ordered by
// key-tile count, longest first, by the set-up kernel (workspace), and dealt to the CTAs in
// snake order.  Every wait is bounded (vf_ptx.cuh).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "vf_ptx.cuh"
#include "vf_internal.h"
#include "../../include/vf_b200.h"

namespace vf {
namespace dfz {

constexpr int kBM = 128;                     // query rows per unit
constexpr int kBN = 128;                     // keys per tile
constexpr int kD = 64;                       // head dim
constexpr int kTile = kBM * kD * 2;          // 16 KB: a 128 x 64 16-bit tile
constexpr int kThreads = 512;
constexpr int kPosWarp0 = 4;                 // position warps 4-11
constexpr int kPosThreads = 256;
constexpr int kLoadWarp = 12;
constexpr int kMmaWarp = 13;
constexpr int kPrepWarp = 14;
constexpr int kTeardownThreads = 128 + kPosThreads + 32;   // softmax, position and MMA warps
constexpr uint32_t kColS = 0, kColP = 128, kColO = 192, kColX = 256, kTmemCols = 512;
constexpr int kMaxRel = 1024;                // index-table radius limit
constexpr int kMaxLut = 2 * kMaxRel + 1;
constexpr int kMaxTiles = 512;               // key tiles per sequence (N <= 65536)
constexpr float kLog2e = 1.4426950408889634f;
// Launched at 128 registers; softmax 200, position warps 112, producers 88
// (128 * (200 + 2 * 112 + 88) = 512 * 128).
constexpr uint32_t kRegsSoftmax = 200, kRegsPos = 112, kRegsProd = 88;
static_assert(128 * (kRegsSoftmax + 2 * kRegsPos + kRegsProd) == 512 * 128, "setmaxnreg split must use the launch budget");

// Shared memory (offsets from a 1024-aligned base).
constexpr int kOffQ = 0;                     // Q tile, 128-byte swizzle (TMA)
constexpr int kOffK = kOffQ + kTile;         // K ring, 2 stages
constexpr int kOffV = kOffK + 2 * kTile;     // V ring, 2 stages
constexpr int kOffKr = kOffV + 2 * kTile;    // KrE window: 256 rows x 128 B, 128-byte swizzle
constexpr int kOffQr = kOffKr + 2 * kTile;   // QrE window
constexpr int kOffXc = kOffQr + 2 * kTile;   // c2p tile: A operand, K-major, 64-byte swizzle, 4 K-blocks of 8 KB
constexpr int kOffXp = kOffXc + 2 * kTile;   // p2c tile: A operand, MN-major, 64-byte swizzle, 4 MN-blocks of 8 KB
constexpr int kOffO = kOffXp + 2 * kTile;    // O staging for the output store
constexpr int kOffI = kOffO + kTile;         // 16 x 16 fp16 identity, K-major, 64-byte swizzle (1 KB)
constexpr int kOffBar = kOffI + 1024;
constexpr int kNumBars = 32;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kOffInfo = kOffMisc + 16;
constexpr int kBytes = kOffInfo + 128;
constexpr int kAlloc = kBytes + 1024;
static_assert(kAlloc <= 232448, "shared memory over the per-CTA limit");

struct __align__(64) FParams {
  CUtensorMap tm_q, tm_k, tm_v, tm_o, tm_kr, tm_qr;
  void* out;
  long long o_sh, o_sm;
  int B, H, M, N;          // B: batch rows (or sequences when packed); M / N: query / key length
  float scale_log2;
  int causal, p_seq;
  int has_c2p, has_p2c;
  int e0;                  // expanded-table row of relative position 0
  const int* seq_lengths;  // padded layout: valid rows / keys per batch row (or null)
  const int* cu_seqlens;   // packed layout (or null)
  int packed_rows;
  const int* order;        // (batch, query block) pairs by cost, longest first
};

struct __align__(64) PrepParams {
  const void* rel_key;
  long long rk_sh, rk_ss;
  const void* rel_query;
  long long rq_sh, rq_ss;
  void* kre;
  void* qre;
  int H, NE, e0, R;
  int* order;
  int B, nqb, M, N, causal, p_seq;
  const int* seq_lengths;
  const int* cu_seqlens;
  int packed_rows;
  short lut[kMaxLut];      // idx(r) for r in [-R, R]
};

struct UnitInfo {
  int valid;
  int b, h, q0;
  int nkv;                 // key tiles [0, nkv)
  int klen, qlen;          // valid keys / rows of the sequence
  int row0;                // first row of the sequence in the views (packed layout)
};

struct SmemMisc {
  uint32_t tmem_base;
  int abort_flag;
};

template <typename T> struct AbFmt;
template <> struct AbFmt<__nv_bfloat16> { static constexpr uint32_t value = 1u; };
template <> struct AbFmt<__half> { static constexpr uint32_t value = 0u; };
template <typename T> __device__ __forceinline__ uint32_t pack_t(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack_t<__nv_bfloat16>(float lo, float hi) { return pack_bf16x2(lo, hi); }
template <> __device__ __forceinline__ uint32_t pack_t<__half>(float lo, float hi) { return pack_f16x2(lo, hi); }
template <typename T> struct Rescale;
template <> struct Rescale<__nv_bfloat16> { static constexpr float value = 32.0f; };
template <> struct Rescale<__half> { static constexpr float value = 8.0f; };

// Valid keys / rows and first row of sequence b (the rules of the compat kernel).
__device__ __forceinline__ void seq_geometry(const int* seq_lengths, const int* cu_seqlens, int packed_rows, int M,
                                             int N, int b, int& klen, int& qlen, int& row0) {
  klen = N;
  qlen = M;
  row0 = 0;
  if (seq_lengths != nullptr) {
    const int L = __ldg(seq_lengths + b);
    klen = min(max(L, 0), N);
    qlen = min(max(L, 0), M);
  }
  if (cu_seqlens != nullptr) {
    const int r0 = __ldg(cu_seqlens + b), r1 = __ldg(cu_seqlens + b + 1);
    if (r0 < 0 || r1 < r0 || r1 > packed_rows || r1 - r0 > M) atomicOr(&g_vf_error, kErrBadInput);
    const int lo = min(max(r0, 0), packed_rows);
    const int L = min(min(max(r1, lo), packed_rows) - lo, M);
    klen = qlen = L;
    row0 = lo;
  }
}

// Key tiles of the unit starting at query row q0: 0 when it has no valid row; trimmed by
// causality (keys n <= m + p_seq).
__device__ __forceinline__ int unit_tiles(int q0, int klen, int qlen, int causal, int p_seq) {
  if (q0 >= qlen) return 0;
  int t_end = (klen + kBN - 1) / kBN;
  if (causal) {
    const int last_key = min(q0 + kBM, qlen) - 1 + p_seq;
    t_end = min(t_end, last_key < 0 ? 0 : last_key / kBN + 1);
  }
  return t_end;
}

// ------------------------------------------------------------------------------ set-up kernel
// Block (0, 0) orders the (batch, query block) pairs by key-tile count (counting sort,
// longest first; the order inside one count is arbitrary and only affects scheduling).
// Blocks (x >= 1, y) fill the expanded position table y / H of head y % H, one 16-byte chunk
// per thread and step (no integer division on the way):
//   KrE[h][e][:] = rel_key[h][idx(e - e0)][:],  QrE likewise.
__global__ void __launch_bounds__(256) prep_kernel(const __grid_constant__ PrepParams p) {
  if (blockIdx.x == 0) {
    if (blockIdx.y != 0) return;
    __shared__ int hist[kMaxTiles + 2];
    __shared__ int top;
    for (int c = threadIdx.x; c < kMaxTiles + 2; c += blockDim.x) hist[c] = 0;
    if (threadIdx.x == 0) top = 0;
    __syncthreads();
    const int P = p.B * p.nqb;
    for (int pi = threadIdx.x; pi < P; pi += blockDim.x) {
      int klen, qlen, row0;
      seq_geometry(p.seq_lengths, p.cu_seqlens, p.packed_rows, p.M, p.N, pi / p.nqb, klen, qlen, row0);
      const int c = min(unit_tiles((pi % p.nqb) * kBM, klen, qlen, p.causal, p.p_seq), kMaxTiles);
      atomicAdd(&hist[c], 1);
      atomicMax(&top, c);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int run = 0;   // exclusive start of each count, counts in decreasing order
      for (int c = top; c >= 0; --c) {
        const int n = hist[c];
        hist[c] = run;
        run += n;
      }
    }
    __syncthreads();
    for (int pi = threadIdx.x; pi < P; pi += blockDim.x) {
      int klen, qlen, row0;
      seq_geometry(p.seq_lengths, p.cu_seqlens, p.packed_rows, p.M, p.N, pi / p.nqb, klen, qlen, row0);
      const int c = min(unit_tiles((pi % p.nqb) * kBM, klen, qlen, p.causal, p.p_seq), kMaxTiles);
      p.order[atomicAdd(&hist[c], 1)] = pi;
    }
    return;
  }
  const int table = blockIdx.y >= static_cast<unsigned>(p.H) ? 1 : 0;
  const int h = blockIdx.y - table * p.H;
  const uint16_t* src_h = table ? reinterpret_cast<const uint16_t*>(p.rel_query) + h * p.rq_sh
                                : reinterpret_cast<const uint16_t*>(p.rel_key) + h * p.rk_sh;
  const long long ss = table ? p.rq_ss : p.rk_ss;
  uint16_t* dst_h = reinterpret_cast<uint16_t*>(table ? p.qre : p.kre) + static_cast<long long>(h) * p.NE * kD;
  const int per_head = p.NE * (kD / 8);
  const int stride = (gridDim.x - 1) * blockDim.x;
  for (int g = (blockIdx.x - 1) * blockDim.x + threadIdx.x; g < per_head; g += stride) {
    const int chunk = g & (kD / 8 - 1);
    const int e = g >> 3;
    const int r = min(max(e - p.e0, -p.R), p.R);
    const int idx = p.lut[r + p.R];
    reinterpret_cast<uint4*>(dst_h + static_cast<long long>(e) * kD)[chunk] =
        __ldg(reinterpret_cast<const uint4*>(src_h + idx * ss) + chunk);
  }
}

// ------------------------------------------------------------------------------ attention kernel
__device__ __forceinline__ bool unit_coords(const FParams& p, int i, int& b, int& h, int& q0) {
  const int nqb = (p.M + kBM - 1) / kBM;
  const long long G = gridDim.x;
  const long long k = (long long)i * G + ((i & 1) ? G - 1 - blockIdx.x : blockIdx.x);
  if (k >= (long long)p.H * nqb * p.B) return false;
  const int pair = __ldg(p.order + static_cast<int>(k / p.H));
  h = static_cast<int>(k % p.H);
  b = pair / nqb;
  q0 = (pair % nqb) * kBM;
  return true;
}

// Address of element (row i, column k) of a 128 x 128 fp16 K-major operand with 64-byte
// swizzle: four K-blocks of 32 columns (8 KB each), 64-byte rows, 16-byte chunks XORed
// with address bits 7-8 (row bits 1-2).
__device__ __forceinline__ uint32_t kmajor_sw64(uint32_t base, int i, int k) {
  const int kin = k & 31;
  return base + (k >> 5) * 8192 + i * 64 + 16 * ((kin >> 3) ^ ((i >> 1) & 3)) + 2 * (kin & 7);
}
// Element (m, k) of a 128 (M) x 128 (K) fp16 MN-major operand with 64-byte swizzle: four
// M-blocks of 32 (8 KB each), 64-byte K-rows, 16-byte chunks XORed with K-row bits 1-2.
__device__ __forceinline__ uint32_t mnmajor_sw64(uint32_t base, int m, int k) {
  const int min_ = m & 31;
  return base + (m >> 5) * 8192 + k * 64 + 16 * ((min_ >> 3) ^ ((k >> 1) & 3)) + 2 * (min_ & 7);
}

// Both staging tiles store 4-byte words (pairs of fp16 along the contiguous dimension): in
// word units, lane row `r` (64 bytes per row) word `t` (0..63) sits at
//   r * 64 + (t / 16) * 8192 + ((4 t mod 64) XOR 16 ((r >> 1) & 3)),
// the two formulas above with the lane terms hoisted (lanebase = base + 64 r, x16).
__device__ __forceinline__ uint32_t sw64_word_addr(uint32_t lanebase, uint32_t x16, int t) {
  const uint32_t u = static_cast<uint32_t>(t);
  return lanebase + ((u >> 4) << 13) + (((u << 2) & 60u) ^ x16);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) fused_kernel(const __grid_constant__ FParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* k_full = bars + 2;      // [2]
  uint64_t* k_empty = bars + 4;     // [2]
  uint64_t* v_full = bars + 6;      // [2]
  uint64_t* v_empty = bars + 8;     // [2]
  uint64_t* kr_full = bars + 10;
  uint64_t* kr_empty = bars + 11;
  uint64_t* qr_full = bars + 12;
  uint64_t* qr_empty = bars + 13;
  uint64_t* x_full = bars + 14;     // a position product is in TMEM X
  uint64_t* x_empty = bars + 15;    // the position warps have read it
  uint64_t* xc_full = bars + 16;    // c2p tile staged
  uint64_t* xc_empty = bars + 17;   // its identity products have read it
  uint64_t* xp_full = bars + 18;
  uint64_t* xp_empty = bars + 19;
  uint64_t* s_full = bars + 20;     // S = QK^T + c2p + p2c in TMEM
  uint64_t* s_consumed = bars + 21;
  uint64_t* p_full = bars + 22;
  uint64_t* pv_done = bars + 23;
  uint64_t* info_full = bars + 24;  // [2]
  uint64_t* info_empty = bars + 26; // [2]
  uint64_t* stage_free = bars + 28;
  uint64_t* stage_full = bars + 29;
  uint64_t* drain = bars + 30;
  SmemMisc* misc = reinterpret_cast<SmemMisc*>(smem + kOffMisc);
  UnitInfo* info = reinterpret_cast<UnitInfo*>(smem + kOffInfo);   // [2]
  volatile int* abort_flag = &misc->abort_flag;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&info_full[s], 32);
      mbar_init(&info_empty[s], 128 + kPosThreads + 1 + 1);
    }
    mbar_init(kr_full, 1);
    mbar_init(kr_empty, 1);
    mbar_init(qr_full, 1);
    mbar_init(qr_empty, 1);
    mbar_init(x_full, 1);
    mbar_init(x_empty, kPosThreads);
    mbar_init(xc_full, kPosThreads);
    mbar_init(xc_empty, 1);
    mbar_init(xp_full, kPosThreads);
    mbar_init(xp_empty, 1);
    mbar_init(s_full, 1);
    mbar_init(s_consumed, 128);
    mbar_init(p_full, 128);
    mbar_init(pv_done, 1);
    mbar_init(stage_free, 1);
    mbar_init(stage_full, 128);
    mbar_init(drain, 1);
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
    if (p.has_c2p) tma_prefetch_desc(&p.tm_kr);
    if (p.has_p2c) tma_prefetch_desc(&p.tm_qr);
  }
  // The 16 x 16 identity B operand of the position-adding products (fp16 1.0 = 0x3C00).
  if (tid < 256) {
    const int n = tid >> 4, k = tid & 15;
    uint16_t* id = reinterpret_cast<uint16_t*>(smem + kOffI);
    const uint32_t off = n * 64 + 16 * ((k >> 3) ^ ((n >> 1) & 3)) + 2 * (k & 7);
    id[off / 2] = n == k ? 0x3C00u : 0u;   // the products read K columns 0-15 only
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc->tmem_base;

  if (warp >= kLoadWarp) {
    reg_dealloc<kRegsProd>();
    if (warp == kPrepWarp) {
      // ---------------------------------------------------------------- unit preparation
      for (int i = 0;; ++i) {
        const int slot = i & 1;
        if (i >= 2) {
          const bool ok = mbar_wait(&info_empty[slot], ((i - 2) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) break;
        }
        int b = 0, h = 0, q0 = 0, klen = 0, qlen = 0, row0 = 0, nkv = 0;
        const bool valid = unit_coords(p, i, b, h, q0);
        if (valid) {
          seq_geometry(p.seq_lengths, p.cu_seqlens, p.packed_rows, p.M, p.N, b, klen, qlen, row0);
          nkv = unit_tiles(q0, klen, qlen, p.causal, p.p_seq);
        }
        if (lane == 0) {
          UnitInfo& u = info[slot];
          u.valid = valid ? 1 : 0;
          u.b = b;
          u.h = h;
          u.q0 = q0;
          u.nkv = nkv;
          u.klen = klen;
          u.qlen = qlen;
          u.row0 = row0;
        }
        __syncwarp();
        mbar_arrive(&info_full[slot]);
        if (!valid) break;
      }
    } else if (warp == kLoadWarp) {
      // ---------------------------------------------------------------- TMA producer
      int G = 0, qi = 0;
      bool stop = false;
      for (int i = 0; !stop; ++i) {
        const int slot = i & 1;
        const bool oki = mbar_wait(&info_full[slot], (i >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, oki)) break;
        const UnitInfo u = info[slot];
        __syncwarp();
        if (lane == 0) mbar_arrive(&info_empty[slot]);
        if (!u.valid) break;
        if (u.nkv == 0) continue;
        const int bc = p.cu_seqlens != nullptr ? 0 : u.b;   // batch coordinate in the views
        if (qi >= 1) {
          const bool ok = mbar_wait(q_empty, (qi - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(q_full, kTile);
          tma_load_4d(smem + kOffQ, &p.tm_q, q_full, 0, u.row0 + u.q0, u.h, bc);
        }
        ++qi;
        for (int t = 0; t < u.nkv; ++t, ++G) {
          const int k0 = t * kBN;
          const int e_lo = u.q0 - k0 - (kBM - 1) + p.e0;
          const int s = G & 1;
          bool ok = true;
          if (p.has_c2p) {
            if (G >= 1) ok = mbar_wait(kr_empty, (G - 1) & 1, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) { stop = true; break; }
            if (lane == 0) {
              mbar_arrive_expect_tx(kr_full, 2 * kTile);
              tma_load_3d(smem + kOffKr, &p.tm_kr, kr_full, 0, e_lo, u.h);
            }
          }
          if (G >= 2) ok = mbar_wait(&k_empty[s], ((G - 2) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) { stop = true; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(&k_full[s], kTile);
            tma_load_4d(smem + kOffK + s * kTile, &p.tm_k, &k_full[s], 0, u.row0 + k0, u.h, bc);
          }
          if (p.has_p2c) {
            if (G >= 1) ok = mbar_wait(qr_empty, (G - 1) & 1, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) { stop = true; break; }
            if (lane == 0) {
              mbar_arrive_expect_tx(qr_full, 2 * kTile);
              tma_load_3d(smem + kOffQr, &p.tm_qr, qr_full, 0, e_lo, u.h);
            }
          }
          if (G >= 2) ok = mbar_wait(&v_empty[s], ((G - 2) >> 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) { stop = true; break; }
          if (lane == 0) {
            mbar_arrive_expect_tx(&v_full[s], kTile);
            tma_load_4d(smem + kOffV + s * kTile, &p.tm_v, &v_full[s], 0, u.row0 + k0, u.h, bc);
          }
        }
      }
      // No TMA write may land after this CTA exits: wait for the last fills (complete on
      // the normal path), ignoring the abort flag but still time-bounded.
      if (lane == 0) {
        if (qi >= 1) mbar_wait_bounded(q_full, (qi - 1) & 1);
        for (int g = max(G - 2, 0); g < G; ++g) {
          mbar_wait_bounded(&k_full[g & 1], (g >> 1) & 1);
          mbar_wait_bounded(&v_full[g & 1], (g >> 1) & 1);
        }
        if (G >= 1 && p.has_c2p) mbar_wait_bounded(kr_full, (G - 1) & 1);
        if (G >= 1 && p.has_p2c) mbar_wait_bounded(qr_full, (G - 1) & 1);
      }
    } else if (warp == kMmaWarp) {
      // ---------------------------------------------------------------- UMMA issuer
      if (lane == 0) {
        constexpr uint32_t fmt = AbFmt<T>::value;
        constexpr uint32_t idesc_qk = idesc_f16(fmt, kBM, kBN, 0, 0);
        constexpr uint32_t idesc_pos = idesc_f16(fmt, kBM, 256, 0, 0);
        constexpr uint32_t idesc_pv = idesc_f16(fmt, kBM, kD, 0, 1);
        constexpr uint32_t idesc_idc = idesc_f16(0u, kBM, 16, 0, 0);   // fp16 x fp16, A K-major
        constexpr uint32_t idesc_idp = idesc_f16(0u, kBM, 16, 1, 0);   // fp16 x fp16, A MN-major
        const uint32_t sQ = smem_u32(smem + kOffQ), sK = smem_u32(smem + kOffK), sV = smem_u32(smem + kOffV);
        const uint32_t sKr = smem_u32(smem + kOffKr), sQr = smem_u32(smem + kOffQr);
        const uint32_t sXc = smem_u32(smem + kOffXc), sXp = smem_u32(smem + kOffXp), sI = smem_u32(smem + kOffI);
        const uint32_t tS = tmem + kColS, tP = tmem + kColP, tO = tmem + kColO, tX = tmem + kColX;
        const uint64_t id_desc = smem_desc(sI, 16, 512, kLayoutSw64);
        int G = 0, prod = 0, qi = 0;
        bool ok = true;
        int pend = -1;               // tile whose O (+)= P V is still to be issued
        int pend_first = 0;          // ... and whether it starts its unit's O (no accumulate)
        auto issue_pv = [&]() -> bool {
          const int g = pend;
          pend = -1;
          if (!mbar_wait(p_full, g & 1, abort_flag) || !mbar_wait(&v_full[g & 1], (g >> 1) & 1, abort_flag))
            return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBN / 16; ++kk) {
            const uint64_t bd = smem_desc(sV + (g & 1) * kTile + kk * 2048, 0, 1024, kLayoutSw128);
            umma_ts(tO, tP + kk * 8, bd, idesc_pv, (!pend_first || kk > 0) ? 1u : 0u);
          }
          umma_commit(pv_done);
          umma_commit(&v_empty[g & 1]);
          return true;
        };
        for (int i = 0; ok; ++i) {
          const int slot = i & 1;
          // The previous unit's last P V waits for the next unit's first scores, unless that
          // unit is not described yet or has no key tiles: its description may need the
          // softmax epilogue of an earlier unit, which waits for that very P V.
          if (pend >= 0) {
            const bool ready = mbar_try_wait(smem_u32(&info_full[slot]), (i >> 1) & 1);
            if ((!ready || !info[slot].valid || info[slot].nkv == 0) && !issue_pv()) { ok = false; break; }
          }
          if (!mbar_wait(&info_full[slot], (i >> 1) & 1, abort_flag)) { ok = false; break; }
          const int valid = info[slot].valid, nkv = info[slot].nkv;
          mbar_arrive(&info_empty[slot]);
          if (!valid) break;
          if (nkv == 0) continue;
          if (!mbar_wait(q_full, qi & 1, abort_flag)) { ok = false; break; }
          ++qi;
          // Pc = Q . KrE_win^T -> X, once X is free (the previous product's columns are in the
          // position warps' registers) and the tile's KrE window has landed.
          auto issue_pc = [&](int g) -> bool {
            if ((prod >= 1 && !mbar_wait(x_empty, (prod - 1) & 1, abort_flag)) ||
                !mbar_wait(kr_full, g & 1, abort_flag))
              return false;
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk)
              umma_ss(tX, smem_desc(sQ + kk * 32, 16, 1024, kLayoutSw128),
                      smem_desc(sKr + kk * 32, 16, 1024, kLayoutSw128), idesc_pos, kk > 0 ? 1u : 0u);
            umma_commit(kr_empty);
            umma_commit(x_full);
            ++prod;
            return true;
          };
          bool pc_ready = false;     // Pc of this tile was issued during the previous tile
          for (int t = 0; t < nkv && ok; ++t, ++G) {
            const int s = G & 1;
            if (p.has_c2p && !pc_ready && !issue_pc(G)) { ok = false; break; }
            // P2 = K . QrE_win^T -> X first: it waits only for this tile's c2p columns to leave
            // X, while S = Q K^T below waits for the previous tile's softmax to read S.
            if (p.has_p2c) {
              if ((prod >= 1 && !mbar_wait(x_empty, (prod - 1) & 1, abort_flag)) ||
                  !mbar_wait(qr_full, G & 1, abort_flag) || !mbar_wait(&k_full[s], (G >> 1) & 1, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < kD / 16; ++kk)
                umma_ss(tX, smem_desc(sK + s * kTile + kk * 32, 16, 1024, kLayoutSw128),
                        smem_desc(sQr + kk * 32, 16, 1024, kLayoutSw128), idesc_pos, kk > 0 ? 1u : 0u);
              umma_commit(qr_empty);
              umma_commit(x_full);
              ++prod;
            }
            // S = Q . K^T
            if (!mbar_wait(&k_full[s], (G >> 1) & 1, abort_flag) ||
                (G >= 1 && !mbar_wait(s_consumed, (G - 1) & 1, abort_flag))) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < kD / 16; ++kk)
              umma_ss(tS, smem_desc(sQ + kk * 32, 16, 1024, kLayoutSw128),
                      smem_desc(sK + s * kTile + kk * 32, 16, 1024, kLayoutSw128), idesc_qk, kk > 0 ? 1u : 0u);
            if (t == nkv - 1) umma_commit(q_empty);
            umma_commit(&k_empty[s]);
            // S += c2p tile, then S += p2c tile (16 columns per product, identity B)
            if (p.has_c2p) {
              if (!mbar_wait(xc_full, G & 1, abort_flag)) { ok = false; break; }
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk)
                umma_ss(tS + 16 * kk, smem_desc(sXc + (kk >> 1) * 8192 + (kk & 1) * 32, 16, 512, kLayoutSw64),
                        id_desc, idesc_idc, 1u);
              umma_commit(xc_empty);
            }
            // O (+)= P V of the previous tile: its P is ready by now, and the tensor cores run it
            // while the position warps store this tile's p2c scores.
            if (pend >= 0 && !issue_pv()) { ok = false; break; }
            // The next tile's Pc as soon as this tile's P2 has left X (same unit): it runs while
            // the p2c scores are being stored.
            pc_ready = p.has_c2p && t + 1 < nkv;
            if (pc_ready && !issue_pc(G + 1)) { ok = false; break; }
            if (p.has_p2c) {
              if (!mbar_wait(xp_full, G & 1, abort_flag)) { ok = false; break; }
              tc_fence_after();
#pragma unroll
              for (int kk = 0; kk < kBN / 16; ++kk)
                umma_ss(tS + 16 * kk, smem_desc(sXp + kk * 1024, 8192, 512, kLayoutSw64), id_desc, idesc_idp, 1u);
              umma_commit(xp_empty);
            }
            umma_commit(s_full);
            pend = G;
            pend_first = t == 0 ? 1 : 0;
          }
        }
        if (ok && pend >= 0) issue_pv();
        // Drain: every MMA issued above has completed before TMEM is released.
        umma_commit(drain);
        {
          const uint32_t a = smem_u32(drain);
          const long long t0 = clock64();
          while (!mbar_try_wait(a, 0) && clock64() - t0 < kWaitCycles) {}
        }
      }
      __syncwarp();
      tc_fence_before();
      named_bar_sync(1, kTeardownThreads);
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
    return;
  }

  if (warp >= kPosWarp0) {
    // ------------------------------------------------------------------ position warps
    reg_dealloc<kRegsPos>();
    const int s = warp & 3;                       // TMEM lane quadrant
    const int half = (warp - kPosWarp0) >> 2;     // 0: first 80 columns of a product's range, 1: the rest
    const int i = 32 * s + lane;                  // TMEM lane: query row (Pc) / key row (P2)
    const uint32_t tX = tmem + (static_cast<uint32_t>(32 * s) << 16) + kColX;
    const uint32_t sXc = smem_u32(smem + kOffXc), sXp = smem_u32(smem + kOffXp);
    // c2p: word of slots (j0, j0 + 1) = (col c, col c - 1); even rows pair (2w+1, 2w) of a
    // 16-column group, odd rows (2w, 2w-1), the latter built from the previous pair's high
    // column.
    const uint32_t sel_c = (i & 1) ? 0x1076u : 0x7654u;
    // p2c: word of M-slots (i0, i0 + 1) = (col c, col c + 1); odd keys pair (2w, 2w+1), even
    // keys (2w+1, 2w+2), built with the next pair's low column.
    const uint32_t sel_p = (i & 1) ? 0x3210u : 0x5432u;
    // Row i needs Pc columns [i, i + 127]: the quadrant reads [32 s, 32 s + 160), this warp its
    // half [32 s + 80 half, + 80), plus the two columns before it (the pairing carry).  Key j
    // needs P2 columns [127 - j, 254 - j]: the quadrant reads [96 - 32 s, 256 - 32 s), this
    // warp its half, plus the two columns after it (the last pair's partner).
    const int cbc = 32 * s + 80 * half;
    const int cbp = 96 - 32 * s + 80 * half;
    // Word addresses: the lane's row (c2p: query row i of Xc; p2c: key row i of the MN-major
    // Xp) and swizzle term, and the word index of the lane's first pair: c2p word
    // t = tc0 - 8 group - w (slots 2t, 2t + 1), p2c word t = tp0 + 8 group + w.
    const uint32_t xc_lane = sXc + 64u * i, xp_lane = sXp + 64u * i, x16 = 16u * ((i >> 1) & 3);
    const int tc0 = ((i + (i & 1)) >> 1) + 63 - (cbc >> 1);
    const int tp0 = (cbp >> 1) + ((i + ((i + 1) & 1) - (kBN - 1)) >> 1);
    int G = 0, prod = 0;
    bool aborted = false;
    for (int ui = 0; !aborted; ++ui) {
      const int slot = ui & 1;
      {
        const bool oki = mbar_wait(&info_full[slot], (ui >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, oki)) break;
      }
      const int valid = info[slot].valid, nkv = info[slot].nkv;
      mbar_arrive(&info_empty[slot]);
      if (!valid) break;
      for (int t = 0; t < nkv; ++t, ++G) {
        if (p.has_c2p) {
          bool ok = mbar_wait(x_full, prod & 1, abort_flag);
          if (G >= 1) ok = ok && mbar_wait(xc_empty, (G - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
          tc_fence_after();
          // 16 columns at a time; the next group's load is in flight while one is stored.
          uint32_t A[16], B[16], E[2];
          tmem_ld_x16_nowait(tX + cbc, A);
          tmem_ld_x2_nowait(tX + (half ? cbc - 2 : cbc), E);
          tmem_wait_ld_regs2(A, E);
          uint32_t carry = half ? pack_f16x2_sat(__uint_as_float(E[1]), __uint_as_float(E[0])) : 0u;
#pragma unroll
          for (int hq = 0; hq < 5; ++hq) {
            uint32_t (&cur)[16] = (hq & 1) ? B : A;
            uint32_t (&nxt)[16] = (hq & 1) ? A : B;
            if (hq < 4) tmem_ld_x16_nowait(tX + cbc + 16 * (hq + 1), nxt);
            uint32_t F[8];
#pragma unroll
            for (int w = 0; w < 8; ++w)
              F[w] = pack_f16x2_sat(__uint_as_float(cur[2 * w + 1]), __uint_as_float(cur[2 * w]));
#pragma unroll
            for (int w = 0; w < 8; ++w) {
              const uint32_t word = prmt(w == 0 ? carry : F[w - 1], F[w], sel_c);
              const int t = tc0 - 8 * hq - w;
              if (static_cast<unsigned>(t) <= 63u) st_shared_u32(sw64_word_addr(xc_lane, x16, t), word);
            }
            carry = F[7];
            if (hq < 4) tmem_wait_ld_regs(nxt);
            if (hq == 3) {
              tc_fence_before();
              mbar_arrive(x_empty);               // every column of this product is in registers
            }
          }
          fence_proxy_async_smem();
          mbar_arrive(xc_full);
          ++prod;
        }
        if (p.has_p2c) {
          bool ok = mbar_wait(x_full, prod & 1, abort_flag);
          if (G >= 1) ok = ok && mbar_wait(xp_empty, (G - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
          tc_fence_after();
          // Each 16-column group is loaded with the two columns after it (its last pair's
          // partner), so no wait falls inside a group; the last group of the second half has
          // no partner it needs.
          uint32_t A[16], B[16], EA[2], EB[2];
          tmem_ld_x16_x2_nowait(tX + cbp, tX + cbp + 16, A, EA);
          tmem_wait_ld_regs2(A, EA);
#pragma unroll
          for (int hq = 0; hq < 5; ++hq) {
            uint32_t (&cur)[16] = (hq & 1) ? B : A;
            uint32_t (&nxt)[16] = (hq & 1) ? A : B;
            uint32_t (&ecur)[2] = (hq & 1) ? EB : EA;
            uint32_t (&enxt)[2] = (hq & 1) ? EA : EB;
            // (the second half's last group has no partner: its extra load re-reads the group
            // start, since the columns after it lie past the product)
            if (hq < 4)
              tmem_ld_x16_x2_nowait(tX + cbp + 16 * (hq + 1),
                                    tX + cbp + 16 * (hq + 1) + ((hq == 3 && half) ? 0 : 16), nxt, enxt);
            uint32_t Gp[9];
#pragma unroll
            for (int w = 0; w < 8; ++w)
              Gp[w] = pack_f16x2_sat(__uint_as_float(cur[2 * w]), __uint_as_float(cur[2 * w + 1]));
            Gp[8] = (hq == 4 && half) ? 0u : pack_f16x2_sat(__uint_as_float(ecur[0]), __uint_as_float(ecur[1]));
#pragma unroll
            for (int w = 0; w < 8; ++w) {
              const uint32_t word = prmt(Gp[w], Gp[w + 1], sel_p);
              const int t = tp0 + 8 * hq + w;
              if (static_cast<unsigned>(t) <= 63u) st_shared_u32(sw64_word_addr(xp_lane, x16, t), word);
            }
            if (hq < 4) tmem_wait_ld_regs2(nxt, enxt);
            if (hq == 3) {
              tc_fence_before();
              mbar_arrive(x_empty);               // the last group is in registers
            }
          }
          fence_proxy_async_smem();
          mbar_arrive(xp_full);
          ++prod;
        }
      }
    }
    tc_fence_before();
    named_bar_sync(1, kTeardownThreads);
    return;
  }

  // -------------------------------------------------------------------- softmax warps
  reg_alloc<kRegsSoftmax>();
  {
    const int row = warp * 32 + lane;               // row inside the unit == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off + kColS;
    const uint32_t tP = tmem + lane_off + kColP;
    const uint32_t tO = tmem + lane_off + kColO;
    const float sc = p.scale_log2;
    int G = 0, ni = 0;                              // tiles so far; epilogue stores so far
    bool aborted = false;
    for (int ui = 0; !aborted; ++ui) {
      const int slot = ui & 1;
      {
        const bool oki = mbar_wait(&info_full[slot], (ui >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, oki)) break;
      }
      const volatile UnitInfo* vu = info + slot;
      if (!vu->valid) {
        mbar_arrive(&info_empty[slot]);
        break;
      }
      const int nkv = vu->nkv;
      const int m = vu->q0 + row;                   // query row in the sequence
      float m_run = -INFINITY, l_run = 0.f;
      for (int t = 0; t < nkv; ++t, ++G) {
        const int k0 = t * kBN;
        const bool ok = mbar_wait(s_full, G & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }
        tc_fence_after();
        float2 x2[kBN / 2];
        tmem_ld_2x64_f2(tS, x2);
        tc_fence_before();
        mbar_arrive(s_consumed);
        // Raw scores s = qk + c2p + p2c; keys past the sequence (and above the causal
        // diagonal) are removed.  The scale is applied in the exponent: for sc > 0,
        // max(s * sc) = max(s) * sc.
        const int klen = vu->klen;
        if (k0 + kBN > klen || p.causal) {
          const float gone = sc >= 0.f ? -INFINITY : INFINITY;   // s * sc = -inf either way
#pragma unroll
          for (int j = 0; j < kBN / 2; ++j) {
            const int n = k0 + 2 * j;
            if (n >= klen || (p.causal && n > m + p.p_seq)) x2[j].x = gone;
            if (n + 1 >= klen || (p.causal && n + 1 > m + p.p_seq)) x2[j].y = gone;
          }
        }
        float mx;
        {
          float a[8];
          if (sc >= 0.f) {
#pragma unroll
            for (int q = 0; q < 8; ++q) a[q] = fmaxf(x2[q].x, x2[q].y);
#pragma unroll
            for (int j = 8; j < kBN / 2; j += 8) {
#pragma unroll
              for (int q = 0; q < 8; ++q) a[q] = fmax3(a[q], x2[j + q].x, x2[j + q].y);
            }
            mx = fmaxf(fmax3(a[0], a[1], a[2]), fmax3(a[3], a[4], fmax3(a[5], a[6], a[7]))) * sc;
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) a[q] = fminf(x2[q].x, x2[q].y);
#pragma unroll
            for (int j = 8; j < kBN / 2; j += 8) {
#pragma unroll
              for (int q = 0; q < 8; ++q) a[q] = fminf(a[q], fminf(x2[j + q].x, x2[j + q].y));
            }
            mx = fminf(fminf(fminf(a[0], a[1]), fminf(a[2], a[3])), fminf(fminf(a[4], a[5]), fminf(a[6], a[7]))) * sc;
          }
          if (mx != mx) mx = -INFINITY;             // every key removed (-inf * sc)
        }
        const float m_new = fmaxf(m_run, mx);
        const bool need = m_new > m_run + Rescale<T>::value;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2_approx(m_run - m_new) : 1.f;
          if (t > 0) {
            const bool okp = mbar_wait(pv_done, (G - 1) & 1, abort_flag);
            if (!__all_sync(0xffffffffu, okp)) { aborted = true; break; }
            tc_fence_after();
#pragma unroll
            for (int ch = 0; ch < kD / 16; ++ch) {
              uint32_t o[16];
              tmem_ld_x16(tO + 16 * ch, o);
#pragma unroll
              for (int q = 0; q < 16; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * alpha);
              tmem_st_x16(tO + 16 * ch, o);
            }
          }
          l_run *= alpha;
          if (need) m_run = m_new;
        }
        const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
        const float2 mul2 = make_float2(sc, sc);
        const float2 add2 = make_float2(-m_use, -m_use);
        float2 ls0 = make_float2(0.f, 0.f), ls1 = make_float2(0.f, 0.f);
        uint32_t pk[kBN / 2];
#pragma unroll
        for (int j = 0; j < kBN / 2; ++j) {
          const float2 y = __ffma2_rn(x2[j], mul2, add2);
          const float2 e = (j % 3 == 2) ? exp2_poly2(y) : make_float2(ex2_approx(y.x), ex2_approx(y.y));
          if (j & 1) ls1 = __fadd2_rn(ls1, e); else ls0 = __fadd2_rn(ls0, e);
          pk[j] = pack_t<T>(e.x, e.y);
        }
        const float2 ls = __fadd2_rn(ls0, ls1);
        l_run += ls.x + ls.y;
        if (G > 0) {
          // P(G - 1) is read by PV(G - 1): the P columns are free once it has completed.
          const bool okp = mbar_wait(pv_done, (G - 1) & 1, abort_flag);
          if (!__all_sync(0xffffffffu, okp)) { aborted = true; break; }
          tc_fence_after();
        }
        tmem_st_x64(tP, pk);
        tc_fence_before();
        mbar_arrive(p_full);
      }

      // Epilogue: O / l, rows past the valid length written as zeros (padded layout) or not
      // at all (packed layout).  The TMEM loads are warp-collective (`have` is uniform).
      bool have = false;
      if (nkv > 0 && !aborted) {
        const bool ok = mbar_wait(pv_done, (G - 1) & 1, abort_flag);
        if (__all_sync(0xffffffffu, ok)) {
          tc_fence_after();
          have = true;
        } else {
          aborted = true;
        }
      }
      const bool row_valid = m < vu->qlen;
      const bool use = have && row_valid && l_run > 0.f;
      const float inv_l = use ? 1.f / l_run : 0.f;
      uint4 pko[kD / 8];
#pragma unroll
      for (int ch = 0; ch < kD / 16; ++ch) {
        uint32_t o[16];
        if (have) {
          tmem_ld_x16(tO + 16 * ch, o);
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) o[q] = 0u;
        }
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float f[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) f[q] = use ? __uint_as_float(o[8 * hf + q]) * inv_l : 0.f;
          uint4& v = pko[2 * ch + hf];
          v.x = pack_t<T>(f[0], f[1]);
          v.y = pack_t<T>(f[2], f[3]);
          v.z = pack_t<T>(f[4], f[5]);
          v.w = pack_t<T>(f[6], f[7]);
        }
      }
      if (p.cu_seqlens != nullptr) {
        // Packed: each thread copies its own row (rows of the next sequence follow).  Step
        // c writes chunk c ^ (row & 7) so the 8 lanes of a store phase use different banks.
        const int rx = row & 7;
#pragma unroll
        for (int bit = 1; bit < 8; bit <<= 1) {
          const bool sw = (rx & bit) != 0;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            if ((c & bit) != 0) continue;
            const uint4 a = pko[c], b = pko[c | bit];
            pko[c] = sw ? b : a;
            pko[c | bit] = sw ? a : b;
          }
        }
        bulk_wait_read_all();
        uint8_t* srow = smem + kOffO + row * 128;
        if (row_valid) {
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(srow + ((c ^ rx) * 16)) = pko[c];
          fence_proxy_async_smem();
          T* dst = reinterpret_cast<T*>(p.out) + vu->h * p.o_sh + (long long)(vu->row0 + m) * p.o_sm;
          bulk_copy_s2g(dst, srow, kD * 2);
          bulk_commit();
        }
      } else {
        if (row == 0) {
          bulk_wait_read_all();               // the previous store has read the staging tile
          mbar_arrive(stage_free);
        }
        const bool okf = mbar_wait(stage_free, ni & 1, abort_flag);
        uint8_t* stg = smem + kOffO + row * 128;
        if (okf) {
#pragma unroll
          for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(stg + ((c ^ (row & 7)) * 16)) = pko[c];
          fence_proxy_async_smem();
        }
        mbar_arrive(stage_full);
        if (row == 0 && mbar_wait(stage_full, ni & 1, abort_flag)) {
          tma_store_4d(&p.tm_o, smem + kOffO, 0, vu->q0, vu->h, vu->b);
          bulk_commit();
        }
        ++ni;
        if (!__all_sync(0xffffffffu, okf)) aborted = true;
      }
      tc_fence_before();
      mbar_arrive(&info_empty[slot]);
    }
  }
  // This thread's output stores have landed (tile stores: row 0; packed rows: every thread).
  if (p.cu_seqlens != nullptr || threadIdx.x == 0) bulk_wait_all();
  tc_fence_before();
  named_bar_sync(1, kTeardownThreads);
}

// Scratch of vf_deberta_attention_fused_noalloc_fwd: the expanded position tables and the
// unit order live here instead of in a caller-provided workspace.  Every GPU that loads the
// library holds these 8 MiB until the process exits.  In host code the name is only a
// host-side stand-in for the device array; its device address comes from
// cudaGetSymbolAddress (noalloc_scratch below).
constexpr long long kNoAllocScratchBytes = 8LL << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Error word of this file (vf_device_error gathers it).
}  // namespace dfz

cudaError_t fused_take_error_word(bool clear, unsigned int* word) { return take_error_word(clear, word); }

}  // namespace vf

// =====================================================================================
// Host side.
// =====================================================================================
namespace {

using vf::set_last_error;

int fail(int code, const std::string& msg) { return set_last_error(code, msg); }

long long ceil128(long long x) { return (x + 127) / 128 * 128; }

struct Geometry {
  long long NE;            // expanded-table rows per head
  long long table_bytes;   // one expanded table
  long long order_bytes;
  long long total;
};

Geometry geometry(long long batch, long long H, long long M, long long N) {
  Geometry g{};
  g.NE = ceil128(M) + ceil128(N);
  g.table_bytes = (H * g.NE * 64 * 2 + 255) / 256 * 256;
  g.order_bytes = (batch * ((M + 127) / 128) * 4 + 255) / 256 * 256;
  g.total = 2 * g.table_bytes + g.order_bytes;
  return g;
}

// Rel table view (1, H, 2S, 64): unit innermost stride, 16-byte aligned rows.
int check_rel(const vf_tensor4d_t& t, long long H, int span, const char* name) {
  const std::string n(name);
  if (t.size[0] != 1) return fail(VF_EUNSUPPORTED, n + ": one position table shared by the batch is supported, (1, H, 2*span, 64)");
  if (t.size[1] != H || t.size[2] < 2LL * span || t.size[3] != 64)
    return fail(VF_EINVAL, n + " must be (1, H, 2*ATT_SPAN, 64)");
  if (t.stride[3] != 1 || (t.stride[2] * 2) % 16 != 0 || (t.stride[1] * 2) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(t.data) & 15) != 0)
    return fail(VF_EINVAL, n + ": rows must be contiguous and 16-byte aligned");
  if (t.stride[2] <= 0 || t.stride[1] < 0 || (2LL * span - 1) * t.stride[2] >= (1LL << 31))
    return fail(VF_EUNSUPPORTED, n + ": strides out of range");
  return VF_OK;
}

int make_table_map(CUtensorMap* map, void* base, long long H, long long NE, vf_dtype_t dt) {
  auto enc = vf::host_encode_fn();
  if (enc == nullptr) return fail(VF_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(NE), static_cast<cuuint64_t>(H)};
  cuuint64_t strides[2] = {128, static_cast<cuuint64_t>(NE * 128)};
  cuuint32_t box[3] = {64, 256, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType ty = dt == VF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, ty, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VF_ECUDA, "position table map: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return VF_OK;
}

template <typename T>
int launch_fused(const vf::dfz::FParams& fp, const vf::dfz::PrepParams& pp, long long units, long long chunks,
                 cudaStream_t stream) {
  auto kern = vf::dfz::fused_kernel<T>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::once_flag flags[64];
  static cudaError_t attr_err[64];
  static int sm_count[64];
  if (dev < 0 || dev >= 64) return fail(VF_ECUDA, "device ordinal out of range");
  std::call_once(flags[dev], [&] {
    attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, vf::dfz::kAlloc);
    if (attr_err[dev] == cudaSuccess) attr_err[dev] = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
  });
  if (attr_err[dev] != cudaSuccess) return fail(VF_ECUDA, std::string("kernel set-up: ") + cudaGetErrorString(attr_err[dev]));
  const int sms = std::max(sm_count[dev], 1);
  // x = 0: the unit order (block (0, 0)); x >= 1: the table rows of head y % H, table y / H.
  const long long per_head = pp.H > 0 ? chunks / (2LL * pp.H) : 0;
  const dim3 prep_grid(static_cast<unsigned>(1 + std::min<long long>((per_head + 255) / 256, 64)),
                       static_cast<unsigned>(std::max(1, 2 * pp.H)));
  vf::dfz::prep_kernel<<<prep_grid, 256, 0, stream>>>(pp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("set-up kernel launch: ") + cudaGetErrorString(e));
  if (units == 0) return VF_OK;
  const dim3 grid(static_cast<unsigned>(std::min<long long>(units, sms)));
  kern<<<grid, vf::dfz::kThreads, vf::dfz::kAlloc, stream>>>(fp);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VF_ECUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return VF_OK;
}

// Shared set-up of the two fused entry points.  `batch` = rows of the padded layout or
// sequences of the packed one; M / N = query / key length (max_seqlen when packed).
int fused_run(const vf_deberta_fused_args_t* a, long long batch, long long M, long long N, const int32_t* cu_seqlens,
              long long packed_rows, void* workspace, int64_t workspace_bytes, cudaStream_t stream) {
  using namespace vf::dfz;
  if (a->dtype != VF_DTYPE_BF16 && a->dtype != VF_DTYPE_F16)
    return fail(VF_EUNSUPPORTED, "deberta fused: q/k/v dtype must be float16 or bfloat16");
  const long long H = a->q.size[1];
  const bool has_c2p = a->rel_key.data != nullptr, has_p2c = a->rel_query.data != nullptr;
  const int span = a->position_buckets > 0 ? a->position_buckets : a->max_relative_distance;
  if ((has_c2p || has_p2c) && span <= 0)
    return fail(VF_EINVAL, "deberta fused: position terms need position_buckets or max_relative_distance > 0");
  int rc;
  if (has_c2p && (rc = check_rel(a->rel_key, H, span, "rel_key"))) return rc;
  if (has_p2c && (rc = check_rel(a->rel_query, H, span, "rel_query"))) return rc;
  if (N > kMaxTiles * kBN || M > kMaxTiles * kBN)
    return fail(VF_EUNSUPPORTED, "deberta fused: sequences longer than 65536 positions");
  const bool log_bucket = a->use_log_bucket && a->position_buckets > 0 && a->max_relative_distance > 0;
  if (log_bucket && (a->position_buckets < 4 || a->max_relative_distance - 1 <= a->position_buckets / 2))
    return fail(VF_EUNSUPPORTED, "deberta fused: log-bucket configuration outside the formula's domain");
  const Geometry g = geometry(batch, H, M, N);
  if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(VF_EINVAL, "deberta fused: workspace must be a non-null, 256-byte aligned device buffer");
  if (workspace_bytes < g.total)
    return fail(VF_EINVAL, "deberta fused: workspace too small (vf_deberta_fused_workspace_bytes gives the size)");

  static thread_local FParams fp;
  static thread_local PrepParams pp;
  std::memset(&fp, 0, sizeof(fp));
  std::memset(&pp, 0, offsetof(PrepParams, lut));
  if ((rc = vf::host_make_tile_map(&fp.tm_q, a->q, a->dtype, "q"))) return rc;
  if ((rc = vf::host_make_tile_map(&fp.tm_k, a->k, a->dtype, "k"))) return rc;
  if ((rc = vf::host_make_tile_map(&fp.tm_v, a->v, a->dtype, "v"))) return rc;
  if ((rc = vf::host_make_tile_map(&fp.tm_o, a->out, a->dtype, "out"))) return rc;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* kre = ws;
  void* qre = ws + g.table_bytes;
  int* order = reinterpret_cast<int*>(ws + 2 * g.table_bytes);
  if (has_c2p && (rc = make_table_map(&fp.tm_kr, kre, H, g.NE, a->dtype))) return rc;
  if (has_p2c && (rc = make_table_map(&fp.tm_qr, qre, H, g.NE, a->dtype))) return rc;
  fp.out = const_cast<void*>(a->out.data);
  fp.o_sh = a->out.stride[1];
  fp.o_sm = a->out.stride[2];
  fp.B = static_cast<int>(batch);
  fp.H = static_cast<int>(H);
  fp.M = static_cast<int>(M);
  fp.N = static_cast<int>(N);
  const float sm_scale = a->has_sm_scale ? a->sm_scale : 1.0f / std::sqrt(64.0f);
  fp.scale_log2 = sm_scale * kLog2e;
  fp.causal = a->causal ? 1 : 0;
  fp.p_seq = static_cast<int>(N - M);
  fp.has_c2p = has_c2p;
  fp.has_p2c = has_p2c;
  fp.e0 = static_cast<int>(ceil128(N) - 1);
  fp.seq_lengths = a->seq_lengths;
  fp.cu_seqlens = cu_seqlens;
  fp.packed_rows = static_cast<int>(packed_rows);
  fp.order = order;

  pp.rel_key = a->rel_key.data;
  pp.rk_sh = a->rel_key.stride[1];
  pp.rk_ss = a->rel_key.stride[2];
  pp.rel_query = a->rel_query.data;
  pp.rq_sh = a->rel_query.stride[1];
  pp.rq_ss = a->rel_query.stride[2];
  pp.kre = kre;
  pp.qre = qre;
  pp.H = static_cast<int>(H);
  pp.NE = static_cast<int>(g.NE);
  pp.e0 = fp.e0;
  pp.order = order;
  pp.B = static_cast<int>(batch);
  pp.nqb = static_cast<int>((M + kBM - 1) / kBM);
  pp.M = fp.M;
  pp.N = fp.N;
  pp.causal = fp.causal;
  pp.p_seq = fp.p_seq;
  pp.seq_lengths = a->seq_lengths;
  pp.cu_seqlens = cu_seqlens;
  pp.packed_rows = fp.packed_rows;
  long long chunks = 0;
  if (has_c2p || has_p2c) {
    const int R = vf::host_deberta_index_table(span, a->position_buckets, a->max_relative_distance, log_bucket,
                                               static_cast<int>(std::max(M, N)), kMaxRel, pp.lut);
    if (R < 0) return fail(VF_EUNSUPPORTED, "deberta fused: relative-position table too large");
    pp.R = R;
    // One table's rows are copied when only one term is present; the other stays unread.
    if (!has_c2p) pp.rel_key = pp.rel_query, pp.rk_sh = pp.rq_sh, pp.rk_ss = pp.rq_ss;
    if (!has_p2c) pp.rel_query = pp.rel_key, pp.rq_sh = pp.rk_sh, pp.rq_ss = pp.rk_ss;
    chunks = 2LL * H * g.NE * 8;
  }
  const long long units = batch * pp.nqb * H;
  if (chunks == 0) {
    // No position term: the set-up kernel only orders the units (block 0).
    pp.H = 0;
  }
  return a->dtype == VF_DTYPE_BF16 ? launch_fused<__nv_bfloat16>(fp, pp, units, chunks, stream)
                                   : launch_fused<__half>(fp, pp, units, chunks, stream);
}

// Device address of the static scratch array on the current device, looked up once per device
// (with that device current) and cached.  Returns nullptr and sets the error message when the
// lookup fails.
void* noalloc_scratch() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    fail(VF_ECUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    return nullptr;
  }
  static std::once_flag flags[64];
  static void* ptr[64];
  static cudaError_t err[64];
  if (dev < 0 || dev >= 64) {
    fail(VF_ECUDA, "device ordinal out of range");
    return nullptr;
  }
  std::call_once(flags[dev], [&] { err[dev] = cudaGetSymbolAddress(&ptr[dev], vf::dfz::g_noalloc_scratch); });
  if (err[dev] != cudaSuccess || ptr[dev] == nullptr) {
    fail(VF_ECUDA, std::string("cudaGetSymbolAddress of the static scratch: ") + cudaGetErrorString(err[dev]));
    return nullptr;
  }
  return ptr[dev];
}

}  // namespace

extern "C" {

int vf_deberta_attention_fused_noalloc_fwd(const vf_deberta_fused_args_t* a, void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  int rc = vf::host_check_qkv(a->q, a->k, a->v, a->out);
  if (rc) return rc;
  const long long need = geometry(a->q.size[0], a->q.size[1], a->q.size[2], a->k.size[2]).total;
  if (need > vf::dfz::kNoAllocScratchBytes)
    return fail(VF_EUNSUPPORTED, "deberta fused noalloc: this call needs " + std::to_string(need) +
                                     " bytes of scratch; the static scratch holds " +
                                     std::to_string(vf::dfz::kNoAllocScratchBytes) +
                                     " (use vf_deberta_attention_fused_fwd with a workspace)");
  void* scratch = noalloc_scratch();
  if (scratch == nullptr) return VF_ECUDA;
  return fused_run(a, a->q.size[0], a->q.size[2], a->k.size[2], nullptr, 0, scratch, vf::dfz::kNoAllocScratchBytes,
                   static_cast<cudaStream_t>(stream));
}

int64_t vf_deberta_fused_workspace_bytes(int64_t batch_or_seqs, int64_t heads, int64_t M, int64_t N) {
  if (batch_or_seqs < 0 || heads < 0 || M < 0 || N < 0) return fail(VF_EINVAL, "negative size");
  return geometry(batch_or_seqs, heads, M, N).total;
}

int vf_deberta_attention_fused_fwd(const vf_deberta_fused_args_t* a, void* workspace, int64_t workspace_bytes,
                                   void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  int rc = vf::host_check_qkv(a->q, a->k, a->v, a->out);
  if (rc) return rc;
  return fused_run(a, a->q.size[0], a->q.size[2], a->k.size[2], nullptr, 0, workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
}

int vf_deberta_attention_fused_varlen_fwd(const vf_deberta_fused_args_t* a, const int32_t* cu_seqlens,
                                          int32_t num_seqs, int32_t max_seqlen, void* workspace,
                                          int64_t workspace_bytes, void* stream) {
  if (a == nullptr) return fail(VF_EINVAL, "null args");
  int rc = vf::host_check_qkv(a->q, a->k, a->v, a->out);
  if (rc) return rc;
  if ((rc = vf::host_check_packed(a->q, a->k, cu_seqlens, num_seqs, max_seqlen, "deberta fused varlen"))) return rc;
  if (a->seq_lengths != nullptr)
    return fail(VF_EUNSUPPORTED, "deberta fused varlen: seq_lengths must be NULL (cu_seqlens gives the lengths)");
  return fused_run(a, num_seqs, max_seqlen, max_seqlen, cu_seqlens, a->q.size[2], workspace, workspace_bytes,
                   static_cast<cudaStream_t>(stream));
}

}  // extern "C"
