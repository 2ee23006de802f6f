// GLiNER span scoring on sm_100a (tcgen05 UMMA, TMEM accumulator, TMA-staged class rows).
//
// The reference scores the spans of a sentence with SpanMarkerV0 + an einsum
// (poolers/gliner.py:118-140 and :285-289; the same marker in poolers/gliner2.py:230-259):
//     rep[s]      = out_project(relu(cat(start_rep[i_s], end_rep[j_s])))          (2D -> 4D -> D MLP)
//     score[s, c] = rep[s] · pe[c]
// The first Linear of out_project acts on a concatenation, so it splits into two per-word
// products, and the second Linear folds into the class side:
//     U = relu(start_rep) W1a^T + b1,   V = relu(end_rep) W1b^T   (per word, [words, 4D])
//     P = pe W2,                        pb = pe · b2               (per class, [classes, 4D])
//     score[s, c] = pb[c] + sum_k relu(U[i_s, k] + V[j_s, k]) * P[c, k]
// The caller forms U, V, P, pb (cuBLAS GEMMs over words and classes, not spans); this file
// does the per-span part: one CTA per 128 spans builds the A operand relu(U[i] + V[j]) in
// tensor memory (each span row is its thread's TMEM lane, 64 K-columns per stage, written
// with tcgen05.st) and multiplies it by the TMA-staged class rows on the tensor cores, A read
// from TMEM.  The tile's word rows come in by TMA with the class rows when its start and end
// words each fit 32 consecutive rows (always so for the reference's default enumeration of
// spans); other tiles load their rows directly.  The reference's [spans, 2D] / [spans, 4D] / [spans, D] intermediates never
// exist, and A never passes through shared memory.
//
// Several sentences (segments) go in one launch: segment g has its own word rows, spans and
// class rows, and its scores form a [spans_g, classes_g] row-major block of the output.  The
// per-segment tables travel as kernel parameters (no device allocation, no host copy).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "vf_internal.h"
#include "vf_ptx.cuh"

namespace vf {
namespace span {

constexpr int kTile = 128;             // spans per CTA: UMMA M, one row-building thread per span
constexpr int kKStep = 64;             // K elements per stage (32 TMEM columns of bf16 / f16 pairs)
constexpr int kStages = 3;
constexpr int kACols = 32;             // TMEM columns of one A stage
constexpr int kAccCol = kStages * kACols;   // first TMEM column of the fp32 accumulator
constexpr int kThreads = 192;          // warps 0-3 rows + epilogue, warp 4 TMA, warp 5 UMMA
#ifndef VF_SPAN_MIN_BLOCKS
#define VF_SPAN_MIN_BLOCKS 3
#endif
constexpr int kMinBlocks = VF_SPAN_MIN_BLOCKS;   // CTAs per SM the register budget allows (latency hiding)
constexpr int kMaxN = 256;             // classes per CTA (UMMA N)
constexpr int kMaxSeg = 256;           // segments per launch (kernel-parameter tables)
constexpr int kRowBox = 32;            // word rows of one staged U / V box
constexpr int kBoxBytes = kRowBox * 128;    // 4 KB: 32 rows x 64 columns of 16-bit
constexpr int kSmemMax = 1024 + kStages * (kMaxN * 128 + 2 * kBoxBytes) + 256;

struct __align__(64) Params {
  CUtensorMap tm_cls;                  // classes [C_total, K], box 64 x npad, 128-byte swizzle
  CUtensorMap tm_u, tm_v;              // start_proj / end_proj [W_total, K], box 64 x kRowBox, 128-byte swizzle
  const void* u;
  const void* v;
  long long us, vs;                    // row strides of U / V (elements)
  const void* idx;
  long long idx_ss, idx_sp;            // span_idx strides (elements)
  const float* cbias;                  // [C_total] or nullptr
  void* out;
  int K, npad, tmem_cols, idx64, out_dtype, nseg;
  int tile_off[kMaxSeg + 1];           // first tile (128 spans) of segment g in this launch
  int word_off[kMaxSeg], word_len[kMaxSeg];
  int class_off[kMaxSeg], class_len[kMaxSeg];
  int span_len[kMaxSeg];
  long long span_off[kMaxSeg];         // first row of segment g in span_idx
  long long out_off[kMaxSeg];          // first element of segment g's block of out
};

// relu(a + b) on two 16-bit lanes, rounded once: fma(a, 1, b) with the .relu clamp.
template <typename T> __device__ __forceinline__ uint32_t add_relu2(uint32_t a, uint32_t b);
template <> __device__ __forceinline__ uint32_t add_relu2<__nv_bfloat16>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("fma.rn.relu.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(0x3F803F80u), "r"(b));
  return d;
}
template <> __device__ __forceinline__ uint32_t add_relu2<__half>(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("fma.rn.relu.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(0x3C003C00u), "r"(b));
  return d;
}
template <typename T> struct AbFmt;
template <> struct AbFmt<__nv_bfloat16> { static constexpr uint32_t value = 1u; };
template <> struct AbFmt<__half> { static constexpr uint32_t value = 0u; };

__device__ __forceinline__ void store_out(void* out, long long off, float x, int dt) {
  if (dt == VF_DTYPE_F32) reinterpret_cast<float*>(out)[off] = x;
  else if (dt == VF_DTYPE_BF16) reinterpret_cast<__nv_bfloat16*>(out)[off] = __float2bfloat16_rn(x);
  else reinterpret_cast<__half*>(out)[off] = __float2half_rn(x);
}

template <typename T>
__global__ void __launch_bounds__(kThreads, kMinBlocks) span_scores_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int npad = p.npad;
  uint8_t* sB = smem;                                   // [kStages][npad rows x 128 B], written by TMA
  uint8_t* sU = sB + kStages * npad * 128;              // [kStages][kRowBox rows x 128 B] (staged tiles)
  uint8_t* sV = sU + kStages * kBoxBytes;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(sV + kStages * kBoxBytes);
  uint64_t* full_b = full_a + kStages;                  // class rows (and staged word rows) landed
  uint64_t* empty = full_b + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* rng = reinterpret_cast<int*>(tmem_slot + 2);     // i_min, i_max, j_min, j_max over rows with i, j > 0

  // This CTA's segment: the last g with tile_off[g] <= tile (segments without tiles have
  // tile_off[g] == tile_off[g + 1] and are passed over).
  const int tile = blockIdx.x;
  int lo = 0, hi = p.nseg - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.tile_off[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  const int g = lo;
  const int s_begin = (tile - p.tile_off[g]) * kTile;   // first span of the tile inside its segment
  const int c0 = blockIdx.y * kMaxN;                     // first class of this CTA
  const int S_g = p.span_len[g], C_g = p.class_len[g];
  if (c0 >= C_g) return;                                 // CTA-uniform, before any barrier or TMEM use
  const int nk = p.K / kKStep;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_a[s], kTile);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    rng[0] = rng[2] = 0x7fffffff;
    rng[1] = rng[3] = -1;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  // The tile's span rows (threads 0-127): word indices clamped to the sentence's words, as
  // the reference's extract_elements clamps them.
  const int t = threadIdx.x;                                // span row of the tile == TMEM lane
  int i = 0, j = 0;
  if (warp < 4) {
    const int sl = min(s_begin + t, S_g - 1);               // rows past the segment repeat its last span
    const long long srow = p.span_off[g] + sl;
    long long i64, j64;
    if (p.idx64) {
      const long long* ix = reinterpret_cast<const long long*>(p.idx) + srow * p.idx_ss;
      i64 = __ldg(ix);
      j64 = __ldg(ix + p.idx_sp);
    } else {
      const int* ix = reinterpret_cast<const int*>(p.idx) + srow * p.idx_ss;
      i64 = __ldg(ix);
      j64 = __ldg(ix + p.idx_sp);
    }
    const long long last = p.word_len[g] - 1;
    i = static_cast<int>(min(max(i64, 0LL), last));
    j = static_cast<int>(min(max(j64, 0LL), last));
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Word 0 is left out of the ranges: masked spans are (0, 0) (the pooler multiplies span_idx by
  // the span mask), and the last tiles of a sentence hold them beside its last words.
  if (warp < 4) {
    if (i > 0) { atomicMin(&rng[0], i); atomicMax(&rng[1], i); }
    if (j > 0) { atomicMin(&rng[2], j); atomicMax(&rng[3], j); }
  }
  __syncthreads();
  // Staged tile: its start words and its end words other than word 0 each lie within kRowBox
  // consecutive rows (the reference's default enumeration gives <= ceil(128 / max_width) + 1
  // and that + max_width - 1), so every stage brings them in as two TMA boxes, and a row
  // outside its box (word 0) is loaded by its own thread; otherwise each thread loads its own
  // rows.  (No row > 0: the boxes start at word 0.)
  const int i_min = rng[1] < 0 ? 0 : rng[0], j_min = rng[3] < 0 ? 0 : rng[2];
  const bool staged = (rng[1] < 0 || rng[1] - i_min < kRowBox) && (rng[3] < 0 || rng[3] - j_min < kRowBox);

  if (warp < 4) {
    // ---------------------------------------------------------------- A rows + epilogue
    const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.u) + (p.word_off[g] + (long long)i) * p.us);
    const uint4* vr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.v) + (p.word_off[g] + (long long)j) * p.vs);
    const uint32_t ru = static_cast<uint32_t>(i - i_min), rv = static_cast<uint32_t>(j - j_min);   // rows in the boxes
    const bool u_box = staged && ru < static_cast<uint32_t>(kRowBox);   // (i < i_min wraps above kRowBox)
    const bool v_box = staged && rv < static_cast<uint32_t>(kRowBox);
    // Each row is read through a generic pointer: its box row in shared memory (16-byte chunk q
    // at q ^ (row & 7), the 128-byte swizzle; the base moves by stage) or its row in global
    // memory (chunk q at q; the base moves by 64 columns a stage).
    const uint8_t* ubase = u_box ? sU + ru * 128 : reinterpret_cast<const uint8_t*>(ur);
    const uint8_t* vbase = v_box ? sV + rv * 128 : reinterpret_cast<const uint8_t*>(vr);
    const uint32_t usw = u_box ? (ru & 7u) : 0u, vsw = v_box ? (rv & 7u) : 0u;
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;   // this warp's TMEM lanes
    bool ok = true;
    for (int kc = 0; kc < nk; ++kc) {
      const int st = kc % kStages;
      if (staged) {
        // The stage's boxes have landed; its TMEM columns are free too (the TMA refilled the
        // stage only after the MMAs that read it had completed).
        ok = mbar_wait(&full_b[st], (kc / kStages) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
      } else if (kc >= kStages) {
        ok = mbar_wait(&empty[st], ((kc / kStages) - 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
      }
      const uint8_t* up = ubase + (u_box ? st * kBoxBytes : kc * 128);
      const uint8_t* vp = vbase + (v_box ? st * kBoxBytes : kc * 128);
      uint4 a[8], b[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        a[q] = *reinterpret_cast<const uint4*>(up + ((static_cast<uint32_t>(q) ^ usw) << 4));
        b[q] = *reinterpret_cast<const uint4*>(vp + ((static_cast<uint32_t>(q) ^ vsw) << 4));
      }
      // Row t of the A stage: 64 elements as 32 packed pairs, K in column order.
      uint32_t r[32];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        r[4 * q + 0] = add_relu2<T>(a[q].x, b[q].x);
        r[4 * q + 1] = add_relu2<T>(a[q].y, b[q].y);
        r[4 * q + 2] = add_relu2<T>(a[q].z, b[q].z);
        r[4 * q + 3] = add_relu2<T>(a[q].w, b[q].w);
      }
      tmem_st_x32(tmem + lane_base + static_cast<uint32_t>(st * kACols), r);   // waits for the store
      tc_fence_before();
      mbar_arrive(&full_a[st]);
    }
    // Epilogue: the 128 x npad fp32 accumulator, 16 columns at a time; each thread writes
    // its own span's classes [c0, c0 + npad) that exist.
    if (ok) ok = mbar_wait(done, 0, abort_flag);
    if (__all_sync(0xffffffffu, ok)) {
      tc_fence_after();
      const bool mine = s_begin + t < S_g;
      const int cend = min(C_g - c0, npad);
      const long long obase = p.out_off[g] + (long long)(s_begin + t) * C_g + c0;
      const float* cb = p.cbias != nullptr ? p.cbias + p.class_off[g] + c0 : nullptr;
      for (int cc = 0; cc < npad; cc += 16) {
        uint32_t r[16];
        tmem_ld_x16(tmem + lane_base + static_cast<uint32_t>(kAccCol + cc), r);   // collective: every lane
        if (mine) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int c = cc + e;
            if (c < cend) store_out(p.out, obase + c, __uint_as_float(r[e]) + (cb != nullptr ? __ldg(cb + c) : 0.f), p.out_dtype);
          }
        }
      }
    }
  } else if (warp == 4) {
    // ---------------------------------------------------------------- class rows (TMA)
    if (lane == 0) {
      int issued = 0;
      const int crow = p.class_off[g] + c0;
      const int urow0 = p.word_off[g] + i_min, vrow0 = p.word_off[g] + j_min;
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % kStages;
        if (kc >= kStages && !mbar_wait(&empty[st], ((kc / kStages) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&full_b[st], static_cast<uint32_t>(npad * 128 + (staged ? 2 * kBoxBytes : 0)));
        tma_load_2d(sB + st * npad * 128, &p.tm_cls, &full_b[st], kc * kKStep, crow);
        if (staged) {
          tma_load_2d(sU + st * kBoxBytes, &p.tm_u, &full_b[st], kc * kKStep, urow0);
          tma_load_2d(sV + st * kBoxBytes, &p.tm_v, &full_b[st], kc * kKStep, vrow0);
        }
        ++issued;
      }
      // No TMA write may land after the CTA exits: wait for the last fills (time-bounded).
      for (int kc = max(issued - kStages, 0); kc < issued; ++kc)
        mbar_wait_bounded(&full_b[kc % kStages], (kc / kStages) & 1);
    }
  } else {
    // ---------------------------------------------------------------- UMMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(AbFmt<T>::value, kTile, static_cast<uint32_t>(npad), 0, 0);
      const uint32_t b0 = smem_u32(sB);
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % kStages;
        const uint32_t par = (kc / kStages) & 1;
        if (!mbar_wait(&full_a[st], par, abort_flag) || !mbar_wait(&full_b[st], par, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kKStep / 16; ++kk) {
          // A: 128 lanes x 8 columns (16 K-elements) of the stage in TMEM; B: the class rows.
          const uint64_t bd = smem_desc_sw128(b0 + st * npad * 128 + kk * 32, 16, 1024);
          umma_ts(tmem + kAccCol, tmem + static_cast<uint32_t>(st * kACols + kk * 8), bd, idesc,
                  (kc > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[st]);
      }
      umma_commit(done);
      // Every MMA issued above has completed before TMEM is released.
      mbar_wait_bounded(done, 0);
    }
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, static_cast<uint32_t>(p.tmem_cols));
  }
}

}  // namespace span

cudaError_t span_take_error_word(bool clear, unsigned int* word) { return take_error_word(clear, word); }

}  // namespace vf

// =====================================================================================
// Host side.
// =====================================================================================
namespace {

int sfail(int code, const std::string& msg) { return vf::set_last_error(code, "span scores: " + msg); }

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <typename T>
int launch_span(const vf::span::Params& prm, unsigned tiles, unsigned ychunks, int smem, cudaStream_t s) {
  auto kern = vf::span::span_scores_kernel<T>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::once_flag flags[64];
  static cudaError_t attr_err[64];
  if (dev < 0 || dev >= 64) return sfail(VF_ECUDA, "device ordinal out of range");
  std::call_once(flags[dev], [&] {
    attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, vf::span::kSmemMax);
  });
  if (attr_err[dev] != cudaSuccess) return sfail(VF_ECUDA, std::string("kernel set-up: ") + cudaGetErrorString(attr_err[dev]));
  kern<<<dim3(tiles, ychunks), vf::span::kThreads, smem, s>>>(prm);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return sfail(VF_ECUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return VF_OK;
}

}  // namespace

extern "C" {

int vf_span_scores_fwd(const vf_span_scores_args_t* a, void* stream) {
  using vf::span::kMaxSeg;
  if (a == nullptr) return sfail(VF_EINVAL, "null args");
  if (a->dtype != VF_DTYPE_BF16 && a->dtype != VF_DTYPE_F16)
    return sfail(VF_EUNSUPPORTED, "start_proj / end_proj / classes dtype must be float16 or bfloat16");
  if (a->out_dtype != VF_DTYPE_F32 && a->out_dtype != VF_DTYPE_BF16 && a->out_dtype != VF_DTYPE_F16)
    return sfail(VF_EINVAL, "out dtype must be float32, float16 or bfloat16");
  const int G = a->num_segments;
  if (G < 0) return sfail(VF_EINVAL, "num_segments must be >= 0");
  if (G == 0) return VF_OK;
  if (!a->word_offsets || !a->span_offsets || !a->class_offsets)
    return sfail(VF_EINVAL, "word_offsets, span_offsets and class_offsets must be host arrays of num_segments + 1");
  const int64_t* wo = a->word_offsets;
  const int64_t* so = a->span_offsets;
  const int64_t* co = a->class_offsets;
  if (wo[0] < 0 || so[0] < 0 || co[0] < 0) return sfail(VF_EINVAL, "offsets must start at >= 0");
  long long work = 0;
  int64_t max_c = 0;
  for (int g = 0; g < G; ++g) {
    if (wo[g + 1] < wo[g] || so[g + 1] < so[g] || co[g + 1] < co[g]) return sfail(VF_EINVAL, "offsets must not decrease");
    const int64_t S = so[g + 1] - so[g], C = co[g + 1] - co[g];
    if (S > 0 && C > 0) {
      if (wo[g + 1] == wo[g]) return sfail(VF_EINVAL, "segment " + std::to_string(g) + " has spans but no words");
      work += S;
      max_c = std::max(max_c, C);
    }
  }
  if (work == 0) return VF_OK;
  if (wo[G] >= (1LL << 31) || co[G] >= (1LL << 31)) return sfail(VF_EUNSUPPORTED, "more than 2^31 - 1 words or classes");
  for (int g = 0; g < G; ++g)
    if (so[g + 1] - so[g] >= (1LL << 31) - vf::span::kTile) return sfail(VF_EUNSUPPORTED, "a segment with 2^31 spans");
  const int64_t K = a->K;
  if (K <= 0 || K % vf::span::kKStep != 0 || K >= (1LL << 31))
    return sfail(VF_EINVAL, "K (the projection width, 4 x hidden) must be a positive multiple of 64");
  if (!a->start_proj || !a->end_proj || !a->classes || !a->span_idx || !a->out)
    return sfail(VF_EINVAL, "start_proj, end_proj, classes, span_idx and out must be non-null");
  if (a->start_row_stride < K || a->end_row_stride < K || a->class_row_stride < K)
    return sfail(VF_EINVAL, "row strides must be at least K");
  if (!al16(a->start_proj) || !al16(a->end_proj) || !al16(a->classes) || (a->start_row_stride * 2) % 16 != 0 ||
      (a->end_row_stride * 2) % 16 != 0 || (a->class_row_stride * 2) % 16 != 0)
    return sfail(VF_EINVAL, "start_proj, end_proj and classes rows must start on 16-byte boundaries");
  if (a->idx_stride_span < 0 || a->idx_stride_pair < 0) return sfail(VF_EINVAL, "negative span_idx strides");

  auto enc = vf::host_encode_fn();
  if (enc == nullptr) return sfail(VF_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  const int npad = static_cast<int>(std::min<int64_t>(vf::span::kMaxN, (max_c + 15) / 16 * 16));
  int tcols = 32;
  while (tcols < vf::span::kAccCol + npad) tcols *= 2;   // A stages + the accumulator

  vf::span::Params prm{};
  {
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(std::max<int64_t>(co[G], 1))};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(a->class_row_stride * 2)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(vf::span::kKStep), static_cast<cuuint32_t>(npad)};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType ty =
        a->dtype == VF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUresult r = enc(&prm.tm_cls, ty, 2, const_cast<void*>(a->classes), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return sfail(VF_ECUDA, "classes map: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
    // start_proj / end_proj rows, 32 at a time (a staged tile's start and end words).
    const void* bases[2] = {a->start_proj, a->end_proj};
    const int64_t rstr[2] = {a->start_row_stride, a->end_row_stride};
    CUtensorMap* maps[2] = {&prm.tm_u, &prm.tm_v};
    for (int w = 0; w < 2; ++w) {
      cuuint64_t wd[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(std::max<int64_t>(wo[G], 1))};
      cuuint64_t ws[1] = {static_cast<cuuint64_t>(rstr[w] * 2)};
      cuuint32_t wb[2] = {static_cast<cuuint32_t>(vf::span::kKStep), static_cast<cuuint32_t>(vf::span::kRowBox)};
      const CUresult rw = enc(maps[w], ty, 2, const_cast<void*>(bases[w]), wd, ws, wb, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (rw != CUDA_SUCCESS)
        return sfail(VF_ECUDA, "word-row map: cuTensorMapEncodeTiled failed (" + std::to_string(int(rw)) + ")");
    }
  }
  prm.u = a->start_proj;
  prm.v = a->end_proj;
  prm.us = a->start_row_stride;
  prm.vs = a->end_row_stride;
  prm.idx = a->span_idx;
  prm.idx_ss = a->idx_stride_span;
  prm.idx_sp = a->idx_stride_pair;
  prm.idx64 = a->span_idx_int64 ? 1 : 0;
  prm.cbias = a->class_bias;
  prm.out = a->out;
  prm.out_dtype = a->out_dtype;
  prm.K = static_cast<int>(K);
  prm.npad = npad;
  prm.tmem_cols = tcols;
  const int smem = 1024 + vf::span::kStages * (npad * 128 + 2 * vf::span::kBoxBytes) + 256;
  const unsigned ych = static_cast<unsigned>((max_c + vf::span::kMaxN - 1) / vf::span::kMaxN);
  if (ych > 65535u) return sfail(VF_EUNSUPPORTED, "more than 65535 x 256 classes in one segment");
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // Segments in groups of kMaxSeg per launch; out_off runs over every segment.
  long long out_off = 0;
  for (int g0 = 0; g0 < G; g0 += kMaxSeg) {
    const int n = std::min(G - g0, kMaxSeg);
    long long tiles = 0;
    for (int q = 0; q < n; ++q) {
      const int g = g0 + q;
      const int64_t S = so[g + 1] - so[g], C = co[g + 1] - co[g];
      prm.tile_off[q] = static_cast<int>(tiles);
      prm.word_off[q] = static_cast<int>(wo[g]);
      prm.word_len[q] = static_cast<int>(wo[g + 1] - wo[g]);
      prm.class_off[q] = static_cast<int>(co[g]);
      prm.class_len[q] = static_cast<int>(C);
      prm.span_len[q] = static_cast<int>(S);
      prm.span_off[q] = so[g];
      prm.out_off[q] = out_off;
      out_off += S * C;
      if (S > 0 && C > 0) tiles += (S + vf::span::kTile - 1) / vf::span::kTile;
      if (tiles >= (1LL << 31)) return sfail(VF_EUNSUPPORTED, "too many span tiles in one launch");
    }
    prm.tile_off[n] = static_cast<int>(tiles);
    prm.nseg = n;
    if (tiles == 0) continue;
    const int rc = a->dtype == VF_DTYPE_BF16
                       ? launch_span<__nv_bfloat16>(prm, static_cast<unsigned>(tiles), ych, smem, s)
                       : launch_span<__half>(prm, static_cast<unsigned>(tiles), ych, smem, s);
    if (rc != VF_OK) return rc;
  }
  return VF_OK;
}

}  // extern "C"
