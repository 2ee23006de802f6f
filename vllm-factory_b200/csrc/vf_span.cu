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
// shared memory, 64 K-columns per stage, and multiplies it by the TMA-staged class rows on
// the tensor cores.  The reference's [spans, 2D] / [spans, 4D] / [spans, D] intermediates
// never exist.
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
constexpr int kKStep = 64;             // K elements per stage: one 128-byte swizzled row per span
constexpr int kStages = 4;
constexpr int kThreads = 192;          // warps 0-3 rows + epilogue, warp 4 TMA, warp 5 UMMA
constexpr int kATile = kTile * 128;    // 16 KB of A per stage
constexpr int kMaxN = 256;             // classes per CTA (UMMA N)
constexpr int kMaxSeg = 256;           // segments per launch (kernel-parameter tables)
constexpr int kSmemMax = 1024 + kStages * (kATile + kMaxN * 128) + 256;

struct __align__(64) Params {
  CUtensorMap tm_cls;                  // classes [C_total, K], box 64 x npad, 128-byte swizzle
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
__global__ void __launch_bounds__(kThreads) span_scores_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int npad = p.npad;
  uint8_t* sA = smem;                                   // [kStages][128 rows x 128 B], 128-byte swizzle
  uint8_t* sB = smem + kStages * kATile;                // [kStages][npad rows x 128 B], written by TMA
  uint64_t* full_a = reinterpret_cast<uint64_t*>(sB + kStages * npad * 128);
  uint64_t* full_b = full_a + kStages;
  uint64_t* empty = full_b + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, static_cast<uint32_t>(p.tmem_cols));
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    // ---------------------------------------------------------------- A rows + epilogue
    const int t = threadIdx.x;                                // span row of the tile == TMEM lane
    const int sl = min(s_begin + t, S_g - 1);                 // rows past the segment repeat its last span
    const long long srow = p.span_off[g] + sl;
    long long i, j;
    if (p.idx64) {
      const long long* ix = reinterpret_cast<const long long*>(p.idx) + srow * p.idx_ss;
      i = __ldg(ix);
      j = __ldg(ix + p.idx_sp);
    } else {
      const int* ix = reinterpret_cast<const int*>(p.idx) + srow * p.idx_ss;
      i = __ldg(ix);
      j = __ldg(ix + p.idx_sp);
    }
    // The reference gathers with indices clamped to the sentence's words (extract_elements).
    const long long last = p.word_len[g] - 1;
    i = min(max(i, 0LL), last);
    j = min(max(j, 0LL), last);
    const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.u) + (p.word_off[g] + i) * p.us);
    const uint4* vr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.v) + (p.word_off[g] + j) * p.vs);
    const uint32_t sw = static_cast<uint32_t>(t & 7);
    bool ok = true;
    for (int kc = 0; kc < nk; ++kc) {
      const int st = kc % kStages;
      uint4 a[8], b[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        a[q] = __ldg(ur + kc * 8 + q);
        b[q] = __ldg(vr + kc * 8 + q);
      }
      if (kc >= kStages) {
        ok = mbar_wait(&empty[st], ((kc / kStages) - 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      }
      uint8_t* row = sA + st * kATile + t * 128;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint4 r;
        r.x = add_relu2<T>(a[q].x, b[q].x);
        r.y = add_relu2<T>(a[q].y, b[q].y);
        r.z = add_relu2<T>(a[q].z, b[q].z);
        r.w = add_relu2<T>(a[q].w, b[q].w);
        *reinterpret_cast<uint4*>(row + ((static_cast<uint32_t>(q) ^ sw) << 4)) = r;   // 16-byte chunk q of row t
      }
      fence_proxy_async_smem();
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
        tmem_ld_x16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + cc, r);   // collective: every lane
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
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % kStages;
        if (kc >= kStages && !mbar_wait(&empty[st], ((kc / kStages) - 1) & 1, abort_flag)) break;
        mbar_arrive_expect_tx(&full_b[st], static_cast<uint32_t>(npad * 128));
        tma_load_2d(sB + st * npad * 128, &p.tm_cls, &full_b[st], kc * kKStep, crow);
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
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
      for (int kc = 0; kc < nk; ++kc) {
        const int st = kc % kStages;
        const uint32_t par = (kc / kStages) & 1;
        if (!mbar_wait(&full_a[st], par, abort_flag) || !mbar_wait(&full_b[st], par, abort_flag)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kKStep / 16; ++kk) {
          const uint64_t ad = smem_desc_sw128(a0 + st * kATile + kk * 32, 16, 1024);
          const uint64_t bd = smem_desc_sw128(b0 + st * npad * 128 + kk * 32, 16, 1024);
          umma_ss(tmem, ad, bd, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
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
  while (tcols < npad) tcols *= 2;

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
  const int smem = 1024 + vf::span::kStages * (vf::span::kATile + npad * 128) + 256;
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
