// Linear + activation GEMMs with the activation in the epilogue, on sm_100a (hand-written:
// TMA tile loads, tcgen05 UMMA into a TMEM accumulator, TMA tile stores):
//   act = GELU_ERF:  out = GELU(x W^T + b)          the DeBERTa feed-forward's first half,
//                    models/deberta_v2/deberta_v2_encoder.py:547-550 (DebertaV2Intermediate:
//                    `self.dense`, then ACT2FN["gelu"], torch's exact GELU);
//   act = GELU_TANH: out = GELU_tanh(x W^T) * mul   the mT5 gated feed-forward,
//                    models/mt5/mt5_encoder.py:427-437 with kernels/ff_fused.py:86 ("gelu_new"):
//                    W = wi_0 (gate), mul = x wi_1^T (up).
// The reference writes the projection to HBM and an elementwise pass reads it back; here the
// activation runs on the fp32 accumulator before the one rounding to the output dtype, so the
// intermediate never exists.
//
// Persistent kernel, one CTA per SM, 320 threads:
//   warp 0      TMA producer: per 64-wide K step, a 128 x 64 tile of x and a 256 x 64 tile of
//               W (2-D maps, 128-byte swizzle, plain single-CTA loads) into a 4-stage ring;
//   warp 1      TMEM owner and UMMA issuer: four M = 128, N = 256, K = 16 tcgen05.mma per K step
//               into one of two 256-column fp32 accumulators (tile i uses i & 1, so the epilogue
//               of one tile overlaps the main loop of the next);
//   warps 2-9   epilogue, two groups of four warps (one per TMEM lane quadrant), group g taking
//               columns [128 g, 128 g + 128) of the tile in 64-column chunks: TMEM -> registers,
//               bias + exact GELU or GELU_tanh * mul in fp32, 16-bit pack, a 128 x 64 staging
//               tile (128-byte swizzle) and one TMA store per chunk.
// Output tiles go in N-fastest order, so the CTAs working at one time share a block of x (read
// from HBM once) and the whole W stays in L2.  Every wait is bounded; a group leaves its loop
// only by a decision all its threads take together (barrier reduction), so no named barrier
// is left waiting.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "vf_internal.h"
#include "vf_ptx.cuh"

namespace vf {
namespace gemm {

constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kStages = 4;
constexpr int kThreads = 320;
constexpr int kEpiThreads = 256;
constexpr int kATile = kBM * kBK * 2;          // 16 KB
constexpr int kBTile = kBN * kBK * 2;          // 32 KB
constexpr int kStage = kBM * 64 * 2;           // 16 KB: one 128 x 64 output chunk
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kATile;
constexpr int kOffStage = kOffB + kStages * kBTile;
constexpr int kOffBar = kOffStage + 2 * kStage;
constexpr int kBytes = kOffBar + 256;
constexpr int kAlloc = kBytes + 1024;
static_assert(kAlloc <= 227 * 1024, "shared memory over the per-CTA limit");

struct __align__(64) Params {
  CUtensorMap tm_x, tm_w, tm_out;
  const void* bias;     // [N] (GELU_ERF)
  const void* mul;      // [M, N] (GELU_TANH), row stride mul_rs
  long long mul_rs;
  int M, N, K, num_n, tiles;
};

template <typename T> struct Pack;
template <> struct Pack<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t two(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  static __device__ __forceinline__ float f(uint16_t u) { return __uint_as_float(static_cast<uint32_t>(u) << 16); }
};
template <> struct Pack<__half> {
  static __device__ __forceinline__ uint32_t two(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  static __device__ __forceinline__ float f(uint16_t u) { return __half2float(__ushort_as_half(u)); }
};
template <typename T> struct Fmt;
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t value = 1u; };
template <> struct Fmt<__half> { static constexpr uint32_t value = 0u; };

// Exact GELU, z Phi(z) with Phi(z) = (1 + erf(z / sqrt 2)) / 2, as torch's F.gelu defines it.
// erfc(a), a = |z| / sqrt 2 >= 0, by Abramowitz & Stegun 7.1.26 (Handbook of Mathematical
// Functions, 1964): erfc(a) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^(-a^2), t = 1 / (1 + p a),
// absolute error <= 1.5e-7; then Phi(z) = 1 - erfc(a) / 2 for z >= 0 and erfc(a) / 2 below.
// Two pairs of MUFU operations (reciprocal, exponential) and packed fp32 arithmetic per pair.
__device__ __forceinline__ float2 gelu_erf2(float2 z) {
  const float2 a = make_float2(fabsf(z.x) * 0.7071067811865476f, fabsf(z.y) * 0.7071067811865476f);
  const float2 d = __ffma2_rn(a, make_float2(0.3275911f, 0.3275911f), make_float2(1.f, 1.f));
  const float2 t = make_float2(__fdividef(1.f, d.x), __fdividef(1.f, d.y));
  float2 s = __ffma2_rn(make_float2(1.061405429f, 1.061405429f), t, make_float2(-1.453152027f, -1.453152027f));
  s = __ffma2_rn(s, t, make_float2(1.421413741f, 1.421413741f));
  s = __ffma2_rn(s, t, make_float2(-0.284496736f, -0.284496736f));
  s = __ffma2_rn(s, t, make_float2(0.254829592f, 0.254829592f));
  s = __fmul2_rn(s, t);
  const float2 a2 = __fmul2_rn(a, a);
  const float2 e = make_float2(ex2_approx(a2.x * -1.4426950408889634f), ex2_approx(a2.y * -1.4426950408889634f));
  const float2 h = __fmul2_rn(__fmul2_rn(s, e), make_float2(0.5f, 0.5f));   // erfc(a) / 2
  const float2 phi = make_float2(z.x >= 0.f ? 1.f - h.x : h.x, z.y >= 0.f ? 1.f - h.y : h.y);
  return __fmul2_rn(z, phi);
}
// GELU with the tanh form, z (1 + tanh u) / 2 = z / (1 + e^(-2u)), u = sqrt(2/pi) (z + 0.044715 z^3):
// the identity the reference kernel uses (2 sigmoid(2u) - 1 for tanh u).
__device__ __forceinline__ float gelu_tanh(float z) {
  const float u2 = 1.5957691216057308f * (z + 0.044715f * z * z * z);
  return __fdividef(z, 1.0f + __expf(-u2));
}
__device__ __forceinline__ float2 gelu_tanh2(float2 z) { return make_float2(gelu_tanh(z.x), gelu_tanh(z.y)); }

template <typename T, bool kGated>
__global__ void __launch_bounds__(kThreads, 1) linear_act_kernel(const __grid_constant__ Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kOffBar);   // [kStages] x and W tiles landed
  uint64_t* empty = full + kStages;                                 // [kStages] the MMAs reading them completed
  uint64_t* acc_full = empty + kStages;                             // [2] accumulator holds a finished tile
  uint64_t* acc_empty = acc_full + 2;                               // [2] the epilogue has read it
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiThreads);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.tm_x);
    tma_prefetch_desc(&p.tm_w);
    tma_prefetch_desc(&p.tm_out);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const int m0 = (t / p.num_n) * kBM, n0 = (t % p.num_n) * kBN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kStages;
          if (it >= kStages && !mbar_wait(&empty[st], ((it / kStages) - 1) & 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[st], kATile + kBTile);
          tma_load_2d(smem + kOffA + st * kATile, &p.tm_x, &full[st], kb * kBK, m0);
          tma_load_2d(smem + kOffB + st * kBTile, &p.tm_w, &full[st], kb * kBK, n0);
        }
      }
      // No TMA write may land after the CTA exits: wait for the last fills (time-bounded).
      for (int j = max(it - kStages, 0); j < it; ++j) mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(Fmt<T>::value, kBM, kBN, 0, 0);
      const uint32_t sA = smem_u32(smem + kOffA), sB = smem_u32(smem + kOffB);
      int it = 0, li = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x, ++li) {
        const int acc = li & 1;
        if (li >= 2 && !mbar_wait(&acc_empty[acc], ((li >> 1) - 1) & 1, abort_flag)) break;
        tc_fence_after();
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int st = it % kStages;
          if (!mbar_wait(&full[st], (it / kStages) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sA + st * kATile + kk * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sB + st * kBTile + kk * 32, 16, 1024);
            umma_ss(tmem + static_cast<uint32_t>(acc * kBN), ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[st]);
        }
        if (ok) umma_commit(&acc_full[acc]);
      }
      // Every MMA issued above has completed before TMEM is released.
      umma_commit(drain);
      mbar_wait_bounded(drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    const int grp = (warp - 2) >> 2;                        // columns [128 grp, 128 grp + 128)
    const int row = (warp & 3) * 32 + lane;                 // tile row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const bool issuer = (threadIdx.x & 127) == 64;          // one thread of the group (lane 0 of its first warp)
    uint8_t* stg = smem + kOffStage + grp * kStage;
    uint8_t* srow = stg + row * 128;
    const uint32_t bar_id = 1 + grp;
    // The 64 columns [col0, col0 + 64) of the row's second operand (mul row for the gated form,
    // the bias for the other; zero past the matrix), as 8 x 16 bytes.
    const auto load_extra = [&](int grow, int col0, uint4 (&w)[8]) {
      const T* src = kGated ? static_cast<const T*>(p.mul) + (long long)min(grow, p.M - 1) * p.mul_rs + col0
                            : static_cast<const T*>(p.bias) + col0;
      const bool in_rows = !kGated || grow < p.M;
      if (in_rows && col0 + 64 <= p.N) {
#pragma unroll
        for (int q = 0; q < 8; ++q) w[q] = __ldg(reinterpret_cast<const uint4*>(src) + q);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          uint16_t h[8];
#pragma unroll
          for (int e = 0; e < 8; ++e)
            h[e] = in_rows && col0 + 8 * q + e < p.N ? __ldg(reinterpret_cast<const unsigned short*>(src) + 8 * q + e) : 0;
          w[q] = make_uint4(h[0] | (uint32_t(h[1]) << 16), h[2] | (uint32_t(h[3]) << 16),
                            h[4] | (uint32_t(h[5]) << 16), h[6] | (uint32_t(h[7]) << 16));
        }
      }
    };
    int li = 0;
    uint4 wcur[8], wnext[8];
    if constexpr (kGated) {
      const int t = blockIdx.x;
      if (t < p.tiles) load_extra((t / p.num_n) * kBM + row, (t % p.num_n) * kBN + grp * 128, wcur);
    }
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x, ++li) {
      const int acc = li & 1;
      const int m0 = (t / p.num_n) * kBM, n0 = (t % p.num_n) * kBN;
      bool ok = mbar_wait(&acc_full[acc], (li >> 1) & 1, abort_flag);
      if (named_bar_any(bar_id, 128, !ok)) break;
      tc_fence_after();
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int c0 = grp * 128 + cc * 64;                 // first column of the chunk in the tile
        const int col0 = n0 + c0;
        uint32_t r[64];
        tmem_ld_x64(tmem + lane_base + static_cast<uint32_t>(acc * kBN + c0), r);
        if (cc == 1) {
          tc_fence_before();
          mbar_arrive(&acc_empty[acc]);                     // the tile's columns are in registers
        }
        if constexpr (kGated) {
          // The next chunk's mul row is loaded now, one chunk ahead of its use (for the last
          // chunk: the first chunk of this CTA's next tile).
          if (cc == 0) {
            load_extra(m0 + row, col0 + 64, wnext);
          } else {
            const int tn = t + gridDim.x;
            if (tn < p.tiles) load_extra((tn / p.num_n) * kBM + row, (tn % p.num_n) * kBN + grp * 128, wnext);
          }
        } else {
          load_extra(0, col0, wcur);                        // the bias: the same 64 values for every row
        }
        // The group's staging tile is free once its previous store has read it.
        if (issuer) bulk_wait_read<0>();
        named_bar_sync(bar_id, 128);
#pragma unroll
        for (int q = 0; q < 8; ++q) {   // 16-byte chunk q of the row at q ^ (row & 7): the store map's 128-byte swizzle
          const uint32_t ws[4] = {wcur[q].x, wcur[q].y, wcur[q].z, wcur[q].w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 8 * q + 2 * e;
            const float2 z = make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1]));
            const float2 b = make_float2(Pack<T>::f(static_cast<uint16_t>(ws[e] & 0xffffu)),
                                         Pack<T>::f(static_cast<uint16_t>(ws[e] >> 16)));
            const float2 y = kGated ? __fmul2_rn(gelu_tanh2(z), b) : gelu_erf2(__fadd2_rn(z, b));
            o[e] = Pack<T>::two(y.x, y.y);
          }
          *reinterpret_cast<uint4*>(srow + ((q ^ (row & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        }
        if constexpr (kGated) {
#pragma unroll
          for (int q = 0; q < 8; ++q) wcur[q] = wnext[q];
        }
        fence_proxy_async_smem();
        named_bar_sync(bar_id, 128);
        if (issuer && col0 < p.N) {
          tma_store_2d(&p.tm_out, stg, col0, m0);           // rows / columns past the output are not written
          bulk_commit();
        }
      }
    }
    if (issuer) bulk_wait_all();
  }
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace gemm

// Error word of this file (vf_device_error gathers it).
cudaError_t gemm_take_error_word(bool clear, unsigned int* word) { return take_error_word(clear, word); }

}  // namespace vf

// =====================================================================================
// Host side.
// =====================================================================================
namespace {

int gfail(int code, const std::string& msg) { return vf::set_last_error(code, "linear act: " + msg); }

int make_map(CUtensorMap* map, const void* base, long long inner, long long rows, long long row_stride,
             vf_dtype_t dt, int box_rows, const char* name) {
  auto enc = vf::host_encode_fn();
  if (enc == nullptr) return gfail(VF_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType ty = dt == VF_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = enc(map, ty, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return gfail(VF_ECUDA, std::string(name) + " map: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
  return VF_OK;
}

template <typename T, bool kGated>
int launch_gemm(const vf::gemm::Params& prm, cudaStream_t s) {
  auto kern = vf::gemm::linear_act_kernel<T, kGated>;
  int dev = 0;
  cudaGetDevice(&dev);
  static std::once_flag flags[64];
  static cudaError_t attr_err[64];
  static int sm_count[64];
  if (dev < 0 || dev >= 64) return gfail(VF_ECUDA, "device ordinal out of range");
  std::call_once(flags[dev], [&] {
    attr_err[dev] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, vf::gemm::kAlloc);
    if (attr_err[dev] == cudaSuccess) attr_err[dev] = cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
  });
  if (attr_err[dev] != cudaSuccess) return gfail(VF_ECUDA, std::string("kernel set-up: ") + cudaGetErrorString(attr_err[dev]));
  const int grid = std::min(prm.tiles, std::max(sm_count[dev], 1));
  kern<<<grid, vf::gemm::kThreads, vf::gemm::kAlloc, s>>>(prm);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gfail(VF_ECUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
  return VF_OK;
}

}  // namespace

extern "C" {

int vf_linear_act_fwd(const vf_linear_act_args_t* a, void* stream) {
  if (a == nullptr) return gfail(VF_EINVAL, "null args");
  if (a->dtype != VF_DTYPE_BF16 && a->dtype != VF_DTYPE_F16) return gfail(VF_EUNSUPPORTED, "dtype must be float16 or bfloat16");
  const bool gated = a->act == VF_ACT_GELU_TANH;
  if (a->act != VF_ACT_GELU_ERF && !gated)
    return gfail(VF_EUNSUPPORTED, "the built forms are VF_ACT_GELU_ERF (+ bias) and VF_ACT_GELU_TANH (x mul)");
  if (a->rows < 0 || a->K <= 0 || a->N <= 0) return gfail(VF_EINVAL, "rows >= 0, K > 0, N > 0");
  if (a->rows >= (1LL << 31) || a->K >= (1LL << 31) || a->N >= (1LL << 31))
    return gfail(VF_EUNSUPPORTED, "sizes must be below 2^31");
  if (a->rows == 0) return VF_OK;
  if (!a->x || !a->weight || !a->out) return gfail(VF_EINVAL, "x, weight and out must be non-null");
  if (gated ? (a->mul == nullptr || a->bias != nullptr) : (a->bias == nullptr || a->mul != nullptr))
    return gfail(VF_EINVAL, "VF_ACT_GELU_ERF takes a bias and no mul, VF_ACT_GELU_TANH a mul and no bias");
  if (a->x_row_stride < a->K || a->weight_row_stride < a->K || a->out_row_stride < a->N ||
      (gated && a->mul_row_stride < a->N))
    return gfail(VF_EINVAL, "row strides must be at least K (x, weight) and N (out, mul)");
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const void* extra = gated ? a->mul : a->bias;
  if (a->K % 8 != 0 || a->N % 8 != 0 || a->x_row_stride % 8 != 0 || a->weight_row_stride % 8 != 0 ||
      a->out_row_stride % 8 != 0 || (gated && a->mul_row_stride % 8 != 0) || !al16(a->x) || !al16(a->weight) ||
      !al16(extra) || !al16(a->out))
    return gfail(VF_EINVAL, "K, N, row strides must be multiples of 8 and pointers 16-byte aligned");
  vf::gemm::Params prm{};
  int rc;
  if ((rc = make_map(&prm.tm_x, a->x, a->K, a->rows, a->x_row_stride, a->dtype, vf::gemm::kBM, "x"))) return rc;
  if ((rc = make_map(&prm.tm_w, a->weight, a->K, a->N, a->weight_row_stride, a->dtype, vf::gemm::kBN, "weight"))) return rc;
  if ((rc = make_map(&prm.tm_out, a->out, a->N, a->rows, a->out_row_stride, a->dtype, vf::gemm::kBM, "out"))) return rc;
  prm.bias = a->bias;
  prm.mul = a->mul;
  prm.mul_rs = a->mul_row_stride;
  prm.M = static_cast<int>(a->rows);
  prm.N = static_cast<int>(a->N);
  prm.K = static_cast<int>(a->K);
  prm.num_n = static_cast<int>((a->N + vf::gemm::kBN - 1) / vf::gemm::kBN);
  const long long tiles = (long long)prm.num_n * ((a->rows + vf::gemm::kBM - 1) / vf::gemm::kBM);
  if (tiles >= (1LL << 31)) return gfail(VF_EUNSUPPORTED, "too many output tiles");
  prm.tiles = static_cast<int>(tiles);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gated)
    return a->dtype == VF_DTYPE_BF16 ? launch_gemm<__nv_bfloat16, true>(prm, s) : launch_gemm<__half, true>(prm, s);
  return a->dtype == VF_DTYPE_BF16 ? launch_gemm<__nv_bfloat16, false>(prm, s) : launch_gemm<__half, false>(prm, s);
}

}  // extern "C"
