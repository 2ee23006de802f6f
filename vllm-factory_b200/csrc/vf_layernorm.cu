// sm_100a residual add + LayerNorm of the DeBERTa-v2 encoder: out = LayerNorm(x + residual).
//
// Replaces the two torch kernels of models/deberta_v2/deberta_v2_encoder.py:507 and :566
// (DebertaV2SelfOutput / DebertaV2Output: `self.LayerNorm(hidden_states + input_tensor)`,
// nn.LayerNorm with weight and bias), which write the sum to HBM and read it back.  Here
// one pass reads x and the residual and writes the result: 3 x rows x cols elements of
// traffic instead of ~5, HBM-bound.
//
// Semantics kept from the reference: the sum is rounded to the input dtype (torch adds two
// 16-bit tensors into a 16-bit tensor before the norm); mean and biased variance of that
// rounded sum in fp32; y = (s - mean) * rsqrt(var + eps) * weight + bias in fp32, rounded
// to the dtype.  Mean and variance are two passes over the row held in registers, so the
// variance never suffers the cancellation of E[s^2] - mean^2.
//
// Layout: one warp per row.  Each lane holds NV 16-byte vectors of the row (lane + 32 i),
// so every load instruction of a warp covers 512 contiguous bytes; weight and bias are
// read per row through L1, where they stay.  Rows
// whose columns or addresses do not allow 16-byte vectors, or that are too wide for the
// register-held form, go through a scalar kernel that re-reads the row from cache.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <string>

#include "../../include/vf_b200.h"

namespace vf {
namespace {

template <typename T> struct LnElem;
template <> struct LnElem<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float ldg(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ float from(float v) { return v; }
};
template <> struct LnElem<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ float ldg(const __half* p) { return __half2float(__ldg(p)); }
  static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
};
template <> struct LnElem<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ float ldg(const __nv_bfloat16* p) { return __bfloat162float(__ldg(p)); }
  static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
};

struct AddNormView {
  const void* x;
  const void* res;
  const void* w;
  const void* b;     // may be null
  void* out;
  long long rows, cols;
  long long xs, rs, os;   // row strides in elements
  float eps;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Register-held rows: cols % kV == 0 and cols / kV <= 32 * NV.  Up to 4 vectors per lane
// the kernel fits 3 resident blocks of 256 threads per SM (<= 85 registers, no spills).
template <typename T, int NV>
__global__ void __launch_bounds__(256, NV <= 4 ? 3 : 1) add_layer_norm_vec_kernel(const AddNormView v) {
  constexpr int kV = 16 / sizeof(T);
  const int lane = threadIdx.x & 31;
  const long long warp0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const int vpr = static_cast<int>(v.cols / kV);
  const T* xg = static_cast<const T*>(v.x);
  const T* rg = static_cast<const T*>(v.res);
  T* og = static_cast<T*>(v.out);
  const float inv_cols = 1.0f / static_cast<float>(v.cols);


  for (long long r = warp0; r < v.rows; r += nwarps) {
    const T* xr = xg + r * v.xs;
    const T* rr = rg + r * v.rs;
    uint4 x4[NV], r4[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int cv = lane + 32 * i;
      x4[i] = r4[i] = make_uint4(0, 0, 0, 0);
      if (cv < vpr) {
        x4[i] = __ldg(reinterpret_cast<const uint4*>(xr) + cv);
        r4[i] = __ldg(reinterpret_cast<const uint4*>(rr) + cv);
      }
    }
    float s[NV][kV];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int cv = lane + 32 * i;
      const T* xe = reinterpret_cast<const T*>(&x4[i]);
      const T* re = reinterpret_cast<const T*>(&r4[i]);
#pragma unroll
      for (int j = 0; j < kV; ++j) {
        // the sum rounded to the dtype, as the reference's tensor add stores it
        s[i][j] = cv < vpr ? LnElem<T>::f(LnElem<T>::from(LnElem<T>::f(xe[j]) + LnElem<T>::f(re[j]))) : 0.0f;
        sum += s[i][j];
      }
    }
    const float mean = warp_sum(sum) * inv_cols;
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int cv = lane + 32 * i;
#pragma unroll
      for (int j = 0; j < kV; ++j) {
        const float d = s[i][j] - mean;
        sq += cv < vpr ? d * d : 0.0f;
      }
    }
    const float rstd = rsqrtf(warp_sum(sq) * inv_cols + v.eps);
    T* orow = og + r * v.os;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int cv = lane + 32 * i;
      if (cv >= vpr) continue;
      // weight and bias per row from L1 (a few KB shared by every row): holding them in
      // registers instead cost 48 registers and one resident block per SM (2.7 % slower)
      const uint4 w4 = __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(v.w)) + cv);
      const uint4 b4 = v.b != nullptr ? __ldg(reinterpret_cast<const uint4*>(static_cast<const T*>(v.b)) + cv)
                                      : make_uint4(0, 0, 0, 0);
      const T* we = reinterpret_cast<const T*>(&w4);
      const T* be = reinterpret_cast<const T*>(&b4);
      uint4 o4;
      T* oe = reinterpret_cast<T*>(&o4);
#pragma unroll
      for (int j = 0; j < kV; ++j)
        oe[j] = LnElem<T>::from((s[i][j] - mean) * rstd * LnElem<T>::f(we[j]) + LnElem<T>::f(be[j]));
      reinterpret_cast<uint4*>(orow)[cv] = o4;
    }
  }
}

// Any width and alignment: one warp per row, three passes over the row (sum, squared
// deviations, output), the second and third from cache.
template <typename T>
__global__ void __launch_bounds__(256) add_layer_norm_scalar_kernel(const AddNormView v) {
  const int lane = threadIdx.x & 31;
  const long long warp0 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const T* xg = static_cast<const T*>(v.x);
  const T* rg = static_cast<const T*>(v.res);
  const T* wg = static_cast<const T*>(v.w);
  const T* bg = static_cast<const T*>(v.b);
  T* og = static_cast<T*>(v.out);
  const float inv_cols = 1.0f / static_cast<float>(v.cols);
  for (long long r = warp0; r < v.rows; r += nwarps) {
    const T* xr = xg + r * v.xs;
    const T* rr = rg + r * v.rs;
    auto at = [&](long long c) {
      return LnElem<T>::f(LnElem<T>::from(LnElem<T>::ldg(xr + c) + LnElem<T>::ldg(rr + c)));
    };
    float sum = 0.0f;
    for (long long c = lane; c < v.cols; c += 32) sum += at(c);
    const float mean = warp_sum(sum) * inv_cols;
    float sq = 0.0f;
    for (long long c = lane; c < v.cols; c += 32) {
      const float d = at(c) - mean;
      sq += d * d;
    }
    const float rstd = rsqrtf(warp_sum(sq) * inv_cols + v.eps);
    T* orow = og + r * v.os;
    for (long long c = lane; c < v.cols; c += 32) {
      const float bias = bg != nullptr ? LnElem<T>::ldg(bg + c) : 0.0f;
      orow[c] = LnElem<T>::from((at(c) - mean) * rstd * LnElem<T>::ldg(wg + c) + bias);
    }
  }
}

}  // namespace
int set_last_error(int code, const std::string& msg);   // vf_attention.cu: feeds vf_last_error()
namespace {

int ln_fail(int code, const std::string& msg) { return set_last_error(code, msg); }

template <typename Kernel>
unsigned grid_for(Kernel k, long long rows, int threads) {
  int dev = 0, sm_count = 0, per_sm = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sm_count <= 0)
    sm_count = 148;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, threads, 0) != cudaSuccess || per_sm <= 0) per_sm = 1;
  // One resident wave of blocks (a multiple of the SM count); warps stride over the rows.
  const long long warps_per_block = threads / 32;
  const long long need = (rows + warps_per_block - 1) / warps_per_block;
  return static_cast<unsigned>(std::max<long long>(1, std::min<long long>(need, (long long)sm_count * per_sm)));
}

template <typename T>
int launch_add_norm(const AddNormView& v, cudaStream_t s) {
  constexpr int kV = 16 / sizeof(T);
  constexpr int kThreads = 256;
  const int es = sizeof(T);
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const long long vpr = v.cols / kV;
  const bool vec = v.cols % kV == 0 && vpr <= 32LL * 8 && al16(v.x) && al16(v.res) && al16(v.out) && al16(v.w) &&
                   (v.b == nullptr || al16(v.b)) && (v.xs * es) % 16 == 0 && (v.rs * es) % 16 == 0 &&
                   (v.os * es) % 16 == 0;
  if (vec) {
    if (vpr <= 32) {
      add_layer_norm_vec_kernel<T, 1><<<grid_for(add_layer_norm_vec_kernel<T, 1>, v.rows, kThreads), kThreads, 0, s>>>(v);
    } else if (vpr <= 64) {
      add_layer_norm_vec_kernel<T, 2><<<grid_for(add_layer_norm_vec_kernel<T, 2>, v.rows, kThreads), kThreads, 0, s>>>(v);
    } else if (vpr <= 128) {
      add_layer_norm_vec_kernel<T, 4><<<grid_for(add_layer_norm_vec_kernel<T, 4>, v.rows, kThreads), kThreads, 0, s>>>(v);
    } else {
      add_layer_norm_vec_kernel<T, 8><<<grid_for(add_layer_norm_vec_kernel<T, 8>, v.rows, kThreads), kThreads, 0, s>>>(v);
    }
  } else {
    add_layer_norm_scalar_kernel<T><<<grid_for(add_layer_norm_scalar_kernel<T>, v.rows, kThreads), kThreads, 0, s>>>(v);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ln_fail(VF_ECUDA, std::string("add layer norm launch: ") + cudaGetErrorString(e));
  return VF_OK;
}

}  // namespace
}  // namespace vf

extern "C" {

int vf_add_layer_norm_fwd(const vf_add_layer_norm_args_t* a, void* stream) {
  using vf::ln_fail;
  if (a == nullptr) return ln_fail(VF_EINVAL, "null args");
  if (a->rows < 0 || a->cols < 0) return ln_fail(VF_EINVAL, "add layer norm: negative sizes");
  if (a->rows == 0 || a->cols == 0) return VF_OK;
  if (!a->x || !a->residual || !a->weight || !a->out)
    return ln_fail(VF_EINVAL, "add layer norm: x, residual, weight and out must be non-null");
  if (a->x_row_stride < a->cols || a->residual_row_stride < a->cols || a->out_row_stride < a->cols)
    return ln_fail(VF_EINVAL, "add layer norm: row strides must be at least cols (rows must not overlap)");
  if (!std::isfinite(a->eps) || a->eps < 0.0f) return ln_fail(VF_EINVAL, "add layer norm: eps must be finite and >= 0");
  vf::AddNormView v{a->x, a->residual, a->weight, a->bias, a->out, a->rows, a->cols,
                    a->x_row_stride, a->residual_row_stride, a->out_row_stride, a->eps};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case VF_DTYPE_BF16: return vf::launch_add_norm<__nv_bfloat16>(v, s);
    case VF_DTYPE_F16: return vf::launch_add_norm<__half>(v, s);
    case VF_DTYPE_F32: return vf::launch_add_norm<float>(v, s);
    default: return ln_fail(VF_EUNSUPPORTED, "add layer norm: dtype must be float32, float16 or bfloat16");
  }
}

}  // extern "C"
