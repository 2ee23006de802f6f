// sm_100a gated activation of the mT5 feed-forward: out = act(gate) * up; with up = NULL
// the plain activation out = act(gate) (the DeBERTa feed-forward's exact GELU).
//
// Replaces the Triton kernel behind kernels/ff_fused.py:86 `fused_gelu_mul_dropout`
// (_fused_gelu_mul_dropout_kernel, :23-74) on its inference path: activation in fp32
// (GELU with the tanh form, exact GELU, ReLU or SiLU), product with `up` in fp32, result
// rounded to the input dtype.  The reference flattens both operands to contiguous copies;
// here gate, up and out are 2-D views (rows x cols, unit column stride, any row stride),
// so the two halves of a stacked [T, 2F] projection are read in place.
//
// The op moves 3 x rows x cols elements and does ~20 flops per element: it is HBM-bound.
// Each thread handles 16-byte vectors (8 x 16-bit or 4 x fp32) with read-only loads;
// the grid is a multiple of the SM count and strides over the vectors.  Views whose
// columns or addresses do not allow 16-byte vectors go through a scalar kernel.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <string>

#include "../../include/vf_b200.h"

namespace vf {
namespace {

// Activation in fp32.  GELU (tanh form) is the published approximation
// 0.5 x (1 + tanh(z)), z = sqrt(2/pi) (x + 0.044715 x^3) (Hendrycks & Gimpel), written as
// x * sigmoid(2z) = x / (1 + e^(-2z)) -- the identity 1 + tanh(z) = 2 sigmoid(2z) that the
// reference kernel also uses (:50-53) -- with the fast exponential and division: one MUFU
// exponential and one reciprocal per element keep the kernel on the HBM roofline.  For
// e^(-2z) = inf the fast division returns 0, the limit.  SiLU x / (1 + e^(-x)) alike; the
// exact GELU keeps erf.
__device__ __forceinline__ float act_f(float x, int act) {
  switch (act) {
    case VF_ACT_GELU_TANH: {
      const float z2 = 1.5957691216057308f * (x + 0.044715f * x * x * x);   // 2 sqrt(2/pi) (...)
      return __fdividef(x, 1.0f + __expf(-z2));
    }
    case VF_ACT_GELU_ERF:
      return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
    case VF_ACT_RELU:
      return fmaxf(x, 0.0f);
    default:   // VF_ACT_SILU
      return __fdividef(x, 1.0f + __expf(-x));
  }
}

// Element conversions: `f` converts a value already in registers, `ldg` reads one element
// of global memory through the read-only path, `from` rounds an fp32 result.
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float f(float v) { return v; }
  static __device__ __forceinline__ float ldg(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ float from(float v) { return v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ float ldg(const __half* p) { return __half2float(__ldg(p)); }
  static __device__ __forceinline__ __half from(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ float ldg(const __nv_bfloat16* p) { return __bfloat162float(__ldg(p)); }
  static __device__ __forceinline__ __nv_bfloat16 from(float v) { return __float2bfloat16_rn(v); }
};

struct GatedView {
  const void* gate;
  const void* up;
  void* out;
  long long rows, cols;
  long long gs, us, os;   // row strides in elements
  int act;
};

// 16-byte vectors: kV elements of T.  Requires cols % kV == 0, 16-byte aligned bases and
// row strides (checked on the host).  The activation is a template parameter.
template <typename T, int kAct, bool kGated>
__global__ void gated_act_vec_kernel(const GatedView v) {
  constexpr int kV = 16 / sizeof(T);
  const long long vpr = v.cols / kV;                 // vectors per row
  const long long nvec = v.rows * vpr;
  const T* gate = static_cast<const T*>(v.gate);
  const T* up = static_cast<const T*>(v.up);
  T* out = static_cast<T*>(v.out);
  // Grid-stride over vectors with the (row, vector) position stepped incrementally: one
  // division per thread instead of one per vector.
  const long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i0 >= nvec) return;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long dr = stride / vpr, dc = stride - dr * vpr;
  long long r = i0 / vpr, cv = i0 - r * vpr;
  for (; r < v.rows; r += dr, cv += dc) {
    if (cv >= vpr) { cv -= vpr; ++r; if (r >= v.rows) break; }
    const long long c = cv * kV;
    const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(gate + r * v.gs + c));
    const uint4 u4 = kGated ? __ldg(reinterpret_cast<const uint4*>(up + r * v.us + c)) : make_uint4(0, 0, 0, 0);
    const T* g = reinterpret_cast<const T*>(&g4);
    const T* u = reinterpret_cast<const T*>(&u4);
    uint4 o4;
    T* o = reinterpret_cast<T*>(&o4);
#pragma unroll
    for (int j = 0; j < kV; ++j) {
      const float a = act_f(Elem<T>::f(g[j]), kAct);
      o[j] = Elem<T>::from(kGated ? a * Elem<T>::f(u[j]) : a);
    }
    *reinterpret_cast<uint4*>(out + r * v.os + c) = o4;
  }
}

template <typename T>
__global__ void gated_act_scalar_kernel(const GatedView v) {
  const long long n = v.rows * v.cols;
  const T* gate = static_cast<const T*>(v.gate);
  const T* up = static_cast<const T*>(v.up);
  T* out = static_cast<T*>(v.out);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / v.cols, c = i - r * v.cols;
    const float a = act_f(Elem<T>::ldg(gate + r * v.gs + c), v.act);
    out[r * v.os + c] = Elem<T>::from(up != nullptr ? a * Elem<T>::ldg(up + r * v.us + c) : a);
  }
}

}  // namespace
int set_last_error(int code, const std::string& msg);   // vf_attention.cu: feeds vf_last_error()
namespace {

int ffn_fail(int code, const std::string& msg) { return set_last_error(code, msg); }

template <typename T, bool kGated>
void launch_vec(const GatedView& v, unsigned nb, int threads, cudaStream_t s) {
  switch (v.act) {
    case VF_ACT_GELU_TANH: gated_act_vec_kernel<T, VF_ACT_GELU_TANH, kGated><<<nb, threads, 0, s>>>(v); break;
    case VF_ACT_GELU_ERF: gated_act_vec_kernel<T, VF_ACT_GELU_ERF, kGated><<<nb, threads, 0, s>>>(v); break;
    case VF_ACT_RELU: gated_act_vec_kernel<T, VF_ACT_RELU, kGated><<<nb, threads, 0, s>>>(v); break;
    default: gated_act_vec_kernel<T, VF_ACT_SILU, kGated><<<nb, threads, 0, s>>>(v); break;
  }
}

template <typename T>
int launch_gated(const GatedView& v, cudaStream_t s) {
  int dev = 0, sm_count = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sm_count <= 0)
    sm_count = 148;
  constexpr int kV = 16 / sizeof(T);
  const int es = sizeof(T);
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool gated = v.up != nullptr;
  const bool vec = v.cols % kV == 0 && al16(v.gate) && (!gated || al16(v.up)) && al16(v.out) &&
                   (v.gs * es) % 16 == 0 && (!gated || (v.us * es) % 16 == 0) && (v.os * es) % 16 == 0;
  const long long work = vec ? v.rows * (v.cols / kV) : v.rows * v.cols;
  const int threads = 256;
  // Enough resident blocks to cover the SMs several times; the kernels stride beyond.
  const long long blocks = std::max<long long>(1, std::min<long long>((work + threads - 1) / threads, 8LL * sm_count));
  const unsigned nb = static_cast<unsigned>(blocks);
  if (vec) {
    if (gated) launch_vec<T, true>(v, nb, threads, s);
    else launch_vec<T, false>(v, nb, threads, s);
  } else
    gated_act_scalar_kernel<T><<<static_cast<unsigned>(blocks), threads, 0, s>>>(v);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ffn_fail(VF_ECUDA, std::string("gated act launch: ") + cudaGetErrorString(e));
  return VF_OK;
}

}  // namespace
}  // namespace vf

extern "C" {

int vf_gated_act_fwd(const vf_gated_act_args_t* a, void* stream) {
  using vf::ffn_fail;
  if (a == nullptr) return ffn_fail(VF_EINVAL, "null args");
  if (a->act < VF_ACT_GELU_TANH || a->act > VF_ACT_SILU) return ffn_fail(VF_EINVAL, "gated act: unknown activation");
  if (a->rows < 0 || a->cols < 0) return ffn_fail(VF_EINVAL, "gated act: negative sizes");
  if (a->rows == 0 || a->cols == 0) return VF_OK;
  if (!a->gate || !a->out) return ffn_fail(VF_EINVAL, "gated act: gate and out must be non-null");
  if (a->gate_row_stride < a->cols || (a->up != nullptr && a->up_row_stride < a->cols) || a->out_row_stride < a->cols)
    return ffn_fail(VF_EINVAL, "gated act: row strides must be at least cols (rows must not overlap)");
  vf::GatedView v{a->gate, a->up, a->out, a->rows, a->cols, a->gate_row_stride, a->up_row_stride, a->out_row_stride,
                  a->act};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (a->dtype) {
    case VF_DTYPE_BF16: return vf::launch_gated<__nv_bfloat16>(v, s);
    case VF_DTYPE_F16: return vf::launch_gated<__half>(v, s);
    case VF_DTYPE_F32: return vf::launch_gated<float>(v, s);
    default: return ffn_fail(VF_EUNSUPPORTED, "gated act: dtype must be float32, float16 or bfloat16");
  }
}

}  // extern "C"
