// Linear + activation GEMMs with the activation in the epilogue, on sm_100a: the DeBERTa
// feed-forward's out = GELU(x W^T + b) and the mT5 feed-forward's out = GELU_tanh(x W0^T) * up.
//
// The reference runs models/deberta_v2/deberta_v2_encoder.py:547-550 (DebertaV2Intermediate:
// `self.dense` then ACT2FN["gelu"]) as a GEMM that writes its [tokens, 4096] result to HBM and
// an elementwise pass that reads it back and writes it again.  Here the activation runs in the
// GEMM's epilogue, on the fp32 accumulator in registers, so the intermediate never exists.
//
// The GEMMs are CUTLASS 3.x sm100 kernels instantiated in this file (CuTe / CUTLASS templates;
// the headers come from the CUTLASS tree found at build time): tcgen05 UMMA with a TMEM
// accumulator, 256 x 256 x 64 tiles on SM pairs (cluster 2 x 1 x 1; CUTLASS's builder gives a
// cluster whose N extent is 1 the 2-SM TMA load without multicast, and no load in this file
// multicasts), a TMA-store epilogue with the per-column bias and
// cutlass::epilogue::thread::GELU (0.5 x (1 + erf(x / sqrt 2)), the formula of torch's
// exact GELU) in fp32 before the rounding to the output dtype.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>

#include "cute/tensor.hpp"
#include "cutlass/cutlass.h"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/epilogue/fusion/operations.hpp"
#include "cutlass/epilogue/thread/activation.h"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/kernel/gemm_universal.hpp"
#include "cutlass/util/packed_stride.hpp"

#include "vf_internal.h"

namespace vf {
namespace gemm {

using namespace cute;

// Tile and schedule shared by both forms: a 256 x 256 x 64 tile on a pair of SMs
// (tcgen05 cta_group::2, cluster 2 x 1 x 1; each SM of the pair loads its own half of A and
// of B, so the pair's TMA loads are 2-SM loads without multicast), or 128 x 256 x 64 on one SM.
#ifndef VF_GEMM_2SM
#define VF_GEMM_2SM 1
#endif
#if VF_GEMM_2SM
using TileShape = Shape<_256, _256, _64>;
using ClusterShape = Shape<_2, _1, _1>;
using EpilogueSchedule = cutlass::epilogue::TmaWarpSpecialized2Sm;
using MainloopSchedule = cutlass::gemm::KernelTmaWarpSpecialized2SmSm100;
#else
using TileShape = Shape<_128, _256, _64>;
using ClusterShape = Shape<_1, _1, _1>;
using EpilogueSchedule = cutlass::epilogue::TmaWarpSpecialized1Sm;
using MainloopSchedule = cutlass::gemm::KernelTmaWarpSpecialized1SmSm100;
#endif

// D[M, N] = GELU(A[M, K] B[K, N] + bias[N]); A = x (row-major, K contiguous), B = W^T with W
// the [N, K] nn.Linear weight (column-major B), D row-major.
template <typename E>
struct LinearGelu {
  using MmaTile = TileShape;
  using Cluster = ClusterShape;
  using Fusion = cutlass::epilogue::fusion::LinCombPerColBiasEltAct<cutlass::epilogue::thread::GELU, E, float, E, E,
                                                                    float>;
  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTile, Cluster,
      cutlass::epilogue::collective::EpilogueTileAuto, float, float, void, cutlass::layout::RowMajor, 8, E,
      cutlass::layout::RowMajor, 8, EpilogueSchedule, Fusion>::CollectiveOp;
  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, E, cutlass::layout::RowMajor, 8, E,
      cutlass::layout::ColumnMajor, 8, float, MmaTile, Cluster,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
      MainloopSchedule>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, void>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
};

// D[M, N] = GELU_tanh(A[M, K] B[K, N]) * C[M, N]: the gated activation of the mT5 feed-forward
// (models/mt5/mt5_encoder.py:427-437 with kernels/ff_fused.py:86, "gelu_new"), C = the up
// projection x Wi_1^T computed first, this GEMM the gate projection x Wi_0^T.  An epilogue visitor
// tree: GELU_taylor (0.5 z (1 + tanh(0.79788456 (z + 0.044715 z^3))), the tanh form of the
// reference kernel, with the tanh.approx instruction) of the accumulator, times the source C.
template <typename E>
struct LinearGeluTanhMul {
  using MmaTile = TileShape;
  using Cluster = ClusterShape;
  static constexpr auto RS = cutlass::FloatRoundStyle::round_to_nearest;
  using Act = cutlass::epilogue::fusion::Sm90EVT<
      cutlass::epilogue::fusion::Sm90Compute<cutlass::epilogue::thread::GELU_taylor, float, float, RS>,
      cutlass::epilogue::fusion::Sm90AccFetch>;
  using Fusion = cutlass::epilogue::fusion::Sm90EVT<
      cutlass::epilogue::fusion::Sm90Compute<cutlass::multiplies, E, float, RS>, Act,
      cutlass::epilogue::fusion::Sm90SrcFetch<E>>;
  using Epilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, MmaTile, Cluster,
      cutlass::epilogue::collective::EpilogueTileAuto, float, float, E, cutlass::layout::RowMajor, 8, E,
      cutlass::layout::RowMajor, 8, EpilogueSchedule, Fusion>::CollectiveOp;
  using Mainloop = typename cutlass::gemm::collective::CollectiveBuilder<
      cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, E, cutlass::layout::RowMajor, 8, E,
      cutlass::layout::ColumnMajor, 8, float, MmaTile, Cluster,
      cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename Epilogue::SharedStorage))>,
      MainloopSchedule>::CollectiveOp;
  using Kernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, Mainloop, Epilogue, void>;
  using Gemm = cutlass::gemm::device::GemmUniversalAdapter<Kernel>;
};

int device_sm_count() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::once_flag flags[64];
  static int sm_count[64];
  if (dev < 0 || dev >= 64) return 148;
  std::call_once(flags[dev], [&] {
    if (cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sm_count[dev] = 0;
  });
  return sm_count[dev] > 0 ? sm_count[dev] : 148;
}

template <class Gemm>
int launch(typename Gemm::Arguments& args, cudaStream_t stream) {
  Gemm gemm;
  if (gemm.can_implement(args) != cutlass::Status::kSuccess)
    return set_last_error(VF_EUNSUPPORTED, "linear act: the GEMM cannot run these sizes / alignments");
  if (Gemm::get_workspace_size(args) != 0)
    return set_last_error(VF_EUNSUPPORTED, "linear act: the GEMM asked for a workspace");
  cutlass::Status st = gemm.initialize(args, nullptr, stream);
  if (st == cutlass::Status::kSuccess) st = gemm.run(stream);
  if (st != cutlass::Status::kSuccess) {
    const cudaError_t e = cudaGetLastError();
    return set_last_error(VF_ECUDA, std::string("linear act: GEMM launch failed: ") + cudaGetErrorString(e));
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(VF_ECUDA, std::string("linear act: ") + cudaGetErrorString(e));
  return VF_OK;
}

template <typename E>
int run_gated(const vf_linear_act_args_t* a, cudaStream_t stream) {
  using G = LinearGeluTanhMul<E>;
  using Kernel = typename G::Kernel;
  const int M = static_cast<int>(a->rows), N = static_cast<int>(a->N), K = static_cast<int>(a->K);
  auto sA = cutlass::make_cute_packed_stride(typename Kernel::StrideA{}, make_shape(M, K, 1));
  auto sB = cutlass::make_cute_packed_stride(typename Kernel::StrideB{}, make_shape(N, K, 1));
  auto sC = cutlass::make_cute_packed_stride(typename Kernel::StrideC{}, make_shape(M, N, 1));
  auto sD = cutlass::make_cute_packed_stride(typename Kernel::StrideD{}, make_shape(M, N, 1));
  get<0>(sA) = a->x_row_stride;
  get<0>(sB) = a->weight_row_stride;
  get<0>(sC) = a->mul_row_stride;
  get<0>(sD) = a->out_row_stride;
  cutlass::KernelHardwareInfo hw;
  cudaGetDevice(&hw.device_id);
  hw.sm_count = device_sm_count();
  typename G::Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                   {M, N, K, 1},
                                   {static_cast<const E*>(a->x), sA, static_cast<const E*>(a->weight), sB},
                                   {{}, static_cast<const E*>(a->mul), sC, static_cast<E*>(a->out), sD},
                                   hw};
  return launch<typename G::Gemm>(args, stream);
}

template <typename E>
int run(const vf_linear_act_args_t* a, cudaStream_t stream) {
  using G = LinearGelu<E>;
  using Kernel = typename G::Kernel;
  const int M = static_cast<int>(a->rows), N = static_cast<int>(a->N), K = static_cast<int>(a->K);
  auto sA = cutlass::make_cute_packed_stride(typename Kernel::StrideA{}, make_shape(M, K, 1));
  auto sB = cutlass::make_cute_packed_stride(typename Kernel::StrideB{}, make_shape(N, K, 1));
  auto sD = cutlass::make_cute_packed_stride(typename Kernel::StrideD{}, make_shape(M, N, 1));
  get<0>(sA) = a->x_row_stride;
  get<0>(sB) = a->weight_row_stride;
  get<0>(sD) = a->out_row_stride;
  cutlass::KernelHardwareInfo hw;
  cudaGetDevice(&hw.device_id);
  hw.sm_count = device_sm_count();
  typename G::Gemm::Arguments args{cutlass::gemm::GemmUniversalMode::kGemm,
                                   {M, N, K, 1},
                                   {static_cast<const E*>(a->x), sA, static_cast<const E*>(a->weight), sB},
                                   {{}, nullptr, sD, static_cast<E*>(a->out), sD},
                                   hw};
  args.epilogue.thread.alpha = 1.0f;
  args.epilogue.thread.beta = 0.0f;
  args.epilogue.thread.bias_ptr = static_cast<const E*>(a->bias);
  return launch<typename G::Gemm>(args, stream);
}

}  // namespace gemm
}  // namespace vf

extern "C" {

int vf_linear_act_fwd(const vf_linear_act_args_t* a, void* stream) {
  using vf::set_last_error;
  if (a == nullptr) return set_last_error(VF_EINVAL, "null args");
  if (a->dtype != VF_DTYPE_BF16 && a->dtype != VF_DTYPE_F16)
    return set_last_error(VF_EUNSUPPORTED, "linear act: dtype must be float16 or bfloat16");
  const bool gated = a->act == VF_ACT_GELU_TANH;
  if (a->act != VF_ACT_GELU_ERF && !gated)
    return set_last_error(VF_EUNSUPPORTED, "linear act: the built forms are VF_ACT_GELU_ERF (+ bias) and VF_ACT_GELU_TANH (x mul)");
  if (a->rows < 0 || a->K <= 0 || a->N <= 0) return set_last_error(VF_EINVAL, "linear act: rows >= 0, K > 0, N > 0");
  if (a->rows >= (1LL << 31) || a->K >= (1LL << 31) || a->N >= (1LL << 31))
    return set_last_error(VF_EUNSUPPORTED, "linear act: sizes must be below 2^31");
  if (a->rows == 0) return VF_OK;
  if (!a->x || !a->weight || !a->out) return set_last_error(VF_EINVAL, "linear act: x, weight and out must be non-null");
  if (gated ? (a->mul == nullptr || a->bias != nullptr) : (a->bias == nullptr || a->mul != nullptr))
    return set_last_error(VF_EINVAL, "linear act: VF_ACT_GELU_ERF takes a bias and no mul, VF_ACT_GELU_TANH a mul and no bias");
  if (a->x_row_stride < a->K || a->weight_row_stride < a->K || a->out_row_stride < a->N ||
      (gated && a->mul_row_stride < a->N))
    return set_last_error(VF_EINVAL, "linear act: row strides must be at least K (x, weight) and N (out, mul)");
  const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const void* extra = gated ? a->mul : a->bias;
  if (a->K % 8 != 0 || a->N % 8 != 0 || a->x_row_stride % 8 != 0 || a->weight_row_stride % 8 != 0 ||
      a->out_row_stride % 8 != 0 || (gated && a->mul_row_stride % 8 != 0) || !al16(a->x) || !al16(a->weight) ||
      !al16(extra) || !al16(a->out))
    return set_last_error(VF_EINVAL, "linear act: K, N, row strides must be multiples of 8 and pointers 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gated)
    return a->dtype == VF_DTYPE_BF16 ? vf::gemm::run_gated<cutlass::bfloat16_t>(a, s)
                                     : vf::gemm::run_gated<cutlass::half_t>(a, s);
  return a->dtype == VF_DTYPE_BF16 ? vf::gemm::run<cutlass::bfloat16_t>(a, s) : vf::gemm::run<cutlass::half_t>(a, s);
}

}  // extern "C"
