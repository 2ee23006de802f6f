// Host helpers shared by the kernel files of libvf_b200.so (hidden symbols; not part of the
// C ABI).  Defined in vf_attention.cu.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <string>

#include "../../include/vf_b200.h"

namespace vf {

// Sets the calling thread's vf_last_error() message and returns `code`.
int set_last_error(int code, const std::string& msg);

// (B, H, L, 64) strided 16-bit view -> 4-D tensor map with a 64 x 128 box, 128-byte swizzle.
int host_make_tile_map(CUtensorMap* map, const vf_tensor4d_t& t, vf_dtype_t dt, const char* name);

// Shape, null and alignment checks of q, k, v, out (head_dim 64, out rows 16-byte aligned).
int host_check_qkv(const vf_tensor4d_t& q, const vf_tensor4d_t& k, const vf_tensor4d_t& v, const vf_tensor4d_t& o);

// Checks of the packed-batch views and offsets array (the *_varlen_fwd rules).
int host_check_packed(const vf_tensor4d_t& q, const vf_tensor4d_t& k, const int32_t* cu_seqlens, int32_t num_seqs,
                      int32_t max_seqlen, const char* what);

// DeBERTa position index idx(r) = clamp(bucket(r) + span, 0, 2 span - 1) for |r| < L: the
// cached table (saturation radius R, lut[r + R] for r in [-R, R]; |r| > R reads lut[0] /
// lut[2R]).  Returns the radius, or -1 when it exceeds `max_radius`.
int host_deberta_index_table(int span, int position_buckets, int max_relative_distance, bool log_bucket, int L,
                             int max_radius, short* lut_out);

// cuTensorMapEncodeTiled from the driver (nullptr when unavailable).
PFN_cuTensorMapEncodeTiled_v12000 host_encode_fn();

// Error word of the fused DeBERTa kernel file (vf_deberta_fused.cu), read and optionally
// cleared in one atomic operation.
cudaError_t fused_take_error_word(bool clear, unsigned int* word);

// The same for the span-score kernel file (vf_span.cu).
cudaError_t span_take_error_word(bool clear, unsigned int* word);

// The same for the feed-forward GEMM file (vf_gemm.cu).
cudaError_t gemm_take_error_word(bool clear, unsigned int* word);

}  // namespace vf
