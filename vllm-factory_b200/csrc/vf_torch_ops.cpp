// torch.ops.vf_b200.* — thin C++ op layer over the C ABI of libvf_b200.so.
//
// Tensors are read here (sizes, strides, data pointers, the current CUDA stream) and
// passed as plain pointers/sizes to vf_rpb_attention_fwd / vf_deberta_attention_fwd; the
// kernels, bucket tables and validation live behind the C ABI.  Only the output tensor is
// allocated (plus fp16 copies for fp32 inputs, below).  CPU tensors raise: there is no CPU
// implementation.
//
// fp32 q / k / v (and DeBERTa position tensors) are computed in fp16: the tensor cores take
// 16-bit operands, and fp16 keeps the 10-bit mantissa of TF32, the precision the reference's
// fp32 Triton path multiplies at.  Inputs are clamped to the fp16 range (+-65504) on the way
// in; scores, softmax and accumulation stay fp32 inside the kernel; the output is returned
// in fp32.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <optional>
#include <string>
#include <vector>

#include <cstdlib>

#include "vf_b200.h"

namespace {

vf_dtype_t dtype_code(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return VF_DTYPE_F32;
    case at::kHalf: return VF_DTYPE_F16;
    case at::kBFloat16: return VF_DTYPE_BF16;
    default: TORCH_CHECK(false, "vf_b200: unsupported dtype ", t.scalar_type());
  }
}

vf_tensor4d_t view4(const at::Tensor& t) {
  TORCH_CHECK(t.dim() == 4, "vf_b200: expected a 4-D tensor, got ", t.sizes());
  vf_tensor4d_t d{};
  d.data = t.data_ptr();
  for (int i = 0; i < 4; ++i) {
    d.size[i] = t.size(i);
    d.stride[i] = t.stride(i);
  }
  return d;
}

// A layout TMA can describe: unit innermost stride, 16-byte aligned base and strides.
at::Tensor tma_ready(const at::Tensor& t) {
  const int64_t es = t.element_size();
  bool ok = t.stride(3) == 1 && (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0;
  for (int i = 0; i < 3 && ok; ++i) ok = t.stride(i) > 0 && (t.stride(i) * es) % 16 == 0;
  return ok ? t : t.contiguous();
}

at::Tensor make_out(const at::Tensor& q) {
  at::Tensor out = at::empty_like(q);
  if (out.stride(3) != 1 || (out.stride(2) * out.element_size()) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(out.data_ptr()) % 16) != 0)
    out = at::empty(q.sizes(), q.options());
  return out;
}

void require_cuda(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), "vf_b200: ", name, " must be a CUDA tensor (no CPU implementation)");
}

// VF_B200_CHECK_DEVICE_ERRORS=1 (read once): after every launch, synchronise and raise if a
// kernel set the device error word (a bounded wait that ran out, a failed index check, packed
// offsets that broke the rules).  A debugging aid: it serialises the caller with the device.
bool device_error_checks() {
  static const bool on = [] {
    const char* v = std::getenv("VF_B200_CHECK_DEVICE_ERRORS");
    return v != nullptr && v[0] != '\0' && v[0] != '0';
  }();
  return on;
}

void check_rc(int rc) {
  TORCH_CHECK(rc == VF_OK, "vf_b200 error ", rc, ": ", vf_last_error());
  if (device_error_checks()) {
    const int word = vf_device_error(1);
    TORCH_CHECK(word >= 0, "vf_b200 error ", word, ": ", vf_last_error());
    TORCH_CHECK(word == 0, "vf_b200: a kernel reported device error word 0x", std::hex, word,
                " (bit 0: a bounded wait ran out; bit 1: an index failed its check; bit 2: packed offsets broke the rules)");
  }
}

// fp32 operands become fp16 (clamped to its finite range); 16-bit ones pass through.
at::Tensor to_kernel_dtype(const at::Tensor& t) {
  if (t.scalar_type() != at::kFloat) return t;
  return at::clamp(t, -65504.0, 65504.0).to(at::kHalf);
}

// Position tensors are gathered along their last dimension with 32-bit offsets: give them
// a unit last-dimension stride (row strides stay as they are).
at::Tensor unit_last(const at::Tensor& t) { return t.stride(-1) == 1 ? t : t.contiguous(); }

at::Tensor rpb_attention(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                         const std::optional<at::Tensor>& rpb_table, int64_t num_buckets,
                         int64_t max_distance, bool is_decoder,
                         const std::optional<at::Tensor>& padding_mask, double dropout_p,
                         double softmax_scale) {
  require_cuda(q_in, "q");
  require_cuda(k_in, "k");
  require_cuda(v_in, "v");
  TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
              "vf_b200: q, k, v must share a dtype");
  c10::cuda::CUDAGuard guard(q_in.device());
  const bool f32 = q_in.scalar_type() == at::kFloat;
  const at::Tensor q = tma_ready(to_kernel_dtype(q_in)), k = tma_ready(to_kernel_dtype(k_in)),
                   v = tma_ready(to_kernel_dtype(v_in));
  at::Tensor out = make_out(q);
  vf_rpb_attention_args_t a{};
  a.dtype = dtype_code(q);
  a.q = view4(q);
  a.k = view4(k);
  a.v = view4(v);
  a.out = view4(out);
  if (rpb_table.has_value()) {
    const at::Tensor& t = *rpb_table;
    require_cuda(t, "rpb_table");
    TORCH_CHECK(t.dim() == 2, "vf_b200: rpb_table must be [num_buckets, heads]");
    a.rpb_table = t.data_ptr();
    a.table_rows = t.size(0);
    a.table_cols = t.size(1);
    a.table_stride_row = t.stride(0);
    a.table_stride_col = t.stride(1);
    a.table_dtype = dtype_code(t);
  }
  a.num_buckets = static_cast<int32_t>(num_buckets);
  a.max_distance = static_cast<int32_t>(max_distance);
  a.is_decoder = is_decoder ? 1 : 0;
  if (padding_mask.has_value()) {
    require_cuda(*padding_mask, "padding_mask");
    a.padding_mask = view4(*padding_mask);
    a.mask_dtype = dtype_code(*padding_mask);
  }
  a.dropout_p = static_cast<float>(dropout_p);
  a.softmax_scale = static_cast<float>(softmax_scale);
  check_rc(vf_rpb_attention_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
  return f32 ? out.to(at::kFloat) : out;
}

// Packed batches: [total, H, D] tensors seen by the kernels as (1, H, total, D) views.
vf_tensor4d_t packed_view(const at::Tensor& t) {
  vf_tensor4d_t d{};
  d.data = t.data_ptr();
  d.size[0] = 1;
  d.size[1] = t.size(1);
  d.size[2] = t.size(0);
  d.size[3] = t.size(2);
  d.stride[0] = std::max<int64_t>(t.size(0) * t.stride(0), 8);
  d.stride[1] = t.stride(1);
  d.stride[2] = t.stride(0);
  d.stride[3] = t.stride(2);
  return d;
}

// Kernel dtype, unit innermost stride, 16-byte aligned base and row / head strides (TMA).
at::Tensor packed_tma_ready(const at::Tensor& t) {
  at::Tensor x = to_kernel_dtype(t);
  const int64_t es = x.element_size();
  if (x.stride(2) != 1 || (x.stride(0) * es) % 16 != 0 || (x.stride(1) * es) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) != 0)
    x = x.contiguous();
  return x;
}

at::Tensor cu_int32(const at::Tensor& cu_seqlens) {
  require_cuda(cu_seqlens, "cu_seqlens");
  TORCH_CHECK(cu_seqlens.dim() == 1 && cu_seqlens.numel() >= 2, "vf_b200: cu_seqlens must be [num_seqs + 1]");
  at::Tensor cu = cu_seqlens;
  if (cu.scalar_type() != at::kInt || !cu.is_contiguous()) cu = cu.to(at::kInt).contiguous();
  return cu;
}

// Packed batch: q, k, v are [total, H, 64] (the rows of every sequence back to back),
// cu_seqlens int32 [num_seqs + 1]; the kernel sees them as (1, H, total, 64) views.
at::Tensor rpb_attention_varlen(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                                const at::Tensor& cu_seqlens, int64_t max_seqlen,
                                const std::optional<at::Tensor>& rpb_table, int64_t num_buckets,
                                int64_t max_distance, bool is_decoder, double softmax_scale) {
  require_cuda(q_in, "q");
  require_cuda(k_in, "k");
  require_cuda(v_in, "v");
  TORCH_CHECK(q_in.dim() == 3 && k_in.dim() == 3 && v_in.dim() == 3, "vf_b200: packed q, k, v must be [total, heads, 64]");
  TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
              "vf_b200: q, k, v must share a dtype");
  c10::cuda::CUDAGuard guard(q_in.device());
  const bool f32 = q_in.scalar_type() == at::kFloat;
  const at::Tensor q = packed_tma_ready(q_in), k = packed_tma_ready(k_in), v = packed_tma_ready(v_in);
  at::Tensor out = at::empty(q.sizes(), q.options());
  const at::Tensor cu = cu_int32(cu_seqlens);
  vf_rpb_attention_args_t a{};
  a.dtype = dtype_code(q);
  a.q = packed_view(q);
  a.k = packed_view(k);
  a.v = packed_view(v);
  a.out = packed_view(out);
  if (rpb_table.has_value()) {
    const at::Tensor& t = *rpb_table;
    require_cuda(t, "rpb_table");
    TORCH_CHECK(t.dim() == 2, "vf_b200: rpb_table must be [num_buckets, heads]");
    a.rpb_table = t.data_ptr();
    a.table_rows = t.size(0);
    a.table_cols = t.size(1);
    a.table_stride_row = t.stride(0);
    a.table_stride_col = t.stride(1);
    a.table_dtype = dtype_code(t);
  }
  a.num_buckets = static_cast<int32_t>(num_buckets);
  a.max_distance = static_cast<int32_t>(max_distance);
  a.is_decoder = is_decoder ? 1 : 0;
  a.softmax_scale = static_cast<float>(softmax_scale);
  TORCH_CHECK(max_seqlen > 0 && max_seqlen <= INT32_MAX, "vf_b200: max_seqlen out of range");
  check_rc(vf_rpb_attention_varlen_fwd(&a, cu.data_ptr<int32_t>(), static_cast<int32_t>(cu.numel() - 1),
                                       static_cast<int32_t>(max_seqlen), at::cuda::getCurrentCUDAStream().stream()));
  return f32 ? out.to(at::kFloat) : out;
}

at::Tensor deberta_attention(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                             const std::optional<at::Tensor>& seq_lengths,
                             const std::optional<at::Tensor>& pos_key,
                             const std::optional<at::Tensor>& pos_query, bool causal,
                             std::optional<double> sm_scale, int64_t position_buckets,
                             int64_t max_relative_distance, bool use_log_bucket) {
  require_cuda(q_in, "q");
  require_cuda(k_in, "k");
  require_cuda(v_in, "v");
  TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
              "vf_b200: q, k, v must share a dtype");
  c10::cuda::CUDAGuard guard(q_in.device());
  const bool f32 = q_in.scalar_type() == at::kFloat;
  const at::Tensor q = tma_ready(to_kernel_dtype(q_in)), k = tma_ready(to_kernel_dtype(k_in)),
                   v = tma_ready(to_kernel_dtype(v_in));
  at::Tensor out = make_out(q);
  vf_deberta_attention_args_t a{};
  a.dtype = dtype_code(q);
  a.q = view4(q);
  a.k = view4(k);
  a.v = view4(v);
  a.out = view4(out);
  at::Tensor lens;
  if (seq_lengths.has_value()) {
    require_cuda(*seq_lengths, "seq_lengths");
    lens = *seq_lengths;
    if (lens.scalar_type() != at::kInt || !lens.is_contiguous()) lens = lens.to(at::kInt).contiguous();
    TORCH_CHECK(lens.numel() == q.size(0), "vf_b200: seq_lengths must have one entry per batch row");
    a.seq_lengths = lens.data_ptr<int32_t>();
  }
  at::Tensor pk, pq;   // keep fp16 copies alive until the launch is enqueued
  if (pos_key.has_value()) {
    require_cuda(*pos_key, "pos_key");
    TORCH_CHECK(pos_key->scalar_type() == q_in.scalar_type(), "vf_b200: pos_key must have the dtype of q");
    pk = unit_last(to_kernel_dtype(*pos_key));
    a.pos_key = view4(pk);
  }
  if (pos_query.has_value()) {
    require_cuda(*pos_query, "pos_query");
    TORCH_CHECK(pos_query->scalar_type() == q_in.scalar_type(), "vf_b200: pos_query must have the dtype of q");
    pq = unit_last(to_kernel_dtype(*pos_query));
    a.pos_query = view4(pq);
  }
  a.causal = causal ? 1 : 0;
  a.has_sm_scale = sm_scale.has_value() ? 1 : 0;
  a.sm_scale = sm_scale.has_value() ? static_cast<float>(*sm_scale) : 0.f;
  a.position_buckets = static_cast<int32_t>(position_buckets);
  a.max_relative_distance = static_cast<int32_t>(max_relative_distance);
  a.use_log_bucket = use_log_bucket ? 1 : 0;
  check_rc(vf_deberta_attention_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
  return f32 ? out.to(at::kFloat) : out;
}

// Packed DeBERTa batch: q, k, v [total, H, 64]; pos_key / pos_query [total, H, 2S].
at::Tensor deberta_attention_varlen(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                                    const at::Tensor& cu_seqlens, int64_t max_seqlen,
                                    const std::optional<at::Tensor>& pos_key,
                                    const std::optional<at::Tensor>& pos_query, bool causal,
                                    std::optional<double> sm_scale, int64_t position_buckets,
                                    int64_t max_relative_distance, bool use_log_bucket) {
  require_cuda(q_in, "q");
  require_cuda(k_in, "k");
  require_cuda(v_in, "v");
  TORCH_CHECK(q_in.dim() == 3 && k_in.dim() == 3 && v_in.dim() == 3, "vf_b200: packed q, k, v must be [total, heads, 64]");
  TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
              "vf_b200: q, k, v must share a dtype");
  c10::cuda::CUDAGuard guard(q_in.device());
  const bool f32 = q_in.scalar_type() == at::kFloat;
  const at::Tensor q = packed_tma_ready(q_in), k = packed_tma_ready(k_in), v = packed_tma_ready(v_in);
  at::Tensor out = at::empty(q.sizes(), q.options());
  const at::Tensor cu = cu_int32(cu_seqlens);
  vf_deberta_attention_args_t a{};
  a.dtype = dtype_code(q);
  a.q = packed_view(q);
  a.k = packed_view(k);
  a.v = packed_view(v);
  a.out = packed_view(out);
  at::Tensor pk, pq;   // kernel-dtype copies stay alive until the launch is enqueued
  if (pos_key.has_value()) {
    require_cuda(*pos_key, "pos_key");
    TORCH_CHECK(pos_key->dim() == 3, "vf_b200: packed pos_key must be [total, heads, 2*span]");
    TORCH_CHECK(pos_key->scalar_type() == q_in.scalar_type(), "vf_b200: pos_key must have the dtype of q");
    pk = unit_last(to_kernel_dtype(*pos_key));
    a.pos_key = packed_view(pk);
  }
  if (pos_query.has_value()) {
    require_cuda(*pos_query, "pos_query");
    TORCH_CHECK(pos_query->dim() == 3, "vf_b200: packed pos_query must be [total, heads, 2*span]");
    TORCH_CHECK(pos_query->scalar_type() == q_in.scalar_type(), "vf_b200: pos_query must have the dtype of q");
    pq = unit_last(to_kernel_dtype(*pos_query));
    a.pos_query = packed_view(pq);
  }
  a.causal = causal ? 1 : 0;
  a.has_sm_scale = sm_scale.has_value() ? 1 : 0;
  a.sm_scale = sm_scale.has_value() ? static_cast<float>(*sm_scale) : 0.f;
  a.position_buckets = static_cast<int32_t>(position_buckets);
  a.max_relative_distance = static_cast<int32_t>(max_relative_distance);
  a.use_log_bucket = use_log_bucket ? 1 : 0;
  TORCH_CHECK(max_seqlen > 0 && max_seqlen <= INT32_MAX, "vf_b200: max_seqlen out of range");
  check_rc(vf_deberta_attention_varlen_fwd(&a, cu.data_ptr<int32_t>(), static_cast<int32_t>(cu.numel() - 1),
                                           static_cast<int32_t>(max_seqlen), at::cuda::getCurrentCUDAStream().stream()));
  return f32 ? out.to(at::kFloat) : out;
}

// Fused DeBERTa mode: rel_key / rel_query (1, H, 2S, 64) in place of pos_key / pos_query; the
// position products run inside the kernel.  The workspace (expanded position tables and
// the unit order) comes from the caching allocator on the call's stream.
at::Tensor rel_ready(const std::optional<at::Tensor>& t, const at::Tensor& q_in, const char* name) {
  if (!t.has_value() || !t->defined()) return at::Tensor();
  require_cuda(*t, name);
  TORCH_CHECK(t->scalar_type() == q_in.scalar_type(), "vf_b200: ", name, " must have the dtype of q");
  at::Tensor x = *t;
  if (x.dim() == 3) x = x.unsqueeze(0);
  TORCH_CHECK(x.dim() == 4, "vf_b200: ", name, " must be (1, H, 2*span, 64) or (H, 2*span, 64)");
  x = to_kernel_dtype(x);
  const int64_t es = x.element_size();
  if (x.stride(3) != 1 || (x.stride(2) * es) % 16 != 0 || (x.stride(1) * es) % 16 != 0 ||
      (reinterpret_cast<uintptr_t>(x.data_ptr()) % 16) != 0)
    x = x.contiguous();
  return x;
}

vf_tensor4d_t view4_or_absent(const at::Tensor& t) { return t.defined() ? view4(t) : vf_tensor4d_t{}; }

at::Tensor deberta_attention_fused(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                                   const std::optional<at::Tensor>& seq_lengths,
                                   const std::optional<at::Tensor>& rel_key,
                                   const std::optional<at::Tensor>& rel_query, bool causal,
                                   std::optional<double> sm_scale, int64_t position_buckets,
                                   int64_t max_relative_distance, bool use_log_bucket) {
  require_cuda(q_in, "q");
  require_cuda(k_in, "k");
  require_cuda(v_in, "v");
  TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
              "vf_b200: q, k, v must share a dtype");
  c10::cuda::CUDAGuard guard(q_in.device());
  const bool f32 = q_in.scalar_type() == at::kFloat;
  const at::Tensor q = tma_ready(to_kernel_dtype(q_in)), k = tma_ready(to_kernel_dtype(k_in)),
                   v = tma_ready(to_kernel_dtype(v_in));
  at::Tensor out = make_out(q);
  const at::Tensor rk = rel_ready(rel_key, q_in, "rel_key"), rq = rel_ready(rel_query, q_in, "rel_query");
  vf_deberta_fused_args_t a{};
  a.dtype = dtype_code(q);
  a.q = view4(q);
  a.k = view4(k);
  a.v = view4(v);
  a.out = view4(out);
  at::Tensor lens;
  if (seq_lengths.has_value()) {
    require_cuda(*seq_lengths, "seq_lengths");
    lens = *seq_lengths;
    if (lens.scalar_type() != at::kInt || !lens.is_contiguous()) lens = lens.to(at::kInt).contiguous();
    TORCH_CHECK(lens.numel() == q.size(0), "vf_b200: seq_lengths must have one entry per batch row");
    a.seq_lengths = lens.data_ptr<int32_t>();
  }
  a.rel_key = view4_or_absent(rk);
  a.rel_query = view4_or_absent(rq);
  a.causal = causal ? 1 : 0;
  a.has_sm_scale = sm_scale.has_value() ? 1 : 0;
  a.sm_scale = sm_scale.has_value() ? static_cast<float>(*sm_scale) : 0.f;
  a.position_buckets = static_cast<int32_t>(position_buckets);
  a.max_relative_distance = static_cast<int32_t>(max_relative_distance);
  a.use_log_bucket = use_log_bucket ? 1 : 0;
  const int64_t ws_bytes = vf_deberta_fused_workspace_bytes(q.size(0), q.size(1), q.size(2), k.size(2));
  check_rc(ws_bytes < 0 ? static_cast<int>(ws_bytes) : VF_OK);
  at::Tensor ws = at::empty({ws_bytes + 256}, q.options().dtype(at::kByte));
  void* ws_ptr = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~uintptr_t(255));
  check_rc(vf_deberta_attention_fused_fwd(&a, ws_ptr, ws_bytes, at::cuda::getCurrentCUDAStream().stream()));
  return f32 ? out.to(at::kFloat) : out;
}

// Packed fused DeBERTa batch: q, k, v [total, H, 64]; rel_key / rel_query (1, H, 2S, 64).
at::Tensor deberta_attention_fused_varlen(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in,
                                          const at::Tensor& cu_seqlens, int64_t max_seqlen,
                                          const std::optional<at::Tensor>& rel_key,
                                          const std::optional<at::Tensor>& rel_query, bool causal,
                                          std::optional<double> sm_scale, int64_t position_buckets,
                                          int64_t max_relative_distance, bool use_log_bucket) {
  require_cuda(q_in, "q");
  require_cuda(k_in, "k");
  require_cuda(v_in, "v");
  TORCH_CHECK(q_in.dim() == 3 && k_in.dim() == 3 && v_in.dim() == 3, "vf_b200: packed q, k, v must be [total, heads, 64]");
  TORCH_CHECK(q_in.scalar_type() == k_in.scalar_type() && q_in.scalar_type() == v_in.scalar_type(),
              "vf_b200: q, k, v must share a dtype");
  c10::cuda::CUDAGuard guard(q_in.device());
  const bool f32 = q_in.scalar_type() == at::kFloat;
  const at::Tensor q = packed_tma_ready(q_in), k = packed_tma_ready(k_in), v = packed_tma_ready(v_in);
  at::Tensor out = at::empty(q.sizes(), q.options());
  const at::Tensor cu = cu_int32(cu_seqlens);
  const at::Tensor rk = rel_ready(rel_key, q_in, "rel_key"), rq = rel_ready(rel_query, q_in, "rel_query");
  vf_deberta_fused_args_t a{};
  a.dtype = dtype_code(q);
  a.q = packed_view(q);
  a.k = packed_view(k);
  a.v = packed_view(v);
  a.out = packed_view(out);
  a.rel_key = view4_or_absent(rk);
  a.rel_query = view4_or_absent(rq);
  a.causal = causal ? 1 : 0;
  a.has_sm_scale = sm_scale.has_value() ? 1 : 0;
  a.sm_scale = sm_scale.has_value() ? static_cast<float>(*sm_scale) : 0.f;
  a.position_buckets = static_cast<int32_t>(position_buckets);
  a.max_relative_distance = static_cast<int32_t>(max_relative_distance);
  a.use_log_bucket = use_log_bucket ? 1 : 0;
  TORCH_CHECK(max_seqlen > 0 && max_seqlen <= INT32_MAX, "vf_b200: max_seqlen out of range");
  const int64_t nseq = cu.numel() - 1;
  const int64_t ws_bytes = vf_deberta_fused_workspace_bytes(nseq, q.size(1), max_seqlen, max_seqlen);
  check_rc(ws_bytes < 0 ? static_cast<int>(ws_bytes) : VF_OK);
  at::Tensor ws = at::empty({ws_bytes + 256}, q.options().dtype(at::kByte));
  void* ws_ptr = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(ws.data_ptr()) + 255) & ~uintptr_t(255));
  check_rc(vf_deberta_attention_fused_varlen_fwd(&a, cu.data_ptr<int32_t>(), static_cast<int32_t>(nseq),
                                                 static_cast<int32_t>(max_seqlen), ws_ptr, ws_bytes,
                                                 at::cuda::getCurrentCUDAStream().stream()));
  return f32 ? out.to(at::kFloat) : out;
}

at::Tensor deberta_attention_fused_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                       const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                                       const std::optional<at::Tensor>&, bool, std::optional<double>, int64_t,
                                       int64_t, bool) {
  TORCH_CHECK(false, "vf_b200: q, k, v must be CUDA tensors (no CPU implementation)");
}
at::Tensor deberta_attention_fused_varlen_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                              const at::Tensor&, int64_t, const std::optional<at::Tensor>&,
                                              const std::optional<at::Tensor>&, bool, std::optional<double>,
                                              int64_t, int64_t, bool) {
  TORCH_CHECK(false, "vf_b200: q, k, v must be CUDA tensors (no CPU implementation)");
}

// Gated activation: out = act(gate) * up over the last dimension; leading dimensions are
// rows.  Each operand only needs a unit stride on the last dimension and leading
// dimensions that collapse to one row stride (as the two column halves of a 2-D [T, 2F]
// projection do); anything else is copied contiguous first.
// A 2-D (rows, cols) view of t with unit column stride, without a copy when possible.
at::Tensor as_rows(const at::Tensor& t, int64_t rows, int64_t cols) {
  at::Tensor x = t;
  if (x.dim() == 1) x = x.unsqueeze(0);
  if (x.stride(-1) != 1) x = x.contiguous();
  if (x.dim() > 2) {
    bool collapses = true;   // leading dims form one row stride
    for (int64_t d = x.dim() - 2; d > 0; --d)
      if (x.size(d - 1) > 1 && x.stride(d - 1) != x.stride(d) * x.size(d)) collapses = false;
    if (!collapses) x = x.contiguous();
    x = x.reshape({rows, cols});
  }
  if (x.size(0) > 1 && x.stride(0) < cols) x = x.contiguous();   // overlapping or broadcast rows
  return x;
}

at::Tensor gated_act(const at::Tensor& gate_in, const std::optional<at::Tensor>& up_opt, int64_t act) {
  require_cuda(gate_in, "gate");
  const bool gated = up_opt.has_value() && up_opt->defined();
  if (gated) {
    require_cuda(*up_opt, "up");
    TORCH_CHECK(gate_in.sizes() == up_opt->sizes(), "vf_b200: gate and up must have identical shapes");
    TORCH_CHECK(gate_in.scalar_type() == up_opt->scalar_type(), "vf_b200: gate and up must share a dtype");
  }
  TORCH_CHECK(gate_in.dim() >= 1, "vf_b200: gate must have at least one dimension");
  c10::cuda::CUDAGuard guard(gate_in.device());
  const int64_t cols = gate_in.size(-1);
  const int64_t rows = cols == 0 ? 0 : gate_in.numel() / cols;
  at::Tensor out = at::empty(gate_in.sizes(), gate_in.options());
  if (rows == 0 || cols == 0) return out;
  const at::Tensor g = as_rows(gate_in, rows, cols);
  const at::Tensor u = gated ? as_rows(*up_opt, rows, cols) : at::Tensor();
  vf_gated_act_args_t a{};
  a.dtype = dtype_code(g);
  a.gate = g.data_ptr();
  a.up = gated ? u.data_ptr() : nullptr;
  a.out = out.data_ptr();
  a.rows = rows;
  a.cols = cols;
  a.gate_row_stride = rows > 1 ? g.stride(0) : cols;
  a.up_row_stride = gated ? (rows > 1 ? u.stride(0) : cols) : cols;
  a.out_row_stride = cols;
  a.act = static_cast<int32_t>(act);
  check_rc(vf_gated_act_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
  return out;
}

at::Tensor gated_act_meta(const at::Tensor& gate, const std::optional<at::Tensor>&, int64_t) {
  return at::empty_like(gate);
}
at::Tensor gated_act_cpu(const at::Tensor&, const std::optional<at::Tensor>&, int64_t) {
  TORCH_CHECK(false, "vf_b200: gate and up must be CUDA tensors (no CPU implementation)");
}

// out = LayerNorm(x + residual) over the last dimension (weight, optional bias), one pass.
at::Tensor add_layer_norm(const at::Tensor& x_in, const at::Tensor& res_in, const at::Tensor& weight_in,
                          const std::optional<at::Tensor>& bias_in, double eps) {
  require_cuda(x_in, "x");
  require_cuda(res_in, "residual");
  require_cuda(weight_in, "weight");
  TORCH_CHECK(x_in.sizes() == res_in.sizes(), "vf_b200: x and residual must have identical shapes");
  TORCH_CHECK(x_in.dim() >= 1, "vf_b200: x must have at least one dimension");
  const int64_t cols = x_in.size(-1);
  TORCH_CHECK(weight_in.dim() == 1 && weight_in.size(0) == cols, "vf_b200: weight must be [", cols, "]");
  TORCH_CHECK(x_in.scalar_type() == res_in.scalar_type() && x_in.scalar_type() == weight_in.scalar_type(),
              "vf_b200: x, residual and weight must share a dtype");
  at::Tensor bias;
  if (bias_in.has_value() && bias_in->defined()) {
    require_cuda(*bias_in, "bias");
    TORCH_CHECK(bias_in->dim() == 1 && bias_in->size(0) == cols, "vf_b200: bias must be [", cols, "]");
    TORCH_CHECK(bias_in->scalar_type() == x_in.scalar_type(), "vf_b200: bias must share the dtype of x");
    bias = bias_in->contiguous();
  }
  c10::cuda::CUDAGuard guard(x_in.device());
  const int64_t rows = cols == 0 ? 0 : x_in.numel() / cols;
  at::Tensor out = at::empty(x_in.sizes(), x_in.options());
  if (rows == 0 || cols == 0) return out;
  const at::Tensor x = as_rows(x_in, rows, cols), r = as_rows(res_in, rows, cols), w = weight_in.contiguous();
  vf_add_layer_norm_args_t a{};
  a.dtype = dtype_code(x);
  a.x = x.data_ptr();
  a.residual = r.data_ptr();
  a.weight = w.data_ptr();
  a.bias = bias.defined() ? bias.data_ptr() : nullptr;
  a.out = out.data_ptr();
  a.rows = rows;
  a.cols = cols;
  a.x_row_stride = rows > 1 ? x.stride(0) : cols;
  a.residual_row_stride = rows > 1 ? r.stride(0) : cols;
  a.out_row_stride = cols;
  a.eps = static_cast<float>(eps);
  check_rc(vf_add_layer_norm_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
  return out;
}

at::Tensor add_layer_norm_meta(const at::Tensor& x, const at::Tensor&, const at::Tensor&,
                               const std::optional<at::Tensor>&, double) {
  return at::empty_like(x);
}
at::Tensor add_layer_norm_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                              const std::optional<at::Tensor>&, double) {
  TORCH_CHECK(false, "vf_b200: x and residual must be CUDA tensors (no CPU implementation)");
}

// ---------------------------------------------------------------- linear + activation
// act(x W^T + bias), or act(x W^T) * mul, over the last dimension of x (any leading shape),
// the activation in the GEMM's epilogue (vf_linear_act_fwd).
at::Tensor linear_act(const at::Tensor& x_in, const at::Tensor& w_in, const std::optional<at::Tensor>& bias_opt,
                      const std::optional<at::Tensor>& mul_opt, int64_t act) {
  require_cuda(x_in, "x");
  require_cuda(w_in, "weight");
  TORCH_CHECK(w_in.dim() == 2, "vf_b200: weight must be [out_features, in_features]");
  TORCH_CHECK(x_in.dim() >= 1 && x_in.size(-1) == w_in.size(1), "vf_b200: x's last dimension must be in_features = ",
              w_in.size(1));
  TORCH_CHECK(x_in.scalar_type() == w_in.scalar_type(), "vf_b200: x and weight must share a dtype");
  c10::cuda::CUDAGuard guard(x_in.device());
  const int64_t K = w_in.size(1), N = w_in.size(0);
  const int64_t rows = K == 0 ? 0 : x_in.numel() / K;
  std::vector<int64_t> out_shape(x_in.sizes().begin(), x_in.sizes().end());
  out_shape.back() = N;
  at::Tensor out = at::empty(out_shape, x_in.options());
  if (rows == 0) return out;
  const int64_t es = x_in.element_size();
  auto rows_ok = [&](const at::Tensor& t) {
    return t.stride(-1) == 1 && (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0 &&
           (t.size(0) <= 1 || ((t.stride(0) * es) % 16 == 0 && t.stride(0) >= t.size(1)));
  };
  at::Tensor x = as_rows(x_in, rows, K);
  if (!rows_ok(x)) x = x.contiguous();
  at::Tensor w = rows_ok(w_in) ? w_in : w_in.contiguous();
  const bool gated = mul_opt.has_value() && mul_opt->defined();
  at::Tensor bias, mul;
  if (gated) {
    // out = act(x W^T) * mul: the gated form takes no bias.
    require_cuda(*mul_opt, "mul");
    TORCH_CHECK(!(bias_opt.has_value() && bias_opt->defined()), "vf_b200: the gated form (mul) takes no bias");
    TORCH_CHECK(mul_opt->scalar_type() == x.scalar_type(), "vf_b200: mul must have x's dtype");
    TORCH_CHECK(mul_opt->numel() == rows * N && mul_opt->size(-1) == N, "vf_b200: mul must be [..., out_features] like the result");
    mul = as_rows(*mul_opt, rows, N);
    if (!rows_ok(mul)) mul = mul.contiguous();
  } else if (bias_opt.has_value() && bias_opt->defined()) {
    require_cuda(*bias_opt, "bias");
    TORCH_CHECK(bias_opt->dim() == 1 && bias_opt->size(0) == N, "vf_b200: bias must be [out_features]");
    bias = bias_opt->to(x.scalar_type()).contiguous();
  } else {
    bias = at::zeros({N}, x.options());
  }
  vf_linear_act_args_t a{};
  a.dtype = dtype_code(x);
  a.x = x.data_ptr();
  a.weight = w.data_ptr();
  a.bias = gated ? nullptr : bias.data_ptr();
  a.mul = gated ? mul.data_ptr() : nullptr;
  a.mul_row_stride = gated ? (rows > 1 ? mul.stride(0) : N) : 0;
  a.out = out.data_ptr();
  a.rows = rows;
  a.K = K;
  a.N = N;
  a.x_row_stride = rows > 1 ? x.stride(0) : K;
  a.weight_row_stride = N > 1 ? w.stride(0) : K;
  a.out_row_stride = N;
  a.act = static_cast<int32_t>(act);
  check_rc(vf_linear_act_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
  return out;
}
at::Tensor linear_act_meta(const at::Tensor& x, const at::Tensor& w, const std::optional<at::Tensor>&,
                           const std::optional<at::Tensor>&, int64_t) {
  std::vector<int64_t> out_shape(x.sizes().begin(), x.sizes().end());
  out_shape.back() = w.size(0);
  return at::empty(out_shape, x.options());
}
at::Tensor linear_act_cpu(const at::Tensor&, const at::Tensor&, const std::optional<at::Tensor>&,
                          const std::optional<at::Tensor>&, int64_t) {
  TORCH_CHECK(false, "vf_b200: x and weight must be CUDA tensors (no CPU implementation)");
}

// ---------------------------------------------------------------- GLiNER span scores
// Rows of a 2-D 16-bit operand as the kernel reads them: unit column stride, 16-byte aligned
// base and row stride (else a contiguous copy).
at::Tensor span_rows(const at::Tensor& t) {
  const int64_t es = t.element_size();
  const bool ok = t.stride(1) == 1 && (reinterpret_cast<uintptr_t>(t.data_ptr()) % 16) == 0 &&
                  (t.size(0) <= 1 || ((t.stride(0) * es) % 16 == 0 && t.stride(0) >= t.size(1)));
  return ok ? t : t.contiguous();
}

int64_t span_scores_numel(at::IntArrayRef span_offsets, at::IntArrayRef class_offsets) {
  TORCH_CHECK(span_offsets.size() == class_offsets.size() && !span_offsets.empty(),
              "vf_b200: span_offsets and class_offsets must both have num_segments + 1 entries");
  int64_t n = 0;
  for (size_t g = 0; g + 1 < span_offsets.size(); ++g) {
    const int64_t S = span_offsets[g + 1] - span_offsets[g], C = class_offsets[g + 1] - class_offsets[g];
    TORCH_CHECK(S >= 0 && C >= 0, "vf_b200: span / class offsets must not decrease");
    n += S * C;
  }
  return n;
}

// Scores of every (span, class) pair of every segment, [sum_g spans_g * classes_g] in
// out_dtype, segment g's [spans_g, classes_g] block after the previous segments' blocks.
at::Tensor span_scores(const at::Tensor& start_in, const at::Tensor& end_in, const at::Tensor& idx_in,
                       const at::Tensor& classes_in, const std::optional<at::Tensor>& bias_opt,
                       at::IntArrayRef word_offsets, at::IntArrayRef span_offsets, at::IntArrayRef class_offsets,
                       at::ScalarType out_dtype) {
  require_cuda(start_in, "start_proj");
  require_cuda(end_in, "end_proj");
  require_cuda(idx_in, "span_idx");
  require_cuda(classes_in, "classes");
  TORCH_CHECK(start_in.dim() == 2 && end_in.dim() == 2 && classes_in.dim() == 2,
              "vf_b200: start_proj, end_proj and classes must be 2-D [rows, K]");
  TORCH_CHECK(start_in.sizes() == end_in.sizes(), "vf_b200: start_proj and end_proj must have the same shape");
  TORCH_CHECK(classes_in.size(1) == start_in.size(1), "vf_b200: classes must have K = ", start_in.size(1), " columns");
  TORCH_CHECK(start_in.scalar_type() == end_in.scalar_type() && start_in.scalar_type() == classes_in.scalar_type(),
              "vf_b200: start_proj, end_proj and classes must share a dtype");
  TORCH_CHECK(idx_in.dim() == 2 && idx_in.size(1) == 2, "vf_b200: span_idx must be [spans, 2]");
  TORCH_CHECK(idx_in.scalar_type() == at::kLong || idx_in.scalar_type() == at::kInt,
              "vf_b200: span_idx must be int64 or int32");
  TORCH_CHECK(word_offsets.size() == span_offsets.size(), "vf_b200: word_offsets must have num_segments + 1 entries");
  TORCH_CHECK(out_dtype == at::kFloat || out_dtype == at::kHalf || out_dtype == at::kBFloat16,
              "vf_b200: out_dtype must be float32, float16 or bfloat16");
  const int64_t G = static_cast<int64_t>(span_offsets.size()) - 1;
  TORCH_CHECK(G <= INT32_MAX, "vf_b200: too many segments");
  TORCH_CHECK(word_offsets.back() <= start_in.size(0), "vf_b200: word_offsets run past start_proj's rows");
  TORCH_CHECK(span_offsets.back() <= idx_in.size(0), "vf_b200: span_offsets run past span_idx's rows");
  TORCH_CHECK(class_offsets.back() <= classes_in.size(0), "vf_b200: class_offsets run past classes' rows");
  c10::cuda::CUDAGuard guard(start_in.device());
  at::Tensor out = at::empty({span_scores_numel(span_offsets, class_offsets)}, start_in.options().dtype(out_dtype));
  if (out.numel() == 0) return out;
  const at::Tensor u = span_rows(start_in), v = span_rows(end_in), c = span_rows(classes_in);
  at::Tensor bias;
  if (bias_opt.has_value() && bias_opt->defined()) {
    require_cuda(*bias_opt, "class_bias");
    TORCH_CHECK(bias_opt->dim() == 1 && bias_opt->size(0) >= class_offsets.back(),
                "vf_b200: class_bias must be 1-D with a value per class");
    bias = bias_opt->to(at::kFloat).contiguous();
  }
  vf_span_scores_args_t a{};
  a.dtype = dtype_code(u);
  a.start_proj = u.data_ptr();
  a.end_proj = v.data_ptr();
  a.start_row_stride = u.size(0) > 1 ? u.stride(0) : u.size(1);
  a.end_row_stride = v.size(0) > 1 ? v.stride(0) : v.size(1);
  a.K = u.size(1);
  a.span_idx = idx_in.data_ptr();
  a.span_idx_int64 = idx_in.scalar_type() == at::kLong ? 1 : 0;
  a.idx_stride_span = idx_in.stride(0);
  a.idx_stride_pair = idx_in.stride(1);
  a.classes = c.data_ptr();
  a.class_row_stride = c.size(0) > 1 ? c.stride(0) : c.size(1);
  a.class_bias = bias.defined() ? bias.data_ptr<float>() : nullptr;
  a.out = out.data_ptr();
  a.out_dtype = dtype_code(out);
  a.num_segments = static_cast<int32_t>(G);
  a.word_offsets = word_offsets.data();
  a.span_offsets = span_offsets.data();
  a.class_offsets = class_offsets.data();
  check_rc(vf_span_scores_fwd(&a, at::cuda::getCurrentCUDAStream().stream()));
  return out;
}
at::Tensor span_scores_meta(const at::Tensor& start_proj, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                            const std::optional<at::Tensor>&, at::IntArrayRef, at::IntArrayRef span_offsets,
                            at::IntArrayRef class_offsets, at::ScalarType out_dtype) {
  return at::empty({span_scores_numel(span_offsets, class_offsets)}, start_proj.options().dtype(out_dtype));
}
at::Tensor span_scores_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                           const std::optional<at::Tensor>&, at::IntArrayRef, at::IntArrayRef, at::IntArrayRef,
                           at::ScalarType) {
  TORCH_CHECK(false, "vf_b200: start_proj must be a CUDA tensor (no CPU implementation)");
}

// Shape functions for tracing (torch.compile / fake tensors).
at::Tensor rpb_attention_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&,
                              const std::optional<at::Tensor>&, int64_t, int64_t, bool,
                              const std::optional<at::Tensor>&, double, double) {
  return at::empty_like(q);
}
at::Tensor deberta_attention_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&,
                                  const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                                  const std::optional<at::Tensor>&, bool, std::optional<double>, int64_t,
                                  int64_t, bool) {
  return at::empty_like(q);
}

at::Tensor rpb_attention_varlen_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                     int64_t, const std::optional<at::Tensor>&, int64_t, int64_t, bool, double) {
  return at::empty_like(q);
}
at::Tensor rpb_attention_varlen_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                    int64_t, const std::optional<at::Tensor>&, int64_t, int64_t, bool, double) {
  TORCH_CHECK(false, "vf_b200: q, k, v must be CUDA tensors (no CPU implementation)");
}

at::Tensor deberta_attention_varlen_meta(const at::Tensor& q, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                         int64_t, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                                         bool, std::optional<double>, int64_t, int64_t, bool) {
  return at::empty_like(q);
}
at::Tensor deberta_attention_varlen_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                        int64_t, const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                                        bool, std::optional<double>, int64_t, int64_t, bool) {
  TORCH_CHECK(false, "vf_b200: q, k, v must be CUDA tensors (no CPU implementation)");
}

at::Tensor rpb_attention_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                             const std::optional<at::Tensor>&, int64_t, int64_t, bool,
                             const std::optional<at::Tensor>&, double, double) {
  TORCH_CHECK(false, "vf_b200: q, k, v must be CUDA tensors (no CPU implementation)");
}
at::Tensor deberta_attention_cpu(const at::Tensor&, const at::Tensor&, const at::Tensor&,
                                 const std::optional<at::Tensor>&, const std::optional<at::Tensor>&,
                                 const std::optional<at::Tensor>&, bool, std::optional<double>, int64_t,
                                 int64_t, bool) {
  TORCH_CHECK(false, "vf_b200: q, k, v must be CUDA tensors (no CPU implementation)");
}

}  // namespace

TORCH_LIBRARY(vf_b200, m) {
  m.def("rpb_attention(Tensor q, Tensor k, Tensor v, Tensor? rpb_table, int num_buckets, int max_distance, "
        "bool is_decoder, Tensor? padding_mask, float dropout_p, float softmax_scale) -> Tensor");
  m.def("rpb_attention_varlen(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens, int max_seqlen, Tensor? rpb_table, "
        "int num_buckets, int max_distance, bool is_decoder, float softmax_scale) -> Tensor");
  m.def("deberta_attention(Tensor q, Tensor k, Tensor v, Tensor? seq_lengths, Tensor? pos_key, "
        "Tensor? pos_query, bool causal, float? sm_scale, int position_buckets, int max_relative_distance, "
        "bool use_log_bucket) -> Tensor");
  m.def("gated_act(Tensor gate, Tensor? up, int act) -> Tensor");
  m.def("add_layer_norm(Tensor x, Tensor residual, Tensor weight, Tensor? bias, float eps) -> Tensor");
  m.def("deberta_attention_varlen(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens, int max_seqlen, Tensor? pos_key, "
        "Tensor? pos_query, bool causal, float? sm_scale, int position_buckets, int max_relative_distance, "
        "bool use_log_bucket) -> Tensor");
  m.def("deberta_attention_fused(Tensor q, Tensor k, Tensor v, Tensor? seq_lengths, Tensor? rel_key, "
        "Tensor? rel_query, bool causal, float? sm_scale, int position_buckets, int max_relative_distance, "
        "bool use_log_bucket) -> Tensor");
  m.def("deberta_attention_fused_varlen(Tensor q, Tensor k, Tensor v, Tensor cu_seqlens, int max_seqlen, "
        "Tensor? rel_key, Tensor? rel_query, bool causal, float? sm_scale, int position_buckets, "
        "int max_relative_distance, bool use_log_bucket) -> Tensor");
  m.def("linear_act(Tensor x, Tensor weight, Tensor? bias, Tensor? mul, int act) -> Tensor");
  m.def("span_scores(Tensor start_proj, Tensor end_proj, Tensor span_idx, Tensor classes, Tensor? class_bias, "
        "int[] word_offsets, int[] span_offsets, int[] class_offsets, ScalarType out_dtype) -> Tensor");
}

TORCH_LIBRARY_IMPL(vf_b200, CUDA, m) {
  m.impl("rpb_attention", &rpb_attention);
  m.impl("rpb_attention_varlen", &rpb_attention_varlen);
  m.impl("deberta_attention", &deberta_attention);
  m.impl("deberta_attention_varlen", &deberta_attention_varlen);
  m.impl("deberta_attention_fused", &deberta_attention_fused);
  m.impl("deberta_attention_fused_varlen", &deberta_attention_fused_varlen);
  m.impl("gated_act", &gated_act);
  m.impl("add_layer_norm", &add_layer_norm);
  m.impl("span_scores", &span_scores);
  m.impl("linear_act", &linear_act);
}

TORCH_LIBRARY_IMPL(vf_b200, CPU, m) {
  m.impl("rpb_attention", &rpb_attention_cpu);
  m.impl("rpb_attention_varlen", &rpb_attention_varlen_cpu);
  m.impl("deberta_attention", &deberta_attention_cpu);
  m.impl("deberta_attention_varlen", &deberta_attention_varlen_cpu);
  m.impl("deberta_attention_fused", &deberta_attention_fused_cpu);
  m.impl("deberta_attention_fused_varlen", &deberta_attention_fused_varlen_cpu);
  m.impl("gated_act", &gated_act_cpu);
  m.impl("add_layer_norm", &add_layer_norm_cpu);
  m.impl("span_scores", &span_scores_cpu);
  m.impl("linear_act", &linear_act_cpu);
}

TORCH_LIBRARY_IMPL(vf_b200, Meta, m) {
  m.impl("rpb_attention", &rpb_attention_meta);
  m.impl("rpb_attention_varlen", &rpb_attention_varlen_meta);
  m.impl("deberta_attention", &deberta_attention_meta);
  m.impl("deberta_attention_varlen", &deberta_attention_varlen_meta);
  m.impl("deberta_attention_fused", &deberta_attention_meta);
  m.impl("deberta_attention_fused_varlen", &deberta_attention_varlen_meta);
  m.impl("gated_act", &gated_act_meta);
  m.impl("add_layer_norm", &add_layer_norm_meta);
  m.impl("span_scores", &span_scores_meta);
  m.impl("linear_act", &linear_act_meta);
}
