/*
 * vf_b200 — C ABI of the sm_100a relative-position encoder attention kernels.
 *
 * Plain pointers, sizes and strides only; no torch types cross this boundary.  All
 * tensor pointers are DEVICE pointers on the current CUDA device; `stream` is a
 * cudaStream_t (NULL = legacy default stream).  Every entry point returns 0 on success
 * or a negative VF_E* code; vf_last_error() then holds a one-line message for the
 * calling thread.  Nothing here allocates device memory: callers own every buffer.
 *
 * The reference (vllm-factory 0.2.2) has no native layer: its two hot-path operators
 * are Python launchers of Triton kernels.  Each entry point below names the Python
 * interface it replaces, and the ctypes binding in vllm-factory_b200/vf_b200/_lib.py is
 * the binding a maintainer of the reference would add.
 */
#ifndef VF_B200_H_
#define VF_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; exactly the entry points below are exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define VF_ABI_VERSION 1

/* Error codes. */
#define VF_OK 0
#define VF_EINVAL (-1)       /* bad shape, stride, dtype or argument value            */
#define VF_EUNSUPPORTED (-2) /* valid for the reference but not implemented here     */
#define VF_ECUDA (-3)        /* a CUDA runtime / driver call failed                  */

typedef enum {
  VF_DTYPE_F32 = 0,
  VF_DTYPE_F16 = 1,
  VF_DTYPE_BF16 = 2,
} vf_dtype_t;

/* A rank-4 strided view.  Strides are in ELEMENTS.  data == NULL means "absent". */
typedef struct {
  const void* data;
  int64_t size[4];
  int64_t stride[4];
} vf_tensor4d_t;

/* ------------------------------------------------------------------------------------
 * T5 relative-position-bias attention (mT5 encoder self-attention).
 * Replaces kernels/flash_attention_rpb.py:296 `flash_attention_rpb_final(q, k, v,
 * rpb_table, num_buckets, max_distance, is_decoder, padding_mask=None, dropout_p=0.0,
 * softmax_scale=1.0, use_autotune=True)` and its kernel (:62-230).
 *
 *   out[b,h,m,:] = softmax_n( scale * q[b,h,m]·k[b,h,n]
 *                              + rpb_table[bucket(n - m), h] + padding_mask[b,h,m,n] ) v[b,h,n,:]
 *
 * q, k, v, out: (B, H, M|N, 64), dtype 16-bit (f16/bf16), innermost stride 1.
 * rpb_table: (num_table_rows, H) 2-D with the given element strides, or NULL (no bias).
 * padding_mask: additive, broadcastable (B|1, H|1, 1|M, N), bf16 / f16 / f32 (mask_dtype);
 * data NULL = none.  A mask that broadcasts over query rows (1) is staged per key tile:
 * rows of a batch whose mask is <= -1e4 on every key of a 128-key tile make that tile
 * contribute exactly zero, so such tiles at either end are skipped.  A mask that varies
 * over query rows (M; the reference reads it with stride_mask_m, :182-185) is added per
 * score by a second kernel instance that visits every key tile.
 * ------------------------------------------------------------------------------------ */
typedef struct {
  vf_dtype_t dtype;
  vf_tensor4d_t q, k, v;
  vf_tensor4d_t out;
  const void* rpb_table;
  int64_t table_rows, table_cols;
  int64_t table_stride_row, table_stride_col;
  vf_dtype_t table_dtype;
  int32_t num_buckets;
  int32_t max_distance;
  int32_t is_decoder;
  vf_tensor4d_t padding_mask;
  vf_dtype_t mask_dtype;
  float dropout_p;
  float softmax_scale;
} vf_rpb_attention_args_t;

int vf_rpb_attention_fwd(const vf_rpb_attention_args_t* args, void* stream);

/* Packed variable-length batch of the same operator: sequence s occupies rows
 * [cu_seqlens[s], cu_seqlens[s+1]) of q, k, v and out, and attends only within itself.
 * Replaces the flat-as-one-sequence call of plugins/mt5_gliner/model.py:178-192 (which
 * lets the requests of one batch attend to each other) and the pad/unpad round trip
 * around kernels/flash_attention_rpb.py:296; the reference has no packed entry point.
 *
 * q, k, v, out: views of size (1, H, total, 64) (a [total, H, 64] tensor has strides
 * (total*H*64, 64, H*64, 1)); k has the rows of q.  cu_seqlens: device int32[num_seqs+1],
 * non-decreasing, cu_seqlens[0] >= 0, cu_seqlens[num_seqs] <= total.  max_seqlen: host
 * bound >= every sequence length (sizes the bucket table and the work list).  padding_mask
 * must be absent.  Rows of out outside every sequence are not written.  Offsets that break
 * these rules set bit 2 of vf_device_error(); the rows used are clamped into the views. */
int vf_rpb_attention_varlen_fwd(const vf_rpb_attention_args_t* args, const int32_t* cu_seqlens,
                                int32_t num_seqs, int32_t max_seqlen, void* stream);

/* ------------------------------------------------------------------------------------
 * DeBERTa disentangled attention (c2p + p2c relative-position scores).
 * Replaces kernels/flash_deberta_attention.py:455 `flash_deberta_attention(q, k, v,
 * seq_lengths=None, pos_key=None, pos_query=None, causal=False, sm_scale=None,
 * position_buckets=0, max_relative_distance=0, use_log_bucket=False)` and its Triton
 * launcher/kernel (:306-372, :145-299).
 *
 *   idx(m, n) = clamp(bucket(m - n) + S, 0, 2S - 1),   S = position_buckets or max_rel
 *   s[m, n]   = sm_scale * (q[m]·k[n] + pos_key[m, idx] + pos_query[n, idx])
 *   out[m]    = softmax over keys n < seq_len(b) of s, times v;  rows m >= seq_len -> 0
 *
 * q, out: (B, H, M, 64); k, v: (B, H, N, 64); 16-bit dtype; innermost stride 1.
 * pos_key: (B, H, M, 2S), pos_query: (B, H, N, 2S), same dtype as q; NULL = term absent.
 * seq_lengths: device int32 (B,) or NULL (all rows/keys valid).
 * has_sm_scale == 0 selects the reference default 1/sqrt(head_dim).
 * ------------------------------------------------------------------------------------ */
typedef struct {
  vf_dtype_t dtype;
  vf_tensor4d_t q, k, v;
  vf_tensor4d_t out;
  const int32_t* seq_lengths;
  vf_tensor4d_t pos_key, pos_query;
  int32_t causal;
  int32_t has_sm_scale;
  float sm_scale;
  int32_t position_buckets;
  int32_t max_relative_distance;
  int32_t use_log_bucket;
} vf_deberta_attention_args_t;

int vf_deberta_attention_fwd(const vf_deberta_attention_args_t* args, void* stream);

/* Packed variable-length batch of the same operator (no counterpart in the reference):
 * sequence s occupies rows [cu_seqlens[s], cu_seqlens[s+1]) of q, k, v, out and of the
 * position tensors, and attends only within itself, with causal masking (if set) inside
 * each sequence.  Replaces the pad/unpad loops around kernels/flash_deberta_attention.py:455
 * in plugins/deberta_gliner/model.py:361-399 and plugins/deberta_gliner_linker/model.py:
 * 170-228, and the flat-as-one-sequence call of plugins/deberta_gliner2/model.py:125-139.
 *
 * q, k, v, out: views of size (1, H, total, 64); pos_key / pos_query: (1, H, total, 2S)
 * or absent.  seq_lengths must be NULL.  cu_seqlens, num_seqs, max_seqlen: as for
 * vf_rpb_attention_varlen_fwd (same rules, same error bit).  Rows of out outside every
 * sequence are not written. */
int vf_deberta_attention_varlen_fwd(const vf_deberta_attention_args_t* args, const int32_t* cu_seqlens,
                                    int32_t num_seqs, int32_t max_seqlen, void* stream);

/* ------------------------------------------------------------------------------------
 * DeBERTa disentangled attention with the position contractions inside the kernel (the
 * "fused" mode).  Same operator as vf_deberta_attention_fwd, but the caller passes the
 * projected position tables instead of their products with q and k:
 *   rel_key   = key_proj(rel_embeddings)   as (1, H, 2S, 64)   (Kr)
 *   rel_query = query_proj(rel_embeddings) as (1, H, 2S, 64)   (Qr)
 * and the kernel forms pos_key[m, idx] = q[m]·Kr[idx] and pos_query[n, idx] = k[n]·Qr[idx]
 * on the tensor cores, tile by tile, so the two (B, H, L, 2S) tensors of
 * models/deberta_v2/deberta_v2_encoder.py:275-286 are never built.  Replaces that caller's
 * two torch.matmul products together with kernels/flash_deberta_attention.py:455; the
 * reference has no fused entry point.
 *
 * q, k, v, out, seq_lengths, causal, sm_scale, position_buckets, max_relative_distance,
 * use_log_bucket: as vf_deberta_attention_args_t.  rel_key / rel_query: 16-bit views of the
 * dtype of q, size (1, H, >= 2S, 64), unit innermost stride, 16-byte aligned rows; data NULL
 * = that term absent.  Sequences of at most 65536 positions.
 * workspace: device scratch of at least vf_deberta_fused_workspace_bytes() bytes, 256-byte
 * aligned, owned by the caller, only used by the call's own kernels (a call on another
 * stream needs its own).  It holds the position tables expanded to one row per relative
 * position (2 x H x (ceil128(M) + ceil128(N)) x 64 elements) and the unit order.
 * ------------------------------------------------------------------------------------ */
typedef struct {
  vf_dtype_t dtype;
  vf_tensor4d_t q, k, v;
  vf_tensor4d_t out;
  const int32_t* seq_lengths;
  vf_tensor4d_t rel_key, rel_query;
  int32_t causal;
  int32_t has_sm_scale;
  float sm_scale;
  int32_t position_buckets;
  int32_t max_relative_distance;
  int32_t use_log_bucket;
} vf_deberta_fused_args_t;

/* Workspace bytes of the fused entry points: batch rows (or packed sequences), heads and the
 * query / key lengths (max_seqlen for the packed form).  Negative VF_E* code on bad sizes. */
int64_t vf_deberta_fused_workspace_bytes(int64_t batch_or_seqs, int64_t heads, int64_t M, int64_t N);

int vf_deberta_attention_fused_fwd(const vf_deberta_fused_args_t* args, void* workspace, int64_t workspace_bytes,
                                   void* stream);

/* Packed variable-length batch of the fused operator: q, k, v, out are (1, H, total, 64)
 * views, sequence s is rows [cu_seqlens[s], cu_seqlens[s+1]) and attends within itself;
 * seq_lengths must be NULL; cu_seqlens / num_seqs / max_seqlen as for
 * vf_deberta_attention_varlen_fwd.  Rows of out outside every sequence are not written. */
int vf_deberta_attention_fused_varlen_fwd(const vf_deberta_fused_args_t* args, const int32_t* cu_seqlens,
                                          int32_t num_seqs, int32_t max_seqlen, void* workspace,
                                          int64_t workspace_bytes, void* stream);

/* The fused operator for callers that cannot allocate device memory per call; it has no
 * counterpart in the reference.  An FFI host (cgo, JNI, ctypes) that embeds this library
 * without a CUDA allocator of its own, or a serving process whose device memory is reserved
 * up front by its own pool (the KV-cache reservation of a vLLM-style engine), may have no
 * way to provide the workspace of vf_deberta_attention_fused_fwd.  This entry point takes
 * the same arguments minus the workspace and uses a fixed 8 MiB scratch array compiled into
 * the library instead (held by every GPU that loads the library, until the process exits).
 * It calls no cudaMalloc, cudaFree or allocating library routine.
 * Limit: the call's scratch, vf_deberta_fused_workspace_bytes(B, H, M, N), must be at most
 * 8 MiB (for example H = 16 with ceil128(M) + ceil128(N) <= 2048); larger calls return
 * VF_EUNSUPPORTED before any launch.
 * The first call on a device looks up the scratch array's device address (once per device,
 * with that device current); make that first call before any stream capture.  Every call
 * shares the one array, so calls that overlap on the GPU (other streams, other host
 * threads) race; nothing in it needs to start at zero, each call rewrites what it reads. */
int vf_deberta_attention_fused_noalloc_fwd(const vf_deberta_fused_args_t* args, void* stream);

/* ------------------------------------------------------------------------------------
 * Gated activation of the mT5 feed-forward: out = act(gate) * up, in fp32, rounded to the
 * dtype.  Replaces kernels/ff_fused.py:86 `fused_gelu_mul_dropout(gate, up, act_fn,
 * dropout_p, training)` and its kernel (:23-74) on the inference path (no dropout).
 * gate, up, out: rows x cols views of one dtype (f32/f16/bf16) with unit column stride and
 * the given row strides in elements (>= cols); e.g. the two halves of a stacked [T, 2F]
 * projection.  act: VF_ACT_GELU_TANH for 'gelu' / 'gelu_new' / 'gelu_fast' /
 * 'gelu_pytorch_tanh', VF_ACT_GELU_ERF for 'gelu_accurate', VF_ACT_RELU, VF_ACT_SILU
 * ('silu' / 'swish') -- the reference's _act_type_map (:77-85).
 * up = NULL (up_row_stride ignored) computes the plain activation out = act(gate): the
 * DeBERTa feed-forward's `intermediate_act_fn` (models/deberta_v2/deberta_v2_encoder.py,
 * exact GELU), which the reference leaves to torch; no counterpart kernel there.
 * ------------------------------------------------------------------------------------ */
enum { VF_ACT_GELU_TANH = 0, VF_ACT_GELU_ERF = 1, VF_ACT_RELU = 2, VF_ACT_SILU = 3 };

typedef struct {
  vf_dtype_t dtype;
  const void* gate;
  const void* up;
  void* out;
  int64_t rows, cols;
  int64_t gate_row_stride, up_row_stride, out_row_stride;
  int32_t act;
} vf_gated_act_args_t;

int vf_gated_act_fwd(const vf_gated_act_args_t* args, void* stream);

/* ------------------------------------------------------------------------------------
 * Linear + activation of the encoder feed-forwards, the activation applied to the fp32
 * accumulator in the GEMM's epilogue.  Replaces
 * models/deberta_v2/deberta_v2_encoder.py:547-550 (DebertaV2Intermediate.forward:
 * `self.dense(hidden_states)` then `self.intermediate_act_fn`, ACT2FN["gelu"] = exact GELU),
 * two torch calls with the [rows, N] intermediate in HBM between them.
 * x: [rows, K], weight: [N, K] (nn.Linear layout), bias: [N] (required), out: [rows, N];
 * one 16-bit dtype, unit column strides, row strides in elements; K, N and every row stride
 * multiples of 8, pointers 16-byte aligned; out must not overlap the inputs.  Built forms:
 *  - act = VF_ACT_GELU_ERF, bias given, mul = NULL: out = GELU(x W^T + bias), GELU the exact
 *    0.5 z (1 + erf(z / sqrt 2));
 *  - act = VF_ACT_GELU_TANH, bias = NULL, mul given: out = GELU_tanh(x W^T) * mul, the gated
 *    activation of the mT5 feed-forward (models/mt5/mt5_encoder.py:427-437 calling
 *    kernels/ff_fused.py:86 with "gelu_new"): W = wi_0 (gate), mul = x wi_1^T (up, [rows, N],
 *    row stride mul_row_stride), replacing the stacked projection + vf_gated_act_fwd pass.
 * ------------------------------------------------------------------------------------ */
typedef struct {
  vf_dtype_t dtype;
  const void* x;
  const void* weight;
  const void* bias;
  const void* mul;
  void* out;
  int64_t rows, K, N;
  int64_t x_row_stride, weight_row_stride, mul_row_stride, out_row_stride;
  int32_t act;
} vf_linear_act_args_t;

int vf_linear_act_fwd(const vf_linear_act_args_t* args, void* stream);

/* ------------------------------------------------------------------------------------
 * Residual add + LayerNorm of the DeBERTa-v2 encoder: out = LayerNorm(x + residual) with
 * weight and bias over the last dimension.  Replaces the two torch kernels of
 * models/deberta_v2/deberta_v2_encoder.py:507 and :566 (`self.LayerNorm(hidden_states +
 * input_tensor)`, nn.LayerNorm) -- a torch call in the reference, not a kernel of its own.
 * The sum is rounded to the dtype (as the reference's tensor add stores it); mean, biased
 * variance and the affine map in fp32; result rounded to the dtype.
 * x, residual, out: rows x cols views of one dtype (f32/f16/bf16), unit column stride, row
 * strides in elements (>= cols); out must not overlap x or residual.  weight, bias: [cols]
 * of the same dtype; bias may be NULL (zero).  eps: finite, >= 0.
 * ------------------------------------------------------------------------------------ */
typedef struct {
  vf_dtype_t dtype;
  const void* x;
  const void* residual;
  const void* weight;
  const void* bias;
  void* out;
  int64_t rows, cols;
  int64_t x_row_stride, residual_row_stride, out_row_stride;
  float eps;
} vf_add_layer_norm_args_t;

int vf_add_layer_norm_fwd(const vf_add_layer_norm_args_t* args, void* stream);

/* ------------------------------------------------------------------------------------
 * GLiNER span scores.  Replaces the span-representation MLP and the class einsum of
 * poolers/gliner.py:118-140 (SpanMarkerV0.forward) and :285-289 (GLiNERSpanPooler.forward:
 * `span_rep = self.span_rep(we, span_idx_masked)`, `scores = torch.einsum("BLKD,BCD->BLKC",
 * span_rep, pe)`); the same marker scores GLiNER2 fields (poolers/gliner2.py:230-259, :384-404).
 * With out_project = Linear(2D, 4D) [W1 = (W1a | W1b), b1] -> ReLU -> Linear(4D, D) [W2, b2],
 * the caller passes per-word and per-class products instead of the per-span MLP:
 *   start_proj = relu(start_rep) W1a^T + b1     [words, K]   (K = 4D)
 *   end_proj   = relu(end_rep)   W1b^T          [words, K]
 *   classes    = pe W2                          [classes, K]
 *   class_bias = pe . b2 (fp32)                 [classes], or NULL
 * and the kernel computes, for span s = (i_s, j_s) of segment g and class c of segment g,
 *   out[s, c] = class_bias[c] + sum_k relu(start_proj[i_s, k] + end_proj[j_s, k]) * classes[c, k]
 * (relu(a + b) rounded once to the 16-bit dtype; products and sum in fp32 on the tensor cores),
 * which equals einsum(out_project(relu(cat(start_rep[i], end_rep[j]))), pe) of the reference.
 * Span indices are local to the segment and clamped to [0, words_g - 1] as the reference's
 * extract_elements clamps them (a masked span, index (0, 0), scores word 0's span).
 * Segments (sentences) g = 0 .. num_segments - 1 are independent: words [word_offsets[g],
 * word_offsets[g+1]) of start_proj / end_proj, spans [span_offsets[g], span_offsets[g+1]) of
 * span_idx, classes [class_offsets[g], class_offsets[g+1]) of classes / class_bias; the
 * offsets are HOST arrays of num_segments + 1 non-decreasing entries.  Segment g's scores are a
 * [spans_g, classes_g] row-major block of `out`, the blocks back to back in segment order
 * (out holds sum_g spans_g * classes_g elements of out_dtype).
 * start_proj, end_proj, classes: 16-bit (f16 / bf16) rows with unit column stride, 16-byte
 * aligned rows, row strides >= K in elements; K a multiple of 64.  span_idx: int64 when
 * span_idx_int64 != 0, else int32; element (s, e) at s * idx_stride_span + e * idx_stride_pair.
 * ------------------------------------------------------------------------------------ */
typedef struct {
  vf_dtype_t dtype;
  const void* start_proj;
  const void* end_proj;
  int64_t start_row_stride, end_row_stride;
  int64_t K;
  const void* span_idx;
  int32_t span_idx_int64;
  int64_t idx_stride_span, idx_stride_pair;
  const void* classes;
  int64_t class_row_stride;
  const float* class_bias;
  void* out;
  vf_dtype_t out_dtype;
  int32_t num_segments;
  const int64_t* word_offsets;
  const int64_t* span_offsets;
  const int64_t* class_offsets;
} vf_span_scores_args_t;

int vf_span_scores_fwd(const vf_span_scores_args_t* args, void* stream);

/* ------------------------------------------------------------------------------------
 * Host-side bucket functions (no GPU needed).  These are the exact integer outputs the
 * kernels use; they restate, in float32 arithmetic like the reference's torch code:
 *  - models/mt5/mt5_encoder.py:125 T5RelativePositionBias._relative_position_bucket
 *    (also the in-kernel copy kernels/flash_attention_rpb.py:13 _get_rp_bucket);
 *  - models/deberta_v2/deberta_v2_encoder.py:70 make_log_bucket_position (also the
 *    in-kernel copy kernels/flash_deberta_attention.py:234-243).
 * They fill out[i] for relative positions r = rmin + i, i in [0, rmax - rmin].
 * ------------------------------------------------------------------------------------ */
int vf_t5_relative_bucket(int32_t num_buckets, int32_t max_distance, int32_t bidirectional,
                          int32_t rmin, int32_t rmax, int32_t* out);
int vf_deberta_log_bucket(int32_t bucket_size, int32_t max_position,
                          int32_t rmin, int32_t rmax, int32_t* out);

/* Thread-local message for the last failing call on this thread ("" if none). */
const char* vf_last_error(void);

/* Reads (and optionally clears) the device error word of the current device: bit 0 = a
 * bounded in-kernel wait ran out of time, bit 1 = a gather index failed its bounds check,
 * bit 2 = packed-batch offsets broke the rules of the *_varlen_fwd entry points.
 * Synchronises the device.  Returns the word (>= 0) or VF_ECUDA. */
int vf_device_error(int32_t clear);

/* Failure-detection self-test (no counterpart in the reference): launches one CTA whose
 * bounded wait is on an mbarrier that nothing arrives at.  After `limit_cycles` SM cycles
 * the wait gives up and sets bit 0 of the device error word (read it with
 * vf_device_error); the kernel returns and the context stays usable.  Synchronises
 * `stream`.  Returns 0 or a negative VF_E* code. */
int vf_selftest_wait_timeout(int64_t limit_cycles, void* stream);

/* VF_ABI_VERSION of the loaded library. */
int vf_abi_version(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* VF_B200_H_ */
