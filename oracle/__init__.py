"""CPU oracle for the relative-position attention hot path — TEST INFRASTRUCTURE ONLY.

Nothing in the product imports this package.  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm may call it, and only as the checker or as the
timed CPU baseline, never as the thing measured on the GPU.

It restates, in plain PyTorch on the CPU, the reference's own algorithms for the path
(vllm-factory 0.2.2):
  * T5 bucket:        models/mt5/mt5_encoder.py:125-148 (T5RelativePositionBias._relative_position_bucket)
  * T5 dense bias:    models/mt5/mt5_encoder.py:150-164 + :75-110 (_make_contiguous_additive_bias)
  * T5 attention:     models/mt5/mt5_encoder.py:309-316 (SDPA, scale=1.0), equal in exact
                      arithmetic to kernels/flash_attention_rpb.py:62-230; the packed form
                      applies it to each cu_seqlens sequence alone
  * DeBERTa bucket:   models/deberta_v2/deberta_v2_encoder.py:70-89 (make_log_bucket_position)
  * DeBERTa op:       kernels/flash_deberta_attention.py:375-448 (_pytorch_flash_deberta_fwd),
                      with the Triton kernel's row semantics (rows >= seq_len are 0,
                      :295-299, :334); the packed form applies it to each cu_seqlens
                      sequence alone
  * DeBERTa layer:    models/deberta_v2/deberta_v2_encoder.py:332-487 (_pytorch_forward)
  * DeBERTa fused:    the caller's products q @ Kr^T, k @ Qr^T (:275-286) + the op above
  * mT5 FFN act:      kernels/ff_fused.py:23-74 (fused_gelu_mul_dropout's kernel, no dropout)
  * DeBERTa FFN in:   models/deberta_v2/deberta_v2_encoder.py:547-550 (dense + exact GELU)
  * GLiNER spans:     poolers/gliner.py:26-45, :118-140, :285-289 (SpanMarkerV0 + class einsum)

Parity pinning: tests/golden/make_golden.py runs the reference's own functions (imported
from the read-only reference checkout in the build container) and commits their outputs
under tests/golden/; tests/test_oracle_golden.py checks this oracle against them.
"""
from .rpb import (  # noqa: F401
    deberta_attention_fused_ref,
    deberta_attention_fused_varlen_ref,
    deberta_attention_ref,
    deberta_attention_varlen_ref,
    deberta_layer_ref,
    deberta_log_bucket_ref,
    rpb_attention_ref,
    rpb_attention_varlen_ref,
    t5_bias_dense_ref,
    t5_relative_bucket_ref,
)
from .ffn import gated_act_ref, linear_gelu_ref  # noqa: F401,E402
from .layernorm import add_layer_norm_ref  # noqa: F401,E402
from .span import (  # noqa: F401,E402
    span_factors_ref,
    span_rep_ref,
    span_scores_factored_ref,
    span_scores_from_factors_ref,
    span_scores_ref,
)
