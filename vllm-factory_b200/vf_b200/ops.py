"""torch.ops.vf_b200.* — loads the C++ op layer (libvf_b200_torch.so).

The ops are defined and implemented in csrc/vf_torch_ops.cpp, which reads tensor sizes,
strides and the current CUDA stream and calls the C ABI of libvf_b200.so:

  torch.ops.vf_b200.rpb_attention(q, k, v, rpb_table?, num_buckets, max_distance,
                                  is_decoder, padding_mask?, dropout_p, softmax_scale)
  torch.ops.vf_b200.rpb_attention_varlen(q, k, v, cu_seqlens, max_seqlen, rpb_table?,
                                         num_buckets, max_distance, is_decoder,
                                         softmax_scale)      # packed [total, H, 64]
  torch.ops.vf_b200.deberta_attention(q, k, v, seq_lengths?, pos_key?, pos_query?, causal,
                                      sm_scale?, position_buckets, max_relative_distance,
                                      use_log_bucket)
  torch.ops.vf_b200.deberta_attention_varlen(q, k, v, cu_seqlens, max_seqlen, pos_key?,
                                             pos_query?, causal, sm_scale?, position_buckets,
                                             max_relative_distance, use_log_bucket)   # packed

  torch.ops.vf_b200.deberta_attention_fused(q, k, v, seq_lengths?, rel_key?, rel_query?, causal,
                                            sm_scale?, position_buckets, max_relative_distance,
                                            use_log_bucket)   # position products in the kernel
  torch.ops.vf_b200.deberta_attention_fused_varlen(q, k, v, cu_seqlens, max_seqlen, rel_key?,
                                                   rel_query?, ...)                    # packed
  torch.ops.vf_b200.gated_act(gate, up, act)                  # mT5 FFN: act(gate) * up (up=None: act(gate))
  torch.ops.vf_b200.add_layer_norm(x, residual, w, b, eps)   # DeBERTa: LayerNorm(x + residual)

All borrow their inputs (layouts TMA cannot describe are copied contiguous), allocate
only the output, launch on the caller's stream, and have Meta implementations for
tracing.  CPU tensors raise: there is no CPU implementation.
"""
from __future__ import annotations

from pathlib import Path

import torch

from . import _lib

TORCH_LIB_PATH = Path(__file__).resolve().parent / "libvf_b200_torch.so"

_lib.load()   # the kernel library first: the op layer links against it
if not TORCH_LIB_PATH.exists():
    raise RuntimeError(f"{TORCH_LIB_PATH} not found: build it with `python -m vf_b200.build`; "
                       "there is no fallback implementation")
torch.ops.load_library(str(TORCH_LIB_PATH))

rpb_attention = torch.ops.vf_b200.rpb_attention
rpb_attention_varlen = torch.ops.vf_b200.rpb_attention_varlen
deberta_attention = torch.ops.vf_b200.deberta_attention
deberta_attention_varlen = torch.ops.vf_b200.deberta_attention_varlen
deberta_attention_fused = torch.ops.vf_b200.deberta_attention_fused
deberta_attention_fused_varlen = torch.ops.vf_b200.deberta_attention_fused_varlen
gated_act = torch.ops.vf_b200.gated_act
add_layer_norm = torch.ops.vf_b200.add_layer_norm
