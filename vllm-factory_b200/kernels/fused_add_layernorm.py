"""Residual add + LayerNorm of the DeBERTa-v2 encoder in one pass.

In vllm-factory the two output blocks of every DeBERTa layer end with
`self.LayerNorm(hidden_states + input_tensor)` (models/deberta_v2/deberta_v2_encoder.py:507,
DebertaV2SelfOutput; :566, DebertaV2Output): two torch kernels, with the sum written to HBM
and read back.  `fused_add_layer_norm` computes the same result in one sm_100a kernel of
libvf_b200.so: the sum rounded to the input dtype (as the tensor add stores it), mean and
biased variance in fp32, weight and bias applied in fp32, result in the input dtype.  There
is no Triton and no CPU path; the reference has no kernel of its own for this step.
"""
from __future__ import annotations

from typing import Optional

import torch

import vf_b200.ops  # noqa: F401  (loads the kernels and registers torch.ops.vf_b200)


def fused_add_layer_norm(
    hidden_states: torch.Tensor,
    input_tensor: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor] = None,
    eps: float = 1e-7,
) -> torch.Tensor:
    """LayerNorm(hidden_states + input_tensor) over the last dimension.  hidden_states,
    input_tensor, weight and bias share one dtype (float32, float16 or bfloat16) and one CUDA
    device; only the last dimension needs unit stride.  Shapes, dtypes and devices are
    checked here, before the op: ValueError / TypeError / RuntimeError (CPU tensors)."""
    if hidden_states.dim() < 1 or input_tensor.shape != hidden_states.shape:
        raise ValueError(f"hidden_states {tuple(hidden_states.shape)} and input_tensor "
                         f"{tuple(input_tensor.shape)} must have one identical shape")
    cols = hidden_states.shape[-1]
    for name, t in (("weight", weight), ("bias", bias)):
        if t is not None and (t.dim() != 1 or t.shape[0] != cols):
            raise ValueError(f"{name} must be [{cols}], got {tuple(t.shape)}")
    tensors = [t for t in (hidden_states, input_tensor, weight, bias) if t is not None]
    if any(t.dtype != hidden_states.dtype for t in tensors):
        raise TypeError("hidden_states, input_tensor, weight and bias must share one dtype")
    if not all(t.is_cuda and t.device == hidden_states.device for t in tensors):
        raise RuntimeError("vf_b200: all operands must be CUDA tensors on one device (no CPU implementation)")
    return torch.ops.vf_b200.add_layer_norm(hidden_states, input_tensor, weight, bias, float(eps))


__all__ = ["fused_add_layer_norm"]
