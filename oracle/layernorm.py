"""CPU restatement of the DeBERTa-v2 residual add + LayerNorm (test infrastructure only).

models/deberta_v2/deberta_v2_encoder.py:507 and :566: `self.LayerNorm(hidden_states +
input_tensor)` with nn.LayerNorm(hidden_size, eps=layer_norm_eps).  The add is done in the
input dtype (torch rounds the sum to it), the normalisation in float64 here: mean, biased
variance, (s - mean) / sqrt(var + eps) * weight + bias; the result is cast to the input
dtype (or returned in float64 with dtype=torch.float64).
"""
from __future__ import annotations

from typing import Optional

import torch


def add_layer_norm_ref(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                       bias: Optional[torch.Tensor], eps: float, dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    s = (x + residual).double()                       # the sum, rounded to x.dtype by the add
    mean = s.mean(dim=-1, keepdim=True)
    var = ((s - mean) ** 2).mean(dim=-1, keepdim=True)
    y = (s - mean) / torch.sqrt(var + eps) * weight.double()
    if bias is not None:
        y = y + bias.double()
    return y.to(dtype or x.dtype)
