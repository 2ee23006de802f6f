"""CPU restatement of the reference's gated feed-forward activation (test infrastructure only).

kernels/ff_fused.py:23-74 (_fused_gelu_mul_dropout_kernel), inference path: the activation
in fp32, the product with `up` in fp32, the result cast to the input dtype.  The tanh of the
GELU is written as the reference kernel writes it, 2 * sigmoid(2 * inner) - 1 (:50-53).
"""
from __future__ import annotations

import torch

ACT_GELU_TANH, ACT_GELU_ERF, ACT_RELU, ACT_SILU = 0, 1, 2, 3


def gated_act_ref(gate: torch.Tensor, up, act: int = ACT_GELU_TANH) -> torch.Tensor:
    """act(gate) * up in fp32, cast to gate's dtype; up = None gives act(gate) alone (the
    DeBERTa feed-forward's activation, models/deberta_v2/deberta_v2_encoder.py)."""
    g = gate.float()
    if act == ACT_GELU_TANH:
        inner = 0.7978845834732056 * (g + 0.044715 * g * g * g)     # :48-51
        g = 0.5 * g * (1.0 + (2.0 * torch.sigmoid(2.0 * inner) - 1.0))
    elif act == ACT_GELU_ERF:
        g = 0.5 * g * (1.0 + torch.erf(g * 0.7071067811865476))      # :55
    elif act == ACT_RELU:
        g = torch.clamp_min(g, 0.0)
    else:
        g = g * torch.sigmoid(g)
    return (g if up is None else g * up.float()).to(gate.dtype)


def linear_gelu_ref(x: torch.Tensor, weight: torch.Tensor, bias, dtype=torch.float64) -> torch.Tensor:
    """DebertaV2Intermediate.forward (models/deberta_v2/deberta_v2_encoder.py:547-550): the dense
    layer (ColumnParallelLinear at one rank: x W^T + b) then ACT2FN["gelu"], the exact GELU
    0.5 x (1 + erf(x / sqrt 2)); in `dtype` arithmetic."""
    y = x.to(dtype) @ weight.to(dtype).T
    if bias is not None:
        y = y + bias.to(dtype)
    return 0.5 * y * (1.0 + torch.erf(y * 0.7071067811865476))
