"""Gated feed-forward activation — drop-in for vllm-factory's kernels/ff_fused.py
(`fused_gelu_mul_dropout`, :86-125), used by models/mt5/mt5_encoder.py:418.

    out = act(gate) * up     (activation and product in fp32, result in the input dtype)

The work runs in the sm_100a kernel of libvf_b200.so (vectorised, read-only loads, one
pass over HBM); there is no Triton and no CPU path.  Operands may be strided views (for
example the two halves of one stacked projection): only the last dimension needs unit
stride.
"""
from __future__ import annotations

import torch

import vf_b200.ops  # noqa: F401  (loads the kernels and registers torch.ops.vf_b200)


def _act_type_map(act_fn: str) -> int:
    """The reference's activation names (:77-85): 0 GELU (tanh), 1 GELU (erf), 2 ReLU,
    3 SiLU; unknown names fall back to GELU (tanh) as there."""
    m = {
        'gelu': 0, 'gelu_new': 0, 'gelu_fast': 0, 'gelu_pytorch_tanh': 0,
        'gelu_accurate': 1,
        'relu': 2,
        'silu': 3, 'swish': 3,
    }
    return m.get(act_fn.lower(), 0)


def fused_gelu_mul_dropout(
    gate: torch.Tensor,
    up: torch.Tensor,
    act_fn: str = 'gelu',
    dropout_p: float = 0.0,
    training: bool = False,
) -> torch.Tensor:
    """Same arguments and result as the reference.  Dropout belongs to training, which this
    inference path does not provide: `training=True` with `dropout_p > 0` raises."""
    if training and dropout_p > 0.0:
        raise NotImplementedError("vf_b200: fused_gelu_mul_dropout supports the inference path only (no dropout)")
    assert gate.shape == up.shape, "gate and up must have identical shapes"
    return torch.ops.vf_b200.gated_act(gate, up, _act_type_map(act_fn))


__all__ = ["fused_gelu_mul_dropout"]
