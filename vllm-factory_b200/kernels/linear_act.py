"""Linear + activation with the activation in the GEMM's epilogue — the DeBERTa feed-forward's
first half, models/deberta_v2/deberta_v2_encoder.py:547-550 (DebertaV2Intermediate.forward:
`self.dense(hidden_states)`, then ACT2FN["gelu"], torch's exact GELU), and the mT5 gated
activation (`gated_gelu_tanh`, below).

The reference writes the [tokens, intermediate_size] product to HBM and reads it back for the
activation; `linear_gelu` runs one sm_100a GEMM (csrc/vf_gemm.cu: TMA tile loads, tcgen05 with
a TMEM accumulator) whose epilogue adds the bias and applies 0.5 x (1 + erf(x / sqrt 2)) to the
fp32 accumulator before rounding.  There is no CPU path:
CPU tensors raise.
"""
from __future__ import annotations

from typing import Optional

import torch

import vf_b200.ops  # noqa: F401  (loads the kernels and registers torch.ops.vf_b200)

ACT_GELU_TANH, ACT_GELU_ERF = 0, 1   # VF_ACT_GELU_TANH, VF_ACT_GELU_ERF


def linear_gelu(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """F.gelu(F.linear(x, weight, bias)) (exact GELU) as one GEMM; x [..., K] 16-bit, weight
    [N, K] (nn.Linear layout), bias [N] or None; K and N multiples of 8."""
    return torch.ops.vf_b200.linear_act(x, weight, bias, None, ACT_GELU_ERF)


def gated_gelu_tanh(x: torch.Tensor, gate_weight: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """The mT5 gated feed-forward activation with the gate projection as its GEMM:
    gelu_tanh(x gate_weight^T) * up (the reference's fused_gelu_mul_dropout(wi_0(x), wi_1(x),
    "gelu_new") at models/mt5/mt5_encoder.py:427-437), `up` = wi_1(x) computed by the caller;
    the activation and the product run in the epilogue, so the gate projection never reaches
    HBM.  x [..., K], gate_weight [N, K], up [..., N], one 16-bit dtype."""
    return torch.ops.vf_b200.linear_act(x, gate_weight, None, up, ACT_GELU_TANH)


def _exact_gelu(act_fn) -> bool:
    """Whether an intermediate_act_fn is the exact (erf) GELU that the kernel applies:
    F.gelu, nn.GELU(approximate="none"), or transformers' GELUActivation (ACT2FN["gelu"],
    whose `act` is F.gelu or its erf formula in Python)."""
    import torch.nn.functional as F
    if act_fn is F.gelu:
        return True
    if isinstance(act_fn, torch.nn.GELU):
        return act_fn.approximate == "none"
    if type(act_fn).__name__ == "GELUActivation":
        inner = getattr(act_fn, "act", None)
        return inner is F.gelu or getattr(inner, "__name__", "") == "_gelu_python"
    return False


def deberta_intermediate_forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
    """DebertaV2Intermediate.forward with the GEMM and the exact GELU as one kernel.  Modules
    whose activation is not the exact GELU, whose dense layer is sharded (tensor parallel) or
    whose activations are fp32 keep the reference's own forward (`_vf_reference_forward`) on
    the GPU; CPU tensors raise."""
    if not hidden_states.is_cuda:
        raise RuntimeError("deberta_intermediate_forward: hidden_states must be a CUDA tensor (no CPU implementation)")
    dense = self.dense
    if not _exact_gelu(self.intermediate_act_fn) or getattr(dense, "tp_size", 1) != 1 or \
            hidden_states.dtype not in (torch.bfloat16, torch.float16):
        return type(self)._vf_reference_forward(self, hidden_states)
    return linear_gelu(hidden_states, dense.weight, dense.bias)


def install_fused_intermediate(intermediate_cls) -> None:
    """Make the reference's DebertaV2Intermediate (passed in) run its dense layer and exact GELU
    as one GEMM: forward becomes deberta_intermediate_forward, the original kept as
    _vf_reference_forward.  Idempotent."""
    if getattr(intermediate_cls, "_vf_reference_forward", None) is None:
        intermediate_cls._vf_reference_forward = intermediate_cls.forward
    intermediate_cls.forward = deberta_intermediate_forward


__all__ = ["linear_gelu", "gated_gelu_tanh", "deberta_intermediate_forward", "install_fused_intermediate"]
