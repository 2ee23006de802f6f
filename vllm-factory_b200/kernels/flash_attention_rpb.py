"""T5 relative-position-bias flash attention — drop-in for vllm-factory's
kernels/flash_attention_rpb.py (`flash_attention_rpb_final`, :296-412).

Computes, per (batch b, head h, query m):
    s[n]   = softmax_scale * q[m]·k[n] + rpb_table[bucket(n - m), h] + padding_mask[b, h, m, n]
    out[m] = softmax(s) @ v
with the T5 bucket of models/mt5/mt5_encoder.py:125-148 (bidirectional unless
`is_decoder`, which also applies a causal mask), clamped to the table's rows.
The work runs in the sm_100a kernel of libvf_b200.so (tcgen05 UMMA, TMEM accumulators,
TMA-staged K/V); there is no Triton and no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch

import vf_b200.ops  # noqa: F401  (loads the kernels and registers torch.ops.vf_b200)

from . import varlen_glue


def flash_attention_rpb_final(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    rpb_table: Optional[torch.Tensor],
    num_buckets: int,
    max_distance: int,
    is_decoder: bool,
    padding_mask: Optional[torch.Tensor] = None,
    dropout_p: float = 0.0,
    softmax_scale: float = 1.0,
    use_autotune: bool = True,
) -> torch.Tensor:
    """Same arguments and result as the reference.  `use_autotune` is accepted and ignored:
    the kernel has a single tile configuration.  `dropout_p` must be 0 (inference path;
    the reference's callers always pass 0).  Inside `varlen_glue.packed_batch`, a flat call
    (q of shape (1, H, T, 64) over the batch's T tokens) runs as the batch's requests, each
    attending only within itself; the flat call's padding mask (all zero) is not read."""
    del use_autotune
    batch = varlen_glue.routes(q)
    if batch is not None:
        if dropout_p != 0.0:
            raise ValueError("flash_attention_rpb_final: dropout_p must be 0 (inference path)")
        rows = varlen_glue.packed_rows
        return varlen_glue.flat_result(flash_attention_rpb_varlen(
            rows(q), rows(k), rows(v), batch.cu_seqlens, batch.max_seqlen, rpb_table, num_buckets, max_distance,
            is_decoder, softmax_scale))
    return torch.ops.vf_b200.rpb_attention(
        q, k, v, rpb_table, int(num_buckets), int(max_distance), bool(is_decoder),
        padding_mask, float(dropout_p), float(softmax_scale))


def flash_attention_rpb_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    rpb_table: Optional[torch.Tensor],
    num_buckets: int,
    max_distance: int,
    is_decoder: bool = False,
    softmax_scale: float = 1.0,
) -> torch.Tensor:
    """Packed variable-length form (no counterpart in the reference).

    q, k, v: [total, heads, 64], sequence s in rows cu_seqlens[s]:cu_seqlens[s+1]
    (int32, on the device).  Each sequence attends only within itself, as if it had been
    padded and passed to `flash_attention_rpb_final` alone with no padding mask; no
    padding FLOPs are spent.  `max_seqlen` must bound every sequence length.  Returns
    [total, heads, 64]; rows outside every sequence are left unwritten."""
    return torch.ops.vf_b200.rpb_attention_varlen(
        q, k, v, cu_seqlens, int(max_seqlen), rpb_table, int(num_buckets), int(max_distance),
        bool(is_decoder), float(softmax_scale))


__all__ = ["flash_attention_rpb_final", "flash_attention_rpb_varlen"]
