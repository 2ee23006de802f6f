"""DeBERTa disentangled flash attention — drop-in for vllm-factory's
kernels/flash_deberta_attention.py (`flash_deberta_attention`, :455-499).

Computes, per (batch b, head h, query m < seq_len[b]):
    idx    = clamp(bucket(m - n) + S, 0, 2S - 1)          S = position_buckets or max_rel
    s[n]   = sm_scale * (q[m]·k[n] + pos_key[m, idx] + pos_query[n, idx]),  n < seq_len[b]
    out[m] = softmax(s) @ v ;   rows m >= seq_len[b] are 0
with bucket() the log bucket of models/deberta_v2/deberta_v2_encoder.py:70-89 when
`use_log_bucket` (DeBERTa v2/v3) and the identity otherwise (DeBERTa v1).
The work runs in the sm_100a kernel of libvf_b200.so; there is no Triton and no CPU path.

`HAS_TRITON` keeps the reference's export name: the reference's encoders enable their
fused path when it is true (models/deberta_v2/deberta_v2_encoder.py:39-40,
models/deberta/deberta_encoder.py:35-36).  Here it means "the fused GPU op is present".

Fused position mode (keyword-only `rel_key` / `rel_query`, no counterpart in the
reference): instead of the caller's products pos_key = q @ Kr^T and pos_query = k @ Qr^T
(models/deberta_v2/deberta_v2_encoder.py:275-286), pass Kr = key_proj(rel) and
Qr = query_proj(rel) themselves as (1, H, 2S, 64) (or (H, 2S, 64)); the kernel forms both
products on the tensor cores tile by tile and never writes the (B, H, L, 2S) tensors.
`HAS_FUSED_POSITIONS` says the build has that mode.
"""
from __future__ import annotations

from typing import Optional

import torch

import vf_b200.ops  # noqa: F401  (loads the kernels and registers torch.ops.vf_b200)

from . import varlen_glue

HAS_TRITON = True
HAS_FUSED_POSITIONS = True


def _fused_args(pos_key, pos_query, rel_key, rel_query):
    if rel_key is None and rel_query is None:
        return False
    if pos_key is not None or pos_query is not None:
        raise ValueError("flash_deberta_attention: pass either pos_key / pos_query (their products) or "
                         "rel_key / rel_query (the projected tables), not both")
    return True


def flash_deberta_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    seq_lengths: Optional[torch.Tensor] = None,
    pos_key: Optional[torch.Tensor] = None,
    pos_query: Optional[torch.Tensor] = None,
    causal: bool = False,
    sm_scale: Optional[float] = None,
    position_buckets: int = 0,
    max_relative_distance: int = 0,
    use_log_bucket: bool = False,
    *,
    rel_key: Optional[torch.Tensor] = None,
    rel_query: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Same arguments and result as the reference (output rows past seq_len are zero).
    With `rel_key` / `rel_query` the position products are formed inside the kernel.
    Inside `varlen_glue.packed_batch`, a flat call (q of shape (1, H, T, 64) over the
    batch's T tokens) runs as the batch's requests, each attending only within itself."""
    batch = varlen_glue.routes(q)
    if batch is not None:
        rows = varlen_glue.packed_rows
        return varlen_glue.flat_result(flash_deberta_attention_varlen(
            rows(q), rows(k), rows(v), batch.cu_seqlens, batch.max_seqlen, rows(pos_key), rows(pos_query),
            causal, sm_scale, position_buckets, max_relative_distance, use_log_bucket,
            rel_key=rel_key, rel_query=rel_query))
    if _fused_args(pos_key, pos_query, rel_key, rel_query):
        return torch.ops.vf_b200.deberta_attention_fused(
            q, k, v, seq_lengths, rel_key, rel_query, bool(causal),
            None if sm_scale is None else float(sm_scale),
            int(position_buckets), int(max_relative_distance), bool(use_log_bucket))
    return torch.ops.vf_b200.deberta_attention(
        q, k, v, seq_lengths, pos_key, pos_query, bool(causal),
        None if sm_scale is None else float(sm_scale),
        int(position_buckets), int(max_relative_distance), bool(use_log_bucket))


def flash_deberta_attention_varlen(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    pos_key: Optional[torch.Tensor] = None,
    pos_query: Optional[torch.Tensor] = None,
    causal: bool = False,
    sm_scale: Optional[float] = None,
    position_buckets: int = 0,
    max_relative_distance: int = 0,
    use_log_bucket: bool = False,
    *,
    rel_key: Optional[torch.Tensor] = None,
    rel_query: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Packed variable-length form (no counterpart in the reference).

    q, k, v: [total, heads, 64]; pos_key / pos_query: [total, heads, 2S] (the per-row
    position scores of the packed rows) or None.  Sequence s is rows
    cu_seqlens[s]:cu_seqlens[s+1] (int32, on the device) and attends only within itself,
    as if it had been passed alone to `flash_deberta_attention` with seq_lengths = its
    length.  `max_seqlen` must bound every sequence length.  Returns [total, heads, 64];
    rows outside every sequence are left unwritten.  `rel_key` / `rel_query`: the fused
    position mode, as for `flash_deberta_attention`."""
    if _fused_args(pos_key, pos_query, rel_key, rel_query):
        return torch.ops.vf_b200.deberta_attention_fused_varlen(
            q, k, v, cu_seqlens, int(max_seqlen), rel_key, rel_query, bool(causal),
            None if sm_scale is None else float(sm_scale),
            int(position_buckets), int(max_relative_distance), bool(use_log_bucket))
    return torch.ops.vf_b200.deberta_attention_varlen(
        q, k, v, cu_seqlens, int(max_seqlen), pos_key, pos_query, bool(causal),
        None if sm_scale is None else float(sm_scale),
        int(position_buckets), int(max_relative_distance), bool(use_log_bucket))


def clear_config_cache() -> None:
    """Reference API (kernels/flash_deberta_attention.py:502).  The reference cached Triton
    tile configurations; this implementation has a single configuration, so there is
    nothing to clear."""


__all__ = ["flash_deberta_attention", "flash_deberta_attention_varlen", "clear_config_cache", "HAS_TRITON",
           "HAS_FUSED_POSITIONS"]
