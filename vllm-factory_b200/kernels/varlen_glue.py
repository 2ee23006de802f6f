"""Packed-batch glue between vLLM's flat token batches and the attention drop-ins
(no counterpart module in the reference).

vLLM hands an encoder-only pooling model one flat batch per step: `input_ids [T]` and
`positions [T]`, the requests laid end to end, each request's positions restarting at 0.
The reference plugins handle it in one of two ways:

* pad the requests into a [B, Lmax] batch with a Python loop per request, run the encoder,
  and cut the padding off again (plugins/deberta_gliner/model.py:173-201,
  plugins/deberta_gliner_linker/model.py:170-228), paying attention FLOPs on the padding;
* pass the flat batch as ONE sequence (plugins/deberta_gliner2/model.py:125-139,
  plugins/mt5_gliner/model.py:178-192), so that the requests of one step attend to one
  another.

`packed_batch(positions)` finds the request boundaries once per forward (the rows where
positions == 0, the same test as plugins/deberta_gliner/model.py:175) and, while the
context is open, makes `flash_deberta_attention` and `flash_attention_rpb_final` treat a
flat call — q of shape (1, H, T, 64) with T the batch's token count — as the packed requests
it holds: each request attends only within itself, exactly as if it had been run alone,
and no padding is computed.  Everything the encoders do between attention calls
(projections, norms, FFN, embeddings without absolute positions) is per token and runs on
the flat batch unchanged, so a plugin keeps its flat call and opens the context around it:

    with packed_batch(positions):
        hs = self.encoder(input_ids=input_ids)          # (1, T, E), requests kept apart

Inside the context the request boundaries replace what the flat call says about padding:
a flat batch has none, so its `seq_lengths` (DeBERTa) are T and its padding mask (mT5)
is all zero, and neither is read.

`deberta_v2_flash_forward` is the fused-position form of the reference's
DisentangledSelfAttentionV2._flash_forward (models/deberta_v2/deberta_v2_encoder.py:246-328):
the same inputs and result, but it hands the projected position tables Kr / Qr to the
kernel instead of forming the (B, H, L, 2S) products in HBM.  `install_fused_positions`
puts it on the reference's class.
"""
from __future__ import annotations

import threading
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Optional, Tuple

import torch


@dataclass(frozen=True)
class PackedBatch:
    """Request boundaries of one flat batch: request s is rows cu_seqlens[s]:cu_seqlens[s+1]."""
    cu_seqlens: torch.Tensor     # int32 [S+1] on the batch's device
    max_seqlen: int
    total: int                   # T, the flat batch's token count

    @property
    def num_seqs(self) -> int:
        return self.cu_seqlens.numel() - 1


_state = threading.local()


def cu_seqlens_from_positions(positions: torch.Tensor) -> Tuple[torch.Tensor, int]:
    """cu_seqlens (int32 [S+1], on positions' device) and the longest request of a flat vLLM
    batch whose requests start where positions == 0.  One device-to-host read of the S start
    offsets (the reference reads them with .tolist(), plugins/deberta_gliner/model.py:175).

    Raises ValueError if positions is not 1-D or its first row does not start a request."""
    if positions.dim() != 1:
        raise ValueError(f"cu_seqlens_from_positions: positions must be 1-D, got shape {tuple(positions.shape)}")
    T = positions.numel()
    if T == 0:
        return torch.zeros(1, dtype=torch.int32, device=positions.device), 0
    starts = torch.nonzero(positions == 0).flatten().to(torch.int32)
    cu = torch.empty(starts.numel() + 1, dtype=torch.int32, device=positions.device)
    cu[:-1] = starts
    cu[-1] = T
    host = cu.cpu()
    if host.numel() < 2 or int(host[0]) != 0:
        raise ValueError("cu_seqlens_from_positions: the first token does not start a request (positions[0] != 0)")
    return cu, int((host[1:] - host[:-1]).max())


@contextmanager
def packed_batch(positions: Optional[torch.Tensor] = None, *, cu_seqlens: Optional[torch.Tensor] = None,
                 max_seqlen: Optional[int] = None):
    """Open a packed-batch context for one flat forward: from vLLM `positions`, or from a
    caller's `cu_seqlens` (int32, on the device) with `max_seqlen`.  Yields the PackedBatch.
    Contexts nest; the innermost one is active.  A batch of one request needs no context
    (the flat call is then already right) but may use one."""
    if (positions is None) == (cu_seqlens is None):
        raise ValueError("packed_batch: pass positions or cu_seqlens (with max_seqlen), not both")
    if positions is not None:
        cu, mx = cu_seqlens_from_positions(positions)
    else:
        if max_seqlen is None:
            raise ValueError("packed_batch: cu_seqlens needs max_seqlen")
        if cu_seqlens.dtype != torch.int32 or cu_seqlens.dim() != 1 or cu_seqlens.numel() < 1:
            raise ValueError("packed_batch: cu_seqlens must be a 1-D int32 tensor")
        cu, mx = cu_seqlens, int(max_seqlen)
    batch = PackedBatch(cu, mx, int(cu[-1].item()) if positions is None else positions.numel())
    stack = getattr(_state, "stack", None)
    if stack is None:
        stack = _state.stack = []
    stack.append(batch)
    try:
        yield batch
    finally:
        stack.pop()


def current() -> Optional[PackedBatch]:
    """The innermost open packed batch of this thread, or None."""
    stack = getattr(_state, "stack", None)
    return stack[-1] if stack else None


def routes(q: torch.Tensor) -> Optional[PackedBatch]:
    """The open packed batch if `q` (B, H, M, D) is a flat call over it (B == 1, M == T) that
    holds more than one request, else None."""
    batch = current()
    if batch is None or q.dim() != 4 or q.size(0) != 1 or q.size(2) != batch.total or batch.num_seqs < 2:
        return None
    return batch


def packed_rows(x: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
    """(1, H, T, C) -> the (T, H, C) view the packed operators take (no copy)."""
    return None if x is None else x[0].transpose(0, 1)


def flat_result(out: torch.Tensor) -> torch.Tensor:
    """(T, H, D) -> the (1, H, T, D) view a flat call returns (no copy)."""
    return out.transpose(0, 1).unsqueeze(0)


def deberta_v2_flash_forward(self, query_layer_out: torch.Tensor, key_layer_out: torch.Tensor,
                             value_layer_out: torch.Tensor, attention_mask: torch.Tensor,
                             rel_embeddings: torch.Tensor) -> torch.Tensor:
    """DisentangledSelfAttentionV2._flash_forward (models/deberta_v2/deberta_v2_encoder.py:246-328)
    with the position products moved into the kernel: Kr = key_proj(rel) and
    Qr = query_proj(rel) (pos_key_proj / pos_query_proj when the key is not shared) go to the
    op as rel_key / rel_query.  Same arguments, scale, buckets, seq_lengths rule and result
    layout as the reference method; a layer without both c2p and p2c terms keeps the
    reference's own method."""
    from kernels.flash_deberta_attention import flash_deberta_attention

    if not ("c2p" in self.pos_att_type and "p2c" in self.pos_att_type):
        return self._vf_reference_flash_forward(query_layer_out, key_layer_out, value_layer_out,
                                                attention_mask, rel_embeddings)
    query_layer = self._transpose_4d(query_layer_out)
    key_layer = self._transpose_4d(key_layer_out)
    value_layer = self._transpose_4d(value_layer_out)

    rel_embeddings = self.pos_dropout(rel_embeddings)
    att_span = self.pos_ebd_size
    rel_emb = rel_embeddings[0:att_span * 2, :].unsqueeze(0)
    sm_scale = 1.0 / (self.attention_head_size * 3) ** 0.5
    key_proj = self.key_proj if self.share_att_key else self.pos_key_proj
    query_proj = self.query_proj if self.share_att_key else self.pos_query_proj
    rel_key = self._transpose_4d(key_proj(rel_emb)[0])
    rel_query = self._transpose_4d(query_proj(rel_emb)[0]).to(dtype=key_layer.dtype)

    M = query_layer.size(2)
    if attention_mask.dim() == 4:
        seq_lengths = attention_mask[:, 0, 0, :].sum(dim=-1).int()
    elif attention_mask.dim() == 2:
        seq_lengths = attention_mask.sum(dim=-1).int()
    else:
        seq_lengths = torch.full((query_layer.size(0),), M, dtype=torch.int32, device=query_layer.device)

    context_layer = flash_deberta_attention(
        q=query_layer, k=key_layer, v=value_layer, seq_lengths=seq_lengths, causal=False, sm_scale=sm_scale,
        position_buckets=self.position_buckets if self.position_buckets > 0 else att_span,
        max_relative_distance=self.max_relative_positions, use_log_bucket=(self.position_buckets > 0),
        rel_key=rel_key, rel_query=rel_query)
    context_layer = context_layer.permute(0, 2, 1, 3).contiguous()
    return context_layer.view(context_layer.size()[:-2] + (-1,))


def install_fused_positions(attention_cls) -> None:
    """Make the reference's DisentangledSelfAttentionV2 (passed in) use the fused position mode:
    its _flash_forward becomes deberta_v2_flash_forward, the original kept as
    _vf_reference_flash_forward.  Idempotent."""
    if getattr(attention_cls, "_vf_reference_flash_forward", None) is None:
        attention_cls._vf_reference_flash_forward = attention_cls._flash_forward
    attention_cls._flash_forward = deberta_v2_flash_forward


__all__ = ["PackedBatch", "cu_seqlens_from_positions", "packed_batch", "current", "deberta_v2_flash_forward",
           "install_fused_positions"]
