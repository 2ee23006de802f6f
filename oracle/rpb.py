"""CPU restatement of the reference's relative-position attention (test infrastructure only).

All functions take and return torch CPU tensors and compute in float32 (attention math
in float64 where noted, to serve as the high-precision reference).  Each cites the
reference lines it restates; see the package docstring for the contract.
"""
from __future__ import annotations

import math
from typing import Optional

import torch


# ---------------------------------------------------------------------------- buckets
def t5_relative_bucket_ref(relative_position: torch.Tensor, bidirectional: bool,
                           num_buckets: int, max_distance: int) -> torch.Tensor:
    """models/mt5/mt5_encoder.py:125-148, step for step in float32 torch ops.

    relative_position = memory_position - context_position (key minus query)."""
    relative_position = relative_position.to(torch.long)
    relative_buckets = torch.zeros_like(relative_position)
    if bidirectional:
        num_buckets //= 2
        relative_buckets = relative_buckets + (relative_position > 0).to(torch.long) * num_buckets
        relative_position = torch.abs(relative_position)
    else:
        relative_position = -torch.min(relative_position, torch.zeros_like(relative_position))
    max_exact = num_buckets // 2
    is_small = relative_position < max_exact
    large = max_exact + (
        torch.log(relative_position.float() / max_exact)
        / torch.log(torch.tensor(max_distance / max_exact))
        * (num_buckets - max_exact)
    ).to(torch.long)
    large = torch.min(large, torch.full_like(large, num_buckets - 1))
    return torch.where(is_small, relative_position, large) + relative_buckets


def deberta_log_bucket_ref(relative_pos: torch.Tensor, bucket_size: int,
                           max_position: int) -> torch.Tensor:
    """models/deberta_v2/deberta_v2_encoder.py:70-89 (make_log_bucket_position), returned
    as long like build_relative_position_v2 (:92-103)."""
    relative_pos = relative_pos.to(torch.long)
    sign = torch.sign(relative_pos)
    mid = bucket_size // 2
    abs_pos = torch.where(
        (relative_pos < mid) & (relative_pos > -mid),
        torch.tensor(mid - 1).type_as(relative_pos),
        torch.abs(relative_pos),
    )
    log_pos = (
        torch.ceil(torch.log(abs_pos / mid) / torch.log(torch.tensor((max_position - 1) / mid)) * (mid - 1))
        + mid
    )
    bucket_pos = torch.where(abs_pos <= mid, relative_pos.type_as(log_pos), log_pos * sign)
    return bucket_pos.to(torch.long)


def deberta_position_index_ref(M: int, N: int, att_span: int, position_buckets: int,
                               max_relative_distance: int, use_log_bucket: bool) -> torch.Tensor:
    """(M, N) gather index clamp(bucket(m - n) + S, 0, 2S-1) of
    kernels/flash_deberta_attention.py:395-422."""
    rel = torch.arange(M)[:, None] - torch.arange(N)[None, :]
    if use_log_bucket and position_buckets > 0 and max_relative_distance > 0:
        bucket = deberta_log_bucket_ref(rel, position_buckets, max_relative_distance)
    else:
        bucket = rel
    return torch.clamp(bucket + att_span, 0, 2 * att_span - 1)


# ---------------------------------------------------------------------------- T5 / mT5
def t5_bias_dense_ref(rpb_table: torch.Tensor, num_buckets: int, max_distance: int,
                      is_decoder: bool, M: int, N: int) -> torch.Tensor:
    """Dense (1, H, M, N) bias: models/mt5/mt5_encoder.py:150-164 with the table given as
    [buckets, heads] (nn.Embedding weight layout), bucket clamped to the table's rows like
    kernels/flash_attention_rpb.py:162."""
    ctx = torch.arange(M)[:, None]
    mem = torch.arange(N)[None, :]
    bucket = t5_relative_bucket_ref(mem - ctx, not is_decoder, num_buckets, max_distance)
    bucket = bucket.clamp(0, rpb_table.shape[0] - 1)
    values = rpb_table.float()[bucket]           # (M, N, H)
    return values.permute(2, 0, 1).unsqueeze(0)  # (1, H, M, N)


def rpb_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      rpb_table: Optional[torch.Tensor], num_buckets: int, max_distance: int,
                      is_decoder: bool, padding_mask: Optional[torch.Tensor] = None,
                      softmax_scale: float = 1.0, dtype=torch.float64) -> torch.Tensor:
    """out = softmax(scale*QK^T + bias + mask) V in `dtype` (default float64).

    Bias + mask are summed into one additive tensor like _make_contiguous_additive_bias
    (models/mt5/mt5_encoder.py:75-110) and applied as SDPA does (:309-316).  With
    is_decoder the kernel's causal mask (kernels/flash_attention_rpb.py:176-178) applies.
    Rows whose every key is masked with a huge negative value become a uniform average,
    as in the reference."""
    B, H, M, _ = q.shape
    N = k.shape[2]
    s = torch.matmul(q.to(dtype), k.to(dtype).transpose(-1, -2)) * softmax_scale
    if rpb_table is not None:
        s = s + t5_bias_dense_ref(rpb_table, num_buckets, max_distance, is_decoder, M, N).to(dtype)
    if padding_mask is not None:
        s = s + padding_mask.to(dtype)
    if is_decoder:
        causal = torch.arange(N)[None, :] > torch.arange(M)[:, None]
        s = s.masked_fill(causal, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, v.to(dtype))


def rpb_attention_varlen_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens,
                             rpb_table: Optional[torch.Tensor], num_buckets: int, max_distance: int,
                             is_decoder: bool, softmax_scale: float = 1.0, dtype=torch.float64,
                             fill: float = float("nan")) -> torch.Tensor:
    """Packed batch: q, k, v [total, H, 64]; sequence s = rows cu_seqlens[s]:cu_seqlens[s+1]
    attends only within itself, i.e. rpb_attention_ref on that sequence alone with no
    padding mask (the per-request call models/mt5/mt5_encoder.py:309-316 makes for one
    unpadded request).  Rows outside every sequence are `fill`."""
    cu = [int(x) for x in torch.as_tensor(cu_seqlens).tolist()]
    out = torch.full(q.shape, fill, dtype=dtype)
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        if b <= a:
            continue
        seq = lambda t: t[a:b].permute(1, 0, 2).unsqueeze(0)     # (1, H, L, 64)
        o = rpb_attention_ref(seq(q), seq(k), seq(v), rpb_table, num_buckets, max_distance, is_decoder,
                              None, softmax_scale, dtype=dtype)
        out[a:b] = o[0].permute(1, 0, 2)
    return out


# ---------------------------------------------------------------------------- DeBERTa
def deberta_attention_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          seq_lengths: Optional[torch.Tensor] = None,
                          pos_key: Optional[torch.Tensor] = None,
                          pos_query: Optional[torch.Tensor] = None,
                          causal: bool = False, sm_scale: Optional[float] = None,
                          position_buckets: int = 0, max_relative_distance: int = 0,
                          use_log_bucket: bool = False, dtype=torch.float64,
                          zero_padded_rows: bool = True) -> torch.Tensor:
    """kernels/flash_deberta_attention.py:375-448 (_pytorch_flash_deberta_fwd) in `dtype`.

    Differences from the fallback, both taken from the Triton kernel the GPU runs:
      * rows m >= seq_len are 0 (:334 zeros_like + masked store :298-299) when
        zero_padded_rows;
      * p2c indexes keys by n (M != N allowed), causal uses P_SEQ = N - M (:274)."""
    B, H, M, D = q.shape
    N = k.shape[2]
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    att_span = position_buckets if position_buckets > 0 else max_relative_distance
    s = torch.matmul(q.to(dtype), k.to(dtype).transpose(-1, -2))
    if pos_key is not None or pos_query is not None:
        idx = deberta_position_index_ref(M, N, att_span, position_buckets,
                                         max_relative_distance, use_log_bucket)
        if pos_key is not None:
            s = s + torch.gather(pos_key.to(dtype), -1, idx.expand(B, H, M, N))
        if pos_query is not None:
            # p2c[m, n] = pos_query[n, idx(m, n)]
            g = torch.gather(pos_query.to(dtype), -1, idx.t().expand(B, H, N, M))
            s = s + g.transpose(-1, -2)
    s = s * sm_scale
    if seq_lengths is not None:
        kmask = torch.arange(N)[None, :] < seq_lengths.to(torch.long)[:, None]
        s = s.masked_fill(~kmask[:, None, None, :], float("-inf"))
    if causal:
        cm = (N - M) + torch.arange(M)[:, None] >= torch.arange(N)[None, :]
        s = s.masked_fill(~cm, float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)
    out = torch.matmul(p, v.to(dtype))
    if zero_padded_rows and seq_lengths is not None:
        rmask = torch.arange(M)[None, :] < seq_lengths.to(torch.long)[:, None]
        out = out * rmask[:, None, :, None].to(dtype)
    return out


def deberta_attention_fused_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                seq_lengths: Optional[torch.Tensor] = None,
                                rel_key: Optional[torch.Tensor] = None,
                                rel_query: Optional[torch.Tensor] = None,
                                causal: bool = False, sm_scale: Optional[float] = None,
                                position_buckets: int = 0, max_relative_distance: int = 0,
                                use_log_bucket: bool = False, dtype=torch.float64) -> torch.Tensor:
    """The fused position mode: the caller's products of
    models/deberta_v2/deberta_v2_encoder.py:279 / :284-286, pos_key = q @ Kr^T and
    pos_query = k @ Qr^T, formed here in `dtype` (not rounded to the input dtype as the
    reference's torch.matmul does), then deberta_attention_ref.  rel_key / rel_query:
    (1, H, 2S, D) or (H, 2S, D)."""
    def prod(x, r):
        if r is None:
            return None
        r = r if r.dim() == 4 else r.unsqueeze(0)
        return torch.matmul(x.to(dtype), r.to(dtype).transpose(-1, -2))
    return deberta_attention_ref(q, k, v, seq_lengths, prod(q, rel_key), prod(k, rel_query), causal, sm_scale,
                                 position_buckets, max_relative_distance, use_log_bucket, dtype=dtype)


def deberta_attention_fused_varlen_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens,
                                       rel_key: Optional[torch.Tensor] = None,
                                       rel_query: Optional[torch.Tensor] = None,
                                       causal: bool = False, sm_scale: Optional[float] = None,
                                       position_buckets: int = 0, max_relative_distance: int = 0,
                                       use_log_bucket: bool = False, dtype=torch.float64,
                                       fill: float = float("nan")) -> torch.Tensor:
    """Packed form of deberta_attention_fused_ref: q, k, v [total, H, D]; each cu_seqlens
    sequence alone; rows outside every sequence are `fill`."""
    cu = [int(x) for x in torch.as_tensor(cu_seqlens).tolist()]
    out = torch.full(q.shape, fill, dtype=dtype)
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        if b <= a:
            continue
        seq = lambda t: t[a:b].permute(1, 0, 2).unsqueeze(0)
        o = deberta_attention_fused_ref(seq(q), seq(k), seq(v), None, rel_key, rel_query, causal, sm_scale,
                                        position_buckets, max_relative_distance, use_log_bucket, dtype=dtype)
        out[a:b] = o[0].permute(1, 0, 2)
    return out


def deberta_attention_varlen_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens,
                                 pos_key: Optional[torch.Tensor] = None,
                                 pos_query: Optional[torch.Tensor] = None,
                                 causal: bool = False, sm_scale: Optional[float] = None,
                                 position_buckets: int = 0, max_relative_distance: int = 0,
                                 use_log_bucket: bool = False, dtype=torch.float64,
                                 fill: float = float("nan")) -> torch.Tensor:
    """Packed batch: q, k, v [total, H, 64], pos_key / pos_query [total, H, 2S]; sequence s =
    rows cu_seqlens[s]:cu_seqlens[s+1] is deberta_attention_ref on that sequence alone
    (every row and key valid: the reference's per-request call, :375-448).  Rows outside
    every sequence are `fill`."""
    cu = [int(x) for x in torch.as_tensor(cu_seqlens).tolist()]
    out = torch.full(q.shape, fill, dtype=dtype)
    for s in range(len(cu) - 1):
        a, b = cu[s], cu[s + 1]
        if b <= a:
            continue
        seq = lambda t: None if t is None else t[a:b].permute(1, 0, 2).unsqueeze(0)   # (1, H, L, .)
        o = deberta_attention_ref(seq(q), seq(k), seq(v), None, seq(pos_key), seq(pos_query), causal, sm_scale,
                                  position_buckets, max_relative_distance, use_log_bucket, dtype=dtype)
        out[a:b] = o[0].permute(1, 0, 2)
    return out


def deberta_layer_ref(hidden: torch.Tensor, attention_mask: torch.Tensor,
                      wq: torch.Tensor, bq: torch.Tensor, wk: torch.Tensor, bk: torch.Tensor,
                      wv: torch.Tensor, bv: torch.Tensor, rel_embeddings: torch.Tensor,
                      num_heads: int, position_buckets: int, max_relative_positions: int,
                      dtype=torch.float32) -> torch.Tensor:
    """DisentangledSelfAttentionV2._pytorch_forward with share_att_key=True and
    pos_att_type = [c2p, p2c] (models/deberta_v2/deberta_v2_encoder.py:332-487).

    hidden (B, L, E); attention_mask (B, L) of 0/1 expanded to the outer-product mask of
    DebertaV2Encoder.get_attention_mask (:776-782); rel_embeddings already LayerNormed
    (:770-774).  Returns the context (B, L, E) before the output projection."""
    B, L, E = hidden.shape
    D = E // num_heads
    hid = hidden.to(dtype)

    def proj(x, w, b):
        return x @ w.to(dtype).t() + b.to(dtype)

    def heads(x):  # (B', L, E) -> (B'*H, L, D)
        return x.view(x.shape[0], x.shape[1], num_heads, D).permute(0, 2, 1, 3).reshape(-1, x.shape[1], D)

    q = heads(proj(hid, wq, bq))
    k = heads(proj(hid, wk, bk))
    v = heads(proj(hid, wv, bv))
    scale_factor = 3
    scale = math.sqrt(D * scale_factor)
    scores = torch.bmm(q, k.transpose(-1, -2) / scale)

    att_span = position_buckets if position_buckets > 0 else max_relative_positions
    rel = rel_embeddings.to(dtype)[0:att_span * 2].unsqueeze(0)
    pos_q = heads(proj(rel, wq, bq)).repeat(B, 1, 1)
    pos_k = heads(proj(rel, wk, bk)).repeat(B, 1, 1)
    rel_idx = torch.arange(L)[:, None] - torch.arange(L)[None, :]
    if position_buckets > 0 and max_relative_positions > 0:
        rel_idx = deberta_log_bucket_ref(rel_idx, position_buckets, max_relative_positions)
    c2p_pos = torch.clamp(rel_idx + att_span, 0, att_span * 2 - 1)
    c2p = torch.gather(torch.bmm(q, pos_k.transpose(-1, -2)), -1, c2p_pos.expand(B * num_heads, L, L))
    p2c_pos = torch.clamp(-rel_idx + att_span, 0, att_span * 2 - 1)
    p2c = torch.gather(torch.bmm(k, pos_q.transpose(-1, -2)), -1,
                       p2c_pos.expand(B * num_heads, L, L)).transpose(-1, -2)
    scores = scores + c2p / scale + p2c / scale
    scores = scores.view(B, num_heads, L, L)
    m = attention_mask.to(dtype)[:, None, None, :]
    full = (m * m.squeeze(-2).unsqueeze(-1)).bool()
    scores = scores.masked_fill(~full, torch.finfo(dtype).min)
    probs = torch.softmax(scores, dim=-1)
    ctx = torch.bmm(probs.view(-1, L, L), v)
    return ctx.view(B, num_heads, L, D).permute(0, 2, 1, 3).reshape(B, L, E)
