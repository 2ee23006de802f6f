"""Seeded synthetic workloads of the benchmark configurations and their FLOP counts.

The reference measures on NuNER samples of <= 768 tokens (bench/registry.py:162); that
dataset is not available here, so seeded synthetic inputs with the configurations'
shapes, sizes and value distributions stand in for it:

  C1  DeBERTa-v3-large disentangled layer: B=8, L=512, hidden 1024, 16 x 64 heads,
      position_buckets 256, max_relative_positions 512, share_att_key; hidden ~ N(0,1),
      W ~ N(0, 0.02), biases 0, rel_embeddings [512, 1024] ~ N(0, 0.02) then LayerNorm,
      lengths ~ U[64, 512] (right padding).
  C2  mT5-large RPB layer: B=16, L=768, d_model 1024, 16 x 64 heads, 32 buckets / 128,
      no QK scaling, table [32, 16] ~ N(0, 0.02), lengths ~ U[256, 768].
  C5  long-context DeBERTa sweep: L in {1024, 2048, 4096}, B = 16384 / L, full length.

Attention FLOPs count valid work only: 4*H*D*sum(L_i^2) for QK^T + PV, plus
4*H*D*sum(L_i * P(L_i)) for DeBERTa's two position contractions, P(L) = number of
distinct clamped position indices over r in [-(L-1), L-1].
"""
from __future__ import annotations

import functools
import math

import torch

from . import _lib

HEADS = 16
HEAD_DIM = 64
D_MODEL = 1024


def _gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def _heads(x: torch.Tensor, H: int) -> torch.Tensor:
    B, L, E = x.shape
    return x.view(B, L, H, E // H).permute(0, 2, 1, 3)


@functools.lru_cache(maxsize=64)
def deberta_positions_used(L: int, position_buckets: int = 256, max_relative_positions: int = 512,
                           use_log_bucket: bool = True) -> int:
    """P(L): distinct clamped indices clamp(bucket(r) + S, 0, 2S-1) for |r| < L."""
    if L <= 0:
        return 0
    S = position_buckets if position_buckets > 0 else max_relative_positions
    if use_log_bucket:
        b = _lib.deberta_log_bucket(position_buckets, max_relative_positions, -(L - 1), L - 1)
    else:
        b = list(range(-(L - 1), L))
    return len({min(max(x + S, 0), 2 * S - 1) for x in b})


def core_flops(lengths, H: int = HEADS, D: int = HEAD_DIM) -> float:
    return float(sum(4 * H * D * int(L) * int(L) for L in lengths))


def deberta_pos_flops(lengths, H: int = HEADS, D: int = HEAD_DIM, position_buckets: int = 256,
                      max_relative_positions: int = 512) -> float:
    return float(sum(4 * H * D * int(L) * deberta_positions_used(int(L), position_buckets, max_relative_positions)
                     for L in lengths))


def mt5_attention_inputs(seed: int = 0, device="cuda", B: int = 16, L: int = 768, H: int = HEADS,
                         lengths=None, dtype=torch.bfloat16):
    """C2: q, k, v (B, H, L, 64) contiguous like models/mt5/mt5_encoder.py:249-251, the
    [32, H] bias table and the additive [B, 1, 1, L] mask of :571-576."""
    g = _gen(seed)
    E = H * HEAD_DIM
    if lengths is None:
        lengths = torch.randint(256, L + 1, (B,), generator=g)
    lengths = torch.as_tensor(lengths, dtype=torch.int64)
    hidden = torch.randn(B, L, D_MODEL, generator=g).to(dtype)
    wq, wk, wv = ((torch.randn(E, D_MODEL, generator=g) * 0.02).to(dtype) for _ in range(3))
    table = (torch.randn(32, H, generator=g) * 0.02).to(dtype)
    dev = torch.device(device)
    hidden, wq, wk, wv = hidden.to(dev), wq.to(dev), wk.to(dev), wv.to(dev)
    q = _heads(hidden @ wq.t(), H).contiguous()
    k = _heads(hidden @ wk.t(), H).contiguous()
    v = _heads(hidden @ wv.t(), H).contiguous()
    m = (torch.arange(L)[None, :] < lengths[:, None]).to(dtype)
    mask = ((1.0 - m[:, None, None, :]) * torch.finfo(dtype).min).to(dtype).to(dev)
    return dict(q=q, k=k, v=v, rpb_table=table.to(dev), padding_mask=mask, lengths=lengths,
                num_buckets=32, max_distance=128)


def mt5_varlen_inputs(seed: int = 0, device="cuda", B: int = 16, L: int = 768, H: int = HEADS,
                      lengths=None, dtype=torch.bfloat16):
    """C2 in the packed layout: the valid rows of mt5_attention_inputs (same seed, same
    lengths, same values) back to back as [total, H, 64], with cu_seqlens int32 [B+1]."""
    w = mt5_attention_inputs(seed=seed, device=device, B=B, L=L, H=H, lengths=lengths, dtype=dtype)
    lens = [int(x) for x in w["lengths"].tolist()]

    def pack(x):   # (B, H, L, D) -> (total, H, D)
        return torch.cat([x[b, :, :n].permute(1, 0, 2) for b, n in enumerate(lens)], 0).contiguous()

    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0).tolist()), dtype=torch.int32)
    return dict(q=pack(w["q"]), k=pack(w["k"]), v=pack(w["v"]), rpb_table=w["rpb_table"],
                cu_seqlens=cu.to(w["q"].device), max_seqlen=max(lens), lengths=w["lengths"],
                num_buckets=32, max_distance=128)


def deberta_attention_inputs(seed: int = 0, device="cuda", B: int = 8, L: int = 512, H: int = HEADS,
                             lengths=None, dtype=torch.bfloat16, position_buckets: int = 256,
                             max_relative_positions: int = 512, with_positions: bool = True):
    """C1 (and C5 with lengths = L): the op's inputs as DisentangledSelfAttentionV2._flash_forward
    builds them (models/deberta_v2/deberta_v2_encoder.py:246-322): permuted (B, H, L, D)
    views, pos_key = Q (W_k rel + b_k)^T, pos_query = K (W_q rel + b_q)^T, seq_lengths."""
    g = _gen(seed)
    E = H * HEAD_DIM
    if lengths is None:
        lengths = torch.randint(64, L + 1, (B,), generator=g)
    lengths = torch.as_tensor(lengths, dtype=torch.int64)
    hidden = torch.randn(B, L, D_MODEL, generator=g).to(dtype)
    wq, wk, wv = ((torch.randn(E, D_MODEL, generator=g) * 0.02).to(dtype) for _ in range(3))
    S = position_buckets if position_buckets > 0 else max_relative_positions
    rel = torch.randn(2 * S, D_MODEL, generator=g) * 0.02
    rel = torch.nn.functional.layer_norm(rel, (D_MODEL,), eps=1e-7).to(dtype)
    dev = torch.device(device)
    hidden, wq, wk, wv, rel = (t.to(dev) for t in (hidden, wq, wk, wv, rel))
    q = _heads(hidden @ wq.t(), H)
    k = _heads(hidden @ wk.t(), H)
    v = _heads(hidden @ wv.t(), H)
    out = dict(q=q, k=k, v=v, seq_lengths=lengths.to(torch.int32).to(dev), lengths=lengths,
               sm_scale=1.0 / math.sqrt(HEAD_DIM * 3), position_buckets=position_buckets,
               max_relative_distance=max_relative_positions, use_log_bucket=position_buckets > 0)
    if with_positions:
        kr = _heads((rel @ wk.t()).unsqueeze(0), H)     # (1, H, 2S, D), bias is 0
        qr = _heads((rel @ wq.t()).unsqueeze(0), H)
        out["pos_key"] = torch.matmul(q, kr.transpose(-1, -2))
        out["pos_query"] = torch.matmul(k, qr.transpose(-1, -2))
        out["rel_key"] = kr
        out["rel_query"] = qr
    return out


def deberta_varlen_inputs(seed: int = 0, device="cuda", B: int = 8, L: int = 512, H: int = HEADS,
                          lengths=None, dtype=torch.bfloat16):
    """C1 in the packed layout: the valid rows of deberta_attention_inputs (same seed, same
    values) back to back: q, k, v [total, H, 64], pos_key / pos_query [total, H, 2S], with
    cu_seqlens int32 [B+1]."""
    w = deberta_attention_inputs(seed=seed, device=device, B=B, L=L, H=H, lengths=lengths, dtype=dtype)
    lens = [int(x) for x in w["lengths"].tolist()]

    def pack(x):   # (B, H, L, X) -> (total, H, X)
        return torch.cat([x[b, :, :n].permute(1, 0, 2) for b, n in enumerate(lens)], 0).contiguous()

    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0).tolist()), dtype=torch.int32)
    out = {k: w[k] for k in ("lengths", "sm_scale", "position_buckets", "max_relative_distance", "use_log_bucket")}
    out.update(q=pack(w["q"]), k=pack(w["k"]), v=pack(w["v"]), pos_key=pack(w["pos_key"]),
               pos_query=pack(w["pos_query"]), cu_seqlens=cu.to(w["q"].device), max_seqlen=max(lens),
               rel_key=w["rel_key"], rel_query=w["rel_query"])
    return out


def rank_lengths(kind: str, rank: int):
    """Valid lengths of rank `rank`'s batch in a weak-scaled attention run: every rank gets
    the lengths of rank 0's seeded batch (seed 1000 for C2, 2000 for C1), rotated by the
    rank, so each rank does the same valid work on its own data.  None for rank 0, whose
    batch draws them itself (the seeded single-GPU input)."""
    if rank == 0:
        return None
    if kind == "mt5":
        base = torch.randint(256, 768 + 1, (16,), generator=_gen(1000))
    else:
        base = torch.randint(64, 512 + 1, (8,), generator=_gen(2000))
    return torch.roll(base, shifts=rank)


# ----------------------------------------------------------------------------- GLiNER span head
SPAN_HIDDEN = 1024        # GLiNER-large (DeBERTa-v3-large backbone) hidden size
SPAN_MAX_WIDTH = 12
SPAN_REQUESTS = 64


def gliner_span_marker(seed: int = 6000, device="cuda", D: int = SPAN_HIDDEN, dtype=torch.bfloat16):
    """A SpanMarkerV0-shaped module (poolers/gliner.py:118-140: project_start / project_end
    Linear(D, 4D) -> ReLU -> Dropout -> Linear(4D, D), out_project Linear(2D, 4D) -> ReLU ->
    Dropout -> Linear(4D, D)) with weights and biases ~ N(0, 0.02), eval mode."""
    from torch import nn

    def proj(din, dout):
        return nn.Sequential(nn.Linear(din, 4 * dout), nn.ReLU(), nn.Dropout(0.0), nn.Linear(4 * dout, dout))

    m = nn.Module()
    m.project_start, m.project_end, m.out_project = proj(D, D), proj(D, D), proj(2 * D, D)
    g = _gen(seed)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    return m.to(device=device, dtype=dtype).eval()


def gliner_span_batch(seed: int = 6100, device="cuda", n_req: int = SPAN_REQUESTS, D: int = SPAN_HIDDEN,
                      W: int = SPAN_MAX_WIDTH, dtype=torch.bfloat16):
    """One vLLM batch for the span head: n_req requests with word counts ~ U[32, 384] and
    entity-label counts ~ U[3, 25]; word / class states ~ N(0, 1); every (start, width) span
    with widths < W, spans ending past the text masked to (0, 0) as the pooler masks them.
    Returns packed words [sum W_g, D], span_idx [sum W_g * W, 2] int64, classes [sum C_g, D]
    and the three offset lists."""
    g = _gen(seed)
    n_words = torch.randint(32, 385, (n_req,), generator=g).tolist()
    n_cls = torch.randint(3, 26, (n_req,), generator=g).tolist()
    words = torch.randn(sum(n_words), D, generator=g).to(dtype)
    classes = torch.randn(sum(n_cls), D, generator=g).to(dtype)
    idx = []
    for n in n_words:
        first = torch.arange(n).repeat_interleave(W)
        last = first + torch.arange(W).repeat(n)
        idx.append(torch.stack([first, last], -1) * (last < n).unsqueeze(-1))
    span_idx = torch.cat(idx, 0)
    wo, so, co = [0], [0], [0]
    for n, c in zip(n_words, n_cls):
        wo.append(wo[-1] + n)
        so.append(so[-1] + n * W)
        co.append(co[-1] + c)
    return dict(words=words.to(device), span_idx=span_idx.to(device), classes=classes.to(device),
                word_offsets=wo, span_offsets=so, class_offsets=co, n_words=n_words, n_classes=n_cls)
