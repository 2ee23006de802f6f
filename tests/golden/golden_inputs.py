"""Seeded inputs of the golden cases, shared by make_golden.py and the tests.

Every case is regenerated bit-identically from torch's CPU generator; make_golden.py
stores a SHA-256 of each input so the tests can prove they see the same bytes.  Values
are rounded to bfloat16 (and held as float32) so the GPU kernels and the fp32/fp64
references consume exactly the same numbers.
"""
from __future__ import annotations

import hashlib

import torch

# Bucket sweeps: relative positions r in [-R_SWEEP, R_SWEEP].
R_SWEEP = 8191
DEBERTA_BUCKET_CONFIGS = [(256, 512), (128, 512), (64, 128), (32, 64), (256, 1024)]
T5_BUCKET_CONFIGS = [(32, 128, True), (32, 128, False), (64, 256, True), (16, 64, True)]


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).to(torch.float32)


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def deberta_op_case(name: str):
    """Inputs for kernels/flash_deberta_attention.py's op.  Returns a dict of tensors/ints."""
    if name == "deberta_log":
        B, H, L, pb, mr, log, lens, seed = 2, 2, 160, 64, 128, True, [160, 101], 11
    elif name == "deberta_linear":
        B, H, L, pb, mr, log, lens, seed = 2, 2, 144, 48, 512, False, [144, 70], 12
    else:
        raise KeyError(name)
    g = torch.Generator().manual_seed(seed)
    D = 64
    q = _bf16(torch.randn(B, H, L, D, generator=g))
    k = _bf16(torch.randn(B, H, L, D, generator=g))
    v = _bf16(torch.randn(B, H, L, D, generator=g))
    S = pb
    pos_key = _bf16(torch.randn(B, H, L, 2 * S, generator=g) * 2.0)
    pos_query = _bf16(torch.randn(B, H, L, 2 * S, generator=g) * 2.0)
    seq = torch.tensor(lens, dtype=torch.int32)
    return dict(q=q, k=k, v=v, pos_key=pos_key, pos_query=pos_query, seq_lengths=seq,
                sm_scale=1.0 / (D * 3) ** 0.5, position_buckets=pb, max_relative_distance=mr,
                use_log_bucket=log)


def t5_case(name: str):
    """Inputs for the mT5 attention path (bias table [buckets, heads], additive mask)."""
    if name == "t5_enc":
        B, H, L, nb, md, lens, seed = 2, 2, 192, 32, 128, [192, 77], 21
    elif name == "t5_qmask":
        B, H, L, nb, md, lens, seed = 2, 2, 160, 32, 128, [160, 101], 23
    else:
        raise KeyError(name)
    g = torch.Generator().manual_seed(seed)
    D = 64
    q = _bf16(torch.randn(B, H, L, D, generator=g))
    k = _bf16(torch.randn(B, H, L, D, generator=g))
    v = _bf16(torch.randn(B, H, L, D, generator=g))
    table = _bf16(torch.randn(nb, H, generator=g))
    m = (torch.arange(L)[None, :] < torch.tensor(lens)[:, None]).to(torch.float32)
    # models/mt5/mt5_encoder.py:571-576: (1 - m) * finfo(dtype).min, [B, 1, 1, L]
    mask = (1.0 - m[:, None, None, :]) * torch.finfo(torch.bfloat16).min
    if name == "t5_qmask":
        # A mask that varies over query rows, [B, 1, L, L]: the padding mask plus blocked keys
        # per row and small finite offsets (the reference adds any broadcastable mask,
        # models/mt5/mt5_encoder.py:107-108; its kernel reads it with stride_mask_m).
        blocked = torch.rand(B, 1, L, L, generator=g) < 0.25
        extra = _bf16(torch.randn(B, 1, L, L, generator=g) * 0.5)
        extra = extra.masked_fill(blocked, torch.finfo(torch.bfloat16).min)
        mask = _bf16(torch.maximum(mask.expand(B, 1, L, L) + extra, torch.full((), torch.finfo(torch.bfloat16).min)))
    return dict(q=q, k=k, v=v, table=table, mask=mask, num_buckets=nb, max_distance=md,
                lens=torch.tensor(lens, dtype=torch.int32))


def deberta_layer_case(name: str = "deberta_layer"):
    """Small DeBERTa-v2 attention layer (share_att_key, c2p|p2c) for the layer oracle."""
    B, L, H, D, pb, mr, lens, seed = 2, 96, 2, 64, 32, 64, [96, 57], 31
    E = H * D
    g = torch.Generator().manual_seed(seed)
    hidden = _bf16(torch.randn(B, L, E, generator=g))
    w = {n: _bf16(torch.randn(E, E, generator=g) * 0.02) for n in ("wq", "wk", "wv")}
    b = {n: _bf16(torch.randn(E, generator=g) * 0.02) for n in ("bq", "bk", "bv")}
    rel = torch.randn(2 * pb, E, generator=g) * 0.02
    rel = _bf16(torch.nn.functional.layer_norm(rel, (E,), eps=1e-7))
    mask = (torch.arange(L)[None, :] < torch.tensor(lens)[:, None]).to(torch.int64)
    return dict(hidden=hidden, mask=mask, rel=rel, num_heads=H, position_buckets=pb,
                max_relative_positions=mr, lens=torch.tensor(lens, dtype=torch.int32), **w, **b)


def span_case(name: str = "gliner_span"):
    """Inputs for the GLiNER span marker + class einsum (poolers/gliner.py:118-140, :285-289):
    word states h [1, L, D], the reference's default span enumeration (start i, width w,
    end i + w; spans ending past the sentence masked to (0, 0)), the marker's weights as
    {name: tensor} with nn.Linear's [out, in] layout, and class embeddings pe [1, C, D]."""
    if name == "gliner_span":
        L, D, W, C, true_len, seed = 37, 64, 5, 7, 33, 31
    else:
        raise KeyError(name)
    g = torch.Generator().manual_seed(seed)
    h = _bf16(torch.randn(1, L, D, generator=g))
    w = {}
    for pre, din, dout in (("start", D, D), ("end", D, D), ("out", 2 * D, D)):
        w[f"{pre}_w1"] = _bf16(torch.randn(4 * dout, din, generator=g) * 0.05)
        w[f"{pre}_b1"] = _bf16(torch.randn(4 * dout, generator=g) * 0.05)
        w[f"{pre}_w2"] = _bf16(torch.randn(dout, 4 * dout, generator=g) * 0.05)
        w[f"{pre}_b2"] = _bf16(torch.randn(dout, generator=g) * 0.05)
    pe = _bf16(torch.randn(1, C, D, generator=g))
    starts = torch.arange(L).repeat_interleave(W)
    widths = torch.arange(W).repeat(L)
    idx = torch.stack([starts, starts + widths], dim=-1)
    mask = (idx[:, 0] < true_len) & (idx[:, 1] < true_len)
    span_idx = (idx * mask.unsqueeze(-1)).unsqueeze(0)
    return dict(h=h, weights=w, pe=pe, span_idx=span_idx, max_width=W)


def intermediate_case(name: str = "deberta_intermediate"):
    """Inputs for DebertaV2Intermediate (dense [4E, E] + exact GELU): x [rows, E], weight, bias."""
    if name != "deberta_intermediate":
        raise KeyError(name)
    g = torch.Generator().manual_seed(41)
    E, rows = 64, 50
    x = _bf16(torch.randn(rows, E, generator=g))
    w = _bf16(torch.randn(4 * E, E, generator=g) * 0.1)
    b = _bf16(torch.randn(4 * E, generator=g) * 0.1)
    return dict(x=x, weight=w, bias=b)
