"""Comparison helpers for the parity tests (north-star gates: max-abs <= 2e-2 and per-row
cosine >= 0.9999 against the fp32/fp64 oracle, valid rows only)."""
from __future__ import annotations

import torch

MAX_ABS = 2e-2
MIN_COS = 0.9999


def row_stats(out: torch.Tensor, ref: torch.Tensor, row_mask: torch.Tensor | None = None):
    """Max abs error and minimum per-row cosine over rows selected by row_mask (B, M)."""
    o = out.detach().float().cpu()
    r = ref.detach().float().cpu()
    if row_mask is not None:
        sel = row_mask[:, None, :].expand(o.shape[0], o.shape[1], o.shape[2])
        o = o[sel]
        r = r[sel]
    else:
        o = o.reshape(-1, o.shape[-1])
        r = r.reshape(-1, r.shape[-1])
    if o.numel() == 0:
        return 0.0, 1.0
    err = (o - r).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(o.double(), r.double(), dim=-1, eps=1e-30)
    # rows that are exactly zero in both count as matching
    both_zero = (o.abs().sum(-1) == 0) & (r.abs().sum(-1) == 0)
    cos = torch.where(both_zero, torch.ones_like(cos), cos)
    return err, cos.min().item()


def assert_close(out, ref, row_mask=None, max_abs=MAX_ABS, min_cos=MIN_COS, what=""):
    err, cos = row_stats(out, ref, row_mask)
    assert err <= max_abs and cos >= min_cos, f"{what}: max_abs={err:.3e} (<= {max_abs}) min_cos={cos:.6f} (>= {min_cos})"
    return err, cos


def lens_mask(lens, M):
    lens = torch.as_tensor(lens).to(torch.long).cpu()
    return torch.arange(M)[None, :] < lens[:, None]
