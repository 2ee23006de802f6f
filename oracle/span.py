"""CPU restatement of the reference's GLiNER span scoring (test infrastructure only).

poolers/gliner.py (the same marker is poolers/gliner2.py:230-259):
  * create_projection_layer (:26-37): Linear(d, 4 o) -> ReLU -> Dropout -> Linear(4 o, o);
    dropout is the identity in eval mode
  * extract_elements (:40-45): gather of rows with indices clamped to [0, L - 1]
  * SpanMarkerV0.forward (:133-140): start / end projections, gathers, cat, relu,
    out_project, view [B, L, max_width, D]
  * GLiNERSpanPooler.forward (:285-289): einsum("BLKD,BCD->BLKC", span_rep, pe).squeeze(0)
span_scores_ref keeps the reference's order of operations (float64 by default).
span_scores_factored_ref is the factored form the GPU kernel evaluates,
    pb[c] + sum_k relu(U[i, k] + V[j, k]) P[c, k],
    U = relu(start_rep) W1a^T + b1,  V = relu(end_rep) W1b^T,  P = pe W2,  pb = pe . b2,
equal to span_scores_ref in exact arithmetic; the tests check the two against each other.
Weights are a dict with nn.Linear's [out, in] layout: {start,end,out}_{w1,b1,w2,b2}.
"""
from __future__ import annotations

import torch


def _mlp(x, w, pre):
    return torch.relu(x @ w[f"{pre}_w1"].T + w[f"{pre}_b1"]) @ w[f"{pre}_w2"].T + w[f"{pre}_b2"]


def _cast(w, dtype):
    return {k: v.to(dtype) for k, v in w.items()}


def span_rep_ref(h: torch.Tensor, span_idx: torch.Tensor, weights: dict, max_width: int,
                 dtype=torch.float64) -> torch.Tensor:
    """SpanMarkerV0.forward: h [B, L, D], span_idx [B, S, 2] -> [B, L, max_width, D]."""
    w = _cast(weights, dtype)
    h = h.to(dtype)
    B, L, D = h.shape
    start_rep = _mlp(h, w, "start")
    end_rep = _mlp(h, w, "end")
    idx = span_idx.clamp(0, L - 1)

    def gather(t, col):
        return t.gather(1, idx[:, :, col].unsqueeze(-1).expand(B, idx.shape[1], D))

    cat = torch.cat([gather(start_rep, 0), gather(end_rep, 1)], dim=-1).relu()
    return _mlp(cat, w, "out").view(B, L, max_width, D)


def span_scores_ref(h, span_idx, weights, pe, max_width, dtype=torch.float64) -> torch.Tensor:
    """einsum("BLKD,BCD->BLKC", SpanMarkerV0(h, span_idx), pe).squeeze(0) -> [L, K, C]."""
    rep = span_rep_ref(h, span_idx, weights, max_width, dtype)
    return torch.einsum("BLKD,BCD->BLKC", rep, pe.to(dtype)).squeeze(0)


def span_factors_ref(h, weights, pe, dtype=torch.float64):
    """Per-word and per-class factors of the factored form: (U, V, P, pb) for one sentence
    (h [1, L, D] or [L, D], pe [1, C, D] or [C, D])."""
    w = _cast(weights, dtype)
    h2 = h.reshape(-1, h.shape[-1]).to(dtype)
    D = h2.shape[-1]
    start_rep = _mlp(h2, w, "start")
    end_rep = _mlp(h2, w, "end")
    w1 = w["out_w1"]
    U = start_rep.relu() @ w1[:, :D].T + w["out_b1"]
    V = end_rep.relu() @ w1[:, D:].T
    pe2 = pe.reshape(-1, pe.shape[-1]).to(dtype)
    P = pe2 @ w["out_w2"]
    pb = pe2 @ w["out_b2"]
    return U, V, P, pb


def span_scores_from_factors_ref(U, V, span_idx, P, pb) -> torch.Tensor:
    """scores[s, c] = pb[c] + sum_k relu(U[i_s, k] + V[j_s, k]) P[c, k], indices clamped to
    [0, words - 1]; span_idx [S, 2] -> [S, C] (float64 arithmetic on the given values)."""
    L = U.shape[0]
    idx = span_idx.reshape(-1, 2).clamp(0, L - 1)
    Ud, Vd, Pd = U.double(), V.double(), P.double()
    h1 = (Ud[idx[:, 0]] + Vd[idx[:, 1]]).relu()
    out = h1 @ Pd.T
    return out + pb.double() if pb is not None else out


def span_scores_factored_ref(h, span_idx, weights, pe, max_width, dtype=torch.float64) -> torch.Tensor:
    """The factored form of span_scores_ref -> [L, K, C]."""
    U, V, P, pb = span_factors_ref(h, weights, pe, dtype)
    out = span_scores_from_factors_ref(U, V, span_idx, P, pb)
    return out.view(h.shape[-2], max_width, -1)
