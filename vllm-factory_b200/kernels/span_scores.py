"""GLiNER span scores on the B200: the span-representation MLP and the class einsum of
vllm-factory's poolers/gliner.py (SpanMarkerV0.forward :133-140, GLiNERSpanPooler.forward
:285-289; the same marker in poolers/gliner2.py:230-259) as one sm_100a kernel launch for
every sentence of a batch.

The reference evaluates out_project = Linear(2D, 4D) -> ReLU -> Linear(4D, D) on each of the
L x max_width spans of a sentence and then contracts with the class embeddings pe.  Its first
Linear acts on relu(cat(start, end)), so it splits into two products per WORD, and its second
Linear folds into the CLASS side:
    U = relu(start_rep) W1a^T + b1,   V = relu(end_rep) W1b^T,   P = pe W2,   pb = pe . b2
    score[s, c] = pb[c] + sum_k relu(U[i_s, k] + V[j_s, k]) P[c, k]
Here U, V, P, pb are torch GEMMs over words and classes (not spans), and the per-span sum runs
in `torch.ops.vf_b200.span_scores` (csrc/vf_span.cu: the A operand relu(U[i] + V[j]) is built
in shared memory and multiplied by TMA-staged class rows on tcgen05).  For D = 1024 and 12
widths this removes ~24 D^2 FLOPs per span (the reference's out_project) in favour of 8 D per
span and class.  There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import sys
from typing import List, Optional, Sequence, Tuple

import torch
from torch import nn

import vf_b200.ops  # noqa: F401  (loads the kernels and registers torch.ops.vf_b200)


def _marker_linears(marker: nn.Module) -> Tuple[nn.Linear, nn.Linear]:
    """The two Linear layers of the marker's out_project (Linear, ReLU, [Dropout], Linear)."""
    lins = [m for m in marker.out_project if isinstance(m, nn.Linear)]
    acts = [m for m in marker.out_project if isinstance(m, nn.ReLU)]
    if len(lins) != 2 or len(acts) != 1 or not isinstance(marker.out_project[0], nn.Linear):
        raise ValueError("span scores: out_project must be Linear -> ReLU -> (Dropout) -> Linear")
    return lins[0], lins[1]


def _kernel_dtype(t: torch.Tensor) -> torch.Tensor:
    # The tensor cores take 16-bit operands: fp32 activations go in as fp16 (10-bit mantissa).
    return t if t.dtype in (torch.bfloat16, torch.float16) else t.clamp(-65504.0, 65504.0).to(torch.float16)


def span_factors(marker: nn.Module, words: torch.Tensor, classes: torch.Tensor):
    """Per-word and per-class factors (U, V, P, pb) of a SpanMarkerV0-like module: words
    [W, D], classes [C, D] -> U, V [W, 4D], P [C, 4D] (16-bit), pb [C] (fp32)."""
    if marker.training:
        raise ValueError("span scores: the marker must be in eval mode (dropout is not applied)")
    lin1, lin2 = _marker_linears(marker)
    D = words.shape[-1]
    start_rep = marker.project_start(words)
    end_rep = marker.project_end(words)
    w1 = lin1.weight
    b1 = lin1.bias if lin1.bias is not None else torch.zeros(w1.shape[0], dtype=w1.dtype, device=w1.device)
    U = torch.addmm(b1, torch.relu(start_rep), w1[:, :D].t())
    V = torch.relu(end_rep) @ w1[:, D:].t()
    P = classes.to(lin2.weight.dtype) @ lin2.weight
    pb = (classes.float() @ lin2.bias.float()) if lin2.bias is not None else None
    dt = _kernel_dtype(U).dtype
    return U.to(dt), V.to(dt), P.to(dt), pb


def span_scores_packed(marker: nn.Module, words: torch.Tensor, span_idx: torch.Tensor, classes: torch.Tensor,
                       word_offsets: Sequence[int], span_offsets: Sequence[int], class_offsets: Sequence[int],
                       out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Scores of a packed batch of sentences in one kernel launch.  Sentence g owns rows
    [word_offsets[g], word_offsets[g+1]) of words [W, D], rows [span_offsets[g],
    span_offsets[g+1]) of span_idx [S, 2] (word indices local to the sentence, clamped to
    [0, W_g - 1] like the reference's extract_elements) and rows [class_offsets[g],
    class_offsets[g+1]) of classes [C, D].  Returns the flat scores: sentence g's
    [S_g, C_g] block (span-major) after the previous sentences' blocks, in out_dtype
    (default: words.dtype)."""
    if words.device.type != "cuda":
        raise RuntimeError("span scores: tensors must be on a CUDA device (no CPU implementation)")
    if span_idx.dtype not in (torch.int64, torch.int32):
        span_idx = span_idx.long()
    U, V, P, pb = span_factors(marker, words, classes)
    return torch.ops.vf_b200.span_scores(U, V, span_idx, P, pb, [int(x) for x in word_offsets],
                                         [int(x) for x in span_offsets], [int(x) for x in class_offsets],
                                         out_dtype or words.dtype)


def span_scores_segments(marker: nn.Module, words: Sequence[torch.Tensor], span_idx: Sequence[torch.Tensor],
                         classes: Sequence[torch.Tensor], out_dtype: Optional[torch.dtype] = None
                         ) -> List[torch.Tensor]:
    """Scores of several sentences in one kernel launch.  Sentence g: word states
    words[g] [W_g, D], spans span_idx[g] [S_g, 2], class embeddings classes[g] [C_g, D].
    Returns [S_g, C_g] per sentence, equal to (marker(words[g][None], span_idx[g][None])[0]
    reshaped to [S_g, D]) @ classes[g].T."""
    G = len(words)
    if not (len(span_idx) == len(classes) == G):
        raise ValueError("span scores: words, span_idx and classes must have one entry per sentence")
    if G == 0:
        return []
    if words[0].device.type != "cuda":
        raise RuntimeError("span scores: tensors must be on a CUDA device (no CPU implementation)")
    w2 = [w.reshape(-1, w.shape[-1]) for w in words]
    s2 = [s.reshape(-1, 2) for s in span_idx]
    c2 = [c.reshape(-1, c.shape[-1]) for c in classes]

    def offsets(parts):
        o = [0]
        for p in parts:
            o.append(o[-1] + p.shape[0])
        return o

    wo, so, co = offsets(w2), offsets(s2), offsets(c2)
    flat = span_scores_packed(marker, torch.cat(w2, 0), torch.cat(s2, 0), torch.cat(c2, 0), wo, so, co,
                              out_dtype or words[0].dtype)
    res, at = [], 0
    for g in range(G):
        S, C = so[g + 1] - so[g], co[g + 1] - co[g]
        res.append(flat[at:at + S * C].view(S, C))
        at += S * C
    return res


def fused_span_scores(marker: nn.Module, h: torch.Tensor, span_idx: torch.Tensor, pe: torch.Tensor) -> torch.Tensor:
    """torch.einsum("BLKD,BCD->BLKC", marker(h, span_idx), pe) in one launch: h [B, L, D],
    span_idx [B, L * max_width, 2], pe [B, C, D] -> [B, L, max_width, C] in h's dtype.
    (GLiNERSpanPooler squeezes B = 1; GLiNER2 contracts the same span_rep with its fields.)"""
    B, L, _ = h.shape
    K = span_idx.shape[1] // L if L > 0 else 0
    outs = span_scores_segments(marker, [h[b] for b in range(B)], [span_idx[b] for b in range(B)],
                                [pe[b] for b in range(B)], out_dtype=h.dtype)
    return torch.stack([o.view(L, K, o.shape[-1]) for o in outs], 0)


# ---------------------------------------------------------------- GLiNERSpanPooler drop-in
def _empty_logits(pooler, dev) -> torch.Tensor:
    return torch.zeros((1, pooler.max_width, 1), device=dev, dtype=torch.float32)


def _span_job(pooler, tok: torch.Tensor, add: dict, prompt_ids):
    """One request's inputs to the span scorer, prepared with the reference pooler's own helpers
    in the order of poolers/gliner.py:225-284: (word states [W, D], masked spans [S, 2], raw
    class-token states [1, C, D]) or None when the request gets the empty logits."""
    dev = tok.device
    if not add:
        return None
    ids = add.get("input_ids", prompt_ids)
    if ids is None:
        return None
    iid = pooler._to_tensor(ids, device=dev, dtype=torch.long)
    wmask = pooler._to_tensor(add["words_mask"], device=dev, dtype=torch.long)
    true_len = int(add["text_lengths"])
    attn = add.get("attention_mask", None)
    if attn is not None:
        attn = pooler._to_tensor(attn, device=dev, dtype=torch.long)
    pe_raw, _pe_mask, we_raw, we_mask = pooler._extract_gliner_reps(tok, iid, attn, true_len, wmask)
    we = pooler.rnn(we_raw, we_mask) if pooler.rnn is not None else we_raw
    given_idx, given_mask = add.get("span_idx", None), add.get("span_mask", None)
    W = pooler.max_width
    if given_idx is not None and given_mask is not None:
        span_idx = pooler._to_tensor(given_idx, device=dev, dtype=torch.long)
        span_mask = pooler._to_tensor(given_mask, device=dev, dtype=torch.long)
        span_idx = span_idx.unsqueeze(0) if span_idx.dim() == 2 else span_idx
        span_mask = span_mask.unsqueeze(0) if span_mask.dim() == 1 else span_mask
    else:
        # Every (start, width) pair of the word block; spans reaching past the text are masked.
        n = we.size(1)
        first = torch.arange(n, device=dev).repeat_interleave(W)
        last = first + torch.arange(W, device=dev).repeat(n)
        span_idx = torch.stack([first, last], dim=-1).unsqueeze(0)
        span_mask = ((first < true_len) & (last < true_len)).unsqueeze(0)
    we, _ = pooler._fit_length(we, we_mask, span_idx.size(1) // W)
    masked = span_idx * span_mask.unsqueeze(-1)
    return we[0], masked[0], pe_raw


def gliner_span_pooler_forward(self, hidden_states: torch.Tensor, ctx) -> list:
    """GLiNERSpanPooler.forward (poolers/gliner.py:194-292) with the scores of every request in
    the batch computed by one span-score launch (the reference runs the marker MLP and the
    einsum per request).  Per-request parsing, LSTM, span enumeration and length fitting use
    the reference pooler's own helpers; outputs are the reference's shape-prefixed tensors."""
    mod = sys.modules[type(self).__module__]
    try:
        sequences = mod.split_hidden_states(hidden_states, ctx.seq_lengths)
    except Exception:
        return [torch.zeros(4, device=hidden_states.device, dtype=hidden_states.dtype)]
    if not ctx.extra_kwargs:
        return [_empty_logits(self, hidden_states.device) for _ in sequences]
    outputs: list = [None] * len(sequences)
    jobs = []
    for i, tok in enumerate(sequences):
        add = ctx.extra_kwargs[i] if i < len(ctx.extra_kwargs) else {}
        prompt_ids = ctx.prompt_token_ids[i] if i < len(ctx.prompt_token_ids) else None
        job = _span_job(self, tok, add, prompt_ids)
        if job is None:
            outputs[i] = _empty_logits(self, tok.device)
        else:
            jobs.append((i, job))
    if jobs:
        W = self.max_width
        pe = [self.prompt_proj(job[2])[0] for _, job in jobs]
        scores = span_scores_segments(self.span_rep, [job[0] for _, job in jobs], [job[1] for _, job in jobs], pe,
                                      out_dtype=jobs[0][1][0].dtype)
        for (i, job), sc in zip(jobs, scores):
            n_words = job[1].shape[0] // W
            outputs[i] = mod.pack_shape_prefixed_tensor([n_words, W, sc.shape[-1]], sc.view(n_words, W, -1))
    return outputs


def install_fused_span_scoring(pooler_cls) -> None:
    """Make the reference's GLiNERSpanPooler (passed in) score spans with this kernel: its
    forward becomes gliner_span_pooler_forward, the original kept as
    _vf_reference_forward.  Idempotent."""
    if getattr(pooler_cls, "_vf_reference_forward", None) is None:
        pooler_cls._vf_reference_forward = pooler_cls.forward
    pooler_cls.forward = gliner_span_pooler_forward


__all__ = ["span_factors", "span_scores_packed", "span_scores_segments", "fused_span_scores", "gliner_span_pooler_forward",
           "install_fused_span_scoring"]
