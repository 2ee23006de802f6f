"""Runs the reference's own GLiNERSpanPooler (poolers/gliner.py) with and without this
repository's span-score kernel installed on its class (kernels/span_scores.py
`install_fused_span_scoring`).

A pooler with seeded random weights (hidden 768, max_width 12, the LSTM on) scores one vLLM
batch of four requests: two with class tokens and words (one with multi-token words), one with
no extra kwargs (the empty-logits path) and one with caller-given span_idx / span_mask.  Three
runs on the same weights and inputs:

  fused       the bf16 pooler with the kernel installed (one span-score launch for the batch);
  torch_bf16  the same bf16 pooler, the reference's forward as shipped;
  torch_fp32  an fp32 copy of the pooler (bf16 weights upcast), the reference's forward.

Prints one JSON line (RESULT {...}): per request, whether the shape prefixes of fused and
torch_bf16 equal torch_fp32's, and the max-abs difference / minimum per-span cosine / score
scale of fused and torch_bf16 against torch_fp32.

    python tests/reference_pooler_run.py --reference <reference install>
"""
import argparse
import copy
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _paths(reference):
    # This repository's package directory first (its `kernels` package), the reference after
    # it (`poolers`, `vllm_factory`).
    for p in (ROOT / "vllm-factory_b200", ROOT):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    sys.path.append(str(reference))


def _requests(torch, gen, ent):
    """(token ids, words_mask, text_lengths, extra) per request; extra holds optional span_idx
    / span_mask.  Class tokens come first ([ENT] label ...), then the words."""
    reqs = []

    def build(n_cls, n_words, multi):
        ids, wmask = [1], [0]
        for _ in range(n_cls):
            ids += [ent, int(torch.randint(1000, 2000, (1,), generator=gen))]
            wmask += [0, 0]
        ids.append(2)
        wmask.append(0)
        for w in range(n_words):
            pieces = 2 if (multi and w % 3 == 0) else 1
            for _ in range(pieces):
                ids.append(int(torch.randint(3000, 9000, (1,), generator=gen)))
                wmask.append(w + 1)
        ids.append(2)
        wmask.append(0)
        return ids, wmask

    ids, wm = build(3, 20, False)
    reqs.append((ids, {"input_ids": ids, "words_mask": wm, "text_lengths": 20}))
    ids, wm = build(7, 45, True)
    reqs.append((ids, {"input_ids": ids, "words_mask": wm, "text_lengths": 45}))
    ids, _ = build(2, 9, False)
    reqs.append((ids, {}))
    ids, wm = build(5, 12, False)
    W = 12
    first = torch.arange(12).repeat_interleave(W)
    last = first + torch.arange(W).repeat(12)
    mask = (last < 12).long()
    reqs.append((ids, {"input_ids": ids, "words_mask": wm, "text_lengths": 12,
                       "span_idx": torch.stack([first, last], -1).tolist(), "span_mask": mask.tolist()}))
    return reqs


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    _paths(args.reference)
    import torch
    import poolers.gliner as ref_mod
    from vllm_factory.pooling.protocol import PoolerContext
    from kernels import span_scores

    dev = torch.device("cuda")
    gen = torch.Generator().manual_seed(0)

    class Cfg:
        hidden_size = 768
        max_width = 12
        class_token_index = 250100
        gliner_dropout = 0.0
        has_rnn = True
        embed_ent_token = True

    pooler = ref_mod.GLiNERSpanPooler(Cfg())
    with torch.no_grad():
        for p in pooler.parameters():
            p.copy_(torch.randn(p.shape, generator=gen) * 0.03)
    pooler = pooler.to(torch.bfloat16).eval()
    p32 = copy.deepcopy(pooler).float().to(dev).eval()
    pooler = pooler.to(dev)

    reqs = _requests(torch, gen, Cfg.class_token_index)
    lens = [len(ids) for ids, _ in reqs]
    hidden = torch.randn(sum(lens), Cfg.hidden_size, generator=gen).to(torch.bfloat16).to(dev)
    ctx = PoolerContext(seq_lengths=lens, extra_kwargs=[e for _, e in reqs],
                        prompt_token_ids=[torch.tensor(ids) for ids, _ in reqs])

    with torch.no_grad():
        fp32 = p32(hidden.float(), ctx)
        bf16 = pooler(hidden, ctx)
        span_scores.install_fused_span_scoring(type(pooler))
        fused = pooler(hidden, ctx)
        type(pooler).forward = type(pooler)._vf_reference_forward   # leave the class as shipped

    res = {"fused_forward": span_scores.gliner_span_pooler_forward.__module__, "requests": []}
    for f, b, r in zip(fused, bf16, fp32):
        r = r.float().cpu()
        entry = {"shape": list(r.shape)}
        for name, o in (("fused", f), ("torch_bf16", b)):
            o = o.float().cpu()
            if o.shape != r.shape:
                entry[name] = {"shape_ok": False, "shape": list(o.shape)}
                continue
            if r.dim() == 1 and r.numel() >= 3:
                # shape-prefixed scores: [L, K, C, then L * K * C values]
                prefix_ok = o[:3].tolist() == r[:3].tolist()
                L, K, C = (int(x) for x in r[:3].tolist())
                a, t = o[3:].view(L * K, C).double(), r[3:].view(L * K, C).double()
            else:
                prefix_ok = True
                a, t = o.reshape(-1, 1).double(), r.reshape(-1, 1).double()
            if t.numel() == 0:
                entry[name] = {"shape_ok": prefix_ok, "max_abs": 0.0, "min_cos": 1.0, "scale": 0.0}
                continue
            cos = 1.0
            if t.shape[1] >= 4:
                cos = torch.nn.functional.cosine_similarity(a, t, dim=-1, eps=1e-30).min().item()
            entry[name] = {"shape_ok": prefix_ok, "max_abs": (a - t).abs().max().item(), "min_cos": cos,
                           "scale": t.abs().max().item()}
        res["requests"].append(entry)
    print("RESULT " + json.dumps(res))


if __name__ == "__main__":
    main()
