"""Encoder stacks around the packed attention ops: the C3 / C4 measurement workloads.

Two 24-layer encoders over a packed batch (token ids [T] and cu_seqlens [S+1]), with
random-init weights ~N(0, 0.02) in bf16.  The GEMMs, norms, activations and embeddings are
plain torch (cuBLAS); the attention of every layer is this package's packed op, so the
stacks measure encoder tokens/s with the hot path in place:

  DebertaV3Encoder  models/deberta_v2/deberta_v2_encoder.py (DebertaV2 embeddings without
                    absolute positions, DisentangledSelfAttentionV2._flash_forward :246-328
                    with share_att_key, c2p|p2c, position_buckets 256 / max_relative 512,
                    rel_embeddings + LayerNorm, exact-GELU FFN, post-LayerNorm residuals
                    through this package's fused_add_layer_norm as at :507 / :566).
  MT5Encoder        models/mt5/mt5_encoder.py (T5 RMS LayerNorm, no QK scaling, the bias
                    table of layer 0 shared by all layers :546-566, gated-GELU FFN with the
                    tanh GELU through this package's fused_gelu_mul_dropout as at :418,
                    final RMS norm).

DeBERTa's position terms: by default the stack passes Kr = key_proj(rel) and
Qr = query_proj(rel) (biases included) to the op's fused mode, which forms q . Kr and
k . Qr on the tensor cores inside the attention kernel.  With `fused_positions=False` it
forms them as the reference's caller does, per packed row (pos_key[t, h, :] = q[t, h] . Kr,
pos_query[t, h, :] = k[t, h] . Qr, two batched GEMMs), and hands them over as [T, H, 2S]
views.
"""
from __future__ import annotations

import math
from typing import Optional
from dataclasses import dataclass

import torch
import torch.nn.functional as F

HIDDEN = 1024
HEADS = 16
HEAD_DIM = 64


@dataclass(frozen=True)
class DebertaConfig:
    layers: int = 24
    hidden: int = HIDDEN
    heads: int = HEADS
    ffn: int = 4096
    vocab: int = 128100
    position_buckets: int = 256
    max_relative_positions: int = 512
    eps: float = 1e-7


@dataclass(frozen=True)
class MT5Config:
    layers: int = 24
    hidden: int = HIDDEN
    heads: int = HEADS
    ffn: int = 2816
    vocab: int = 250112
    num_buckets: int = 32
    max_distance: int = 128
    eps: float = 1e-6


def _normal(gen: torch.Generator, shape, device, dtype) -> torch.Tensor:
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * 0.02).to(dtype)


def _layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), w, b, eps)


def add_layer_norm_torch(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, b: torch.Tensor,
                         eps: float) -> torch.Tensor:
    """The reference's two torch calls, LayerNorm(x + residual): the encoders' CPU form."""
    return _layer_norm(x + residual, w, b, eps)


def exact_gelu_kernel(x: torch.Tensor) -> torch.Tensor:
    """The DeBERTa feed-forward's exact (erf) GELU on this package's activation kernel
    (torch.ops.vf_b200.gated_act with no `up`): one pass at the HBM rate."""
    import vf_b200.ops  # noqa: F401
    from vf_b200 import _lib
    return torch.ops.vf_b200.gated_act(x, None, _lib.VF_ACT_GELU_ERF)


def _rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    # T5LayerNorm (no mean subtraction, no bias) as torch's fused RMS norm, which keeps the
    # variance in fp32 for 16-bit inputs like models/mt5/mt5_encoder.py does
    return F.rms_norm(x, (x.shape[-1],), w, eps)


class DebertaV3Encoder:
    """DeBERTa-v3 encoder over a packed batch; attention = flash_deberta_attention_varlen and
    the residual add + LayerNorm = fused_add_layer_norm (or, with `attention_fn` / `add_norm`,
    any function of the same signature, e.g. a CPU oracle)."""

    def __init__(self, cfg: DebertaConfig = DebertaConfig(), device="cuda", dtype=torch.bfloat16, seed: int = 0,
                 attention_fn=None, add_norm=None, act_fn=None, fused_positions: bool = True,
                 fused_ffn: Optional[bool] = None):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        g = torch.Generator(device=self.device).manual_seed(seed)
        E, F_, S2 = cfg.hidden, cfg.ffn, 2 * cfg.position_buckets
        n = lambda *shape: _normal(g, shape, self.device, dtype)
        ones = lambda k: torch.ones(k, device=self.device, dtype=dtype)
        zeros = lambda k: torch.zeros(k, device=self.device, dtype=dtype)
        self.word = n(cfg.vocab, E)
        self.emb_ln = (ones(E), zeros(E))
        # rel_embeddings [2S, E]; the encoder's LayerNorm is applied in forward
        # (get_rel_embedding with norm_rel_ebd = "layer_norm")
        self.rel = n(S2, E)
        self.rel_ln = (ones(E), zeros(E))
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append(dict(
                wqkv=n(3 * E, E), bqkv=zeros(3 * E),          # query_proj, key_proj, value_proj
                wo=n(E, E), bo=zeros(E), ln1=(ones(E), zeros(E)),
                w1=n(F_, E), b1=zeros(F_), w2=n(E, F_), b2=zeros(E), ln2=(ones(E), zeros(E))))
        if attention_fn is None:
            from kernels.flash_deberta_attention import flash_deberta_attention_varlen as attention_fn
        self.attention_fn = attention_fn
        if add_norm is None:
            from kernels.fused_add_layernorm import fused_add_layer_norm as add_norm
        self.add_norm = add_norm
        # torch's exact GELU (the reference's ACT2FN["gelu"]); exact_gelu_kernel, this
        # package's activation-only kernel, measured the same C3 tokens/s in its place
        self.act_fn = F.gelu if act_fn is None else act_fn
        self.fused_positions = fused_positions
        # The feed-forward's dense layer + exact GELU as one GEMM with the activation in its
        # epilogue (kernels.linear_act), unless another activation was given.
        self.fused_ffn = (act_fn is None) if fused_ffn is None else fused_ffn
        if self.fused_ffn:
            from kernels.linear_act import linear_gelu
            self.linear_gelu = linear_gelu

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int) -> torch.Tensor:
        cfg, E, H, D = self.cfg, self.cfg.hidden, self.cfg.heads, HEAD_DIM
        T = ids.shape[0]
        h = _layer_norm(self.word[ids], *self.emb_ln, cfg.eps)
        rel = _layer_norm(self.rel, *self.rel_ln, cfg.eps)                     # [2S, E]
        sm_scale = 1.0 / math.sqrt(D * 3)
        for L in self.layers:
            qkv = torch.addmm(L["bqkv"], h, L["wqkv"].t()).view(T, 3, H, D)
            q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
            # share_att_key: Kr = key_proj(rel), Qr = query_proj(rel), biases included
            rq = torch.addmm(L["bqkv"][:E], rel, L["wqkv"][:E].t()).view(-1, H, D)
            rk = torch.addmm(L["bqkv"][E:2 * E], rel, L["wqkv"][E:2 * E].t()).view(-1, H, D)
            if self.fused_positions:
                # (H, 2S, D) views of the projections; the kernel forms q . Kr and k . Qr
                ctx = self.attention_fn(q, k, v, cu_seqlens, max_seqlen, None, None, False, sm_scale,
                                        cfg.position_buckets, cfg.max_relative_positions, True,
                                        rel_key=rk.permute(1, 0, 2), rel_query=rq.permute(1, 0, 2))
            else:
                pos_key = torch.bmm(q.transpose(0, 1), rk.permute(1, 2, 0)).transpose(0, 1)     # [T, H, 2S]
                pos_query = torch.bmm(k.transpose(0, 1), rq.permute(1, 2, 0)).transpose(0, 1)
                ctx = self.attention_fn(q, k, v, cu_seqlens, max_seqlen, pos_key, pos_query, False, sm_scale,
                                        cfg.position_buckets, cfg.max_relative_positions, True)
            a = torch.addmm(L["bo"], ctx.reshape(T, E).to(h.dtype), L["wo"].t())
            h = self.add_norm(a, h, *L["ln1"], cfg.eps)
            if self.fused_ffn:
                f = self.linear_gelu(h, L["w1"], L["b1"])
            else:
                f = self.act_fn(torch.addmm(L["b1"], h, L["w1"].t()))
            h = self.add_norm(torch.addmm(L["b2"], f, L["w2"].t()), h, *L["ln2"], cfg.eps)
        return h

    def flops_per_token_gemm(self) -> float:
        E, F_ = self.cfg.hidden, self.cfg.ffn
        return self.cfg.layers * 2.0 * (4 * E * E + 2 * E * F_)

    def own_launches_per_layer(self) -> int:
        """This package's kernel launches per layer: the attention (with the fused mode's
        set-up kernel), two add + LayerNorm and the fused dense + GELU."""
        return (4 if self.fused_positions else 3) + (1 if self.fused_ffn else 0)


class MT5Encoder:
    """mT5 encoder over a packed batch; attention = flash_attention_rpb_varlen and the
    gated-GELU of the FFN = fused_gelu_mul_dropout (or `attention_fn` / `gated_act` of the
    same signatures)."""

    def __init__(self, cfg: MT5Config = MT5Config(), device="cuda", dtype=torch.bfloat16, seed: int = 0,
                 attention_fn=None, gated_act=None, fused_ffn: Optional[bool] = None):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        g = torch.Generator(device=self.device).manual_seed(seed)
        E, F_ = cfg.hidden, cfg.ffn
        n = lambda *shape: _normal(g, shape, self.device, dtype)
        ones = lambda k: torch.ones(k, device=self.device, dtype=dtype)
        self.word = n(cfg.vocab, E)
        self.table = n(cfg.num_buckets, cfg.heads)          # relative_attention_bias of layer 0
        self.layers = []
        for _ in range(cfg.layers):
            self.layers.append(dict(
                ln1=ones(E), wqkv=n(3 * E, E), wo=n(E, E),
                ln2=ones(E), wi=n(2 * F_, E), wo_ff=n(E, F_)))  # wi_0 and wi_1 stacked
        self.final_ln = ones(E)
        if attention_fn is None:
            from kernels.flash_attention_rpb import flash_attention_rpb_varlen as attention_fn
        self.attention_fn = attention_fn
        # The gated-GELU in the gate projection's GEMM epilogue (kernels.linear_act), unless
        # another activation function was given: up = x wi_1^T, then gelu_tanh(x wi_0^T) * up.
        self.fused_ffn = (gated_act is None) if fused_ffn is None else fused_ffn
        if gated_act is None:
            from kernels.ff_fused import fused_gelu_mul_dropout as gated_act
        self.gated_act = gated_act
        if self.fused_ffn:
            from kernels.linear_act import gated_gelu_tanh
            self.gated_gelu_tanh = gated_gelu_tanh

    @torch.no_grad()
    def forward(self, ids: torch.Tensor, cu_seqlens: torch.Tensor, max_seqlen: int) -> torch.Tensor:
        cfg, E, H, D, F_ = self.cfg, self.cfg.hidden, self.cfg.heads, HEAD_DIM, self.cfg.ffn
        T = ids.shape[0]
        h = self.word[ids]
        for L in self.layers:
            x = _rms_norm(h, L["ln1"], cfg.eps)
            qkv = (x @ L["wqkv"].t()).view(T, 3, H, D)
            ctx = self.attention_fn(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu_seqlens, max_seqlen, self.table,
                                    cfg.num_buckets, cfg.max_distance, False, 1.0)
            h = h + ctx.reshape(T, E).to(h.dtype) @ L["wo"].t()
            x = _rms_norm(h, L["ln2"], cfg.eps)
            if self.fused_ffn:
                up = x @ L["wi"][F_:].t()
                f = self.gated_gelu_tanh(x, L["wi"][:F_], up)
            else:
                gu = x @ L["wi"].t()
                f = self.gated_act(gu[:, :F_], gu[:, F_:], "gelu_new")     # gated-GELU, halves read in place
            h = h + f @ L["wo_ff"].t()
        return _rms_norm(h, self.final_ln, cfg.eps)

    def flops_per_token_gemm(self) -> float:
        E, F_ = self.cfg.hidden, self.cfg.ffn
        return self.cfg.layers * 2.0 * (4 * E * E + 3 * E * F_)

    def own_launches_per_layer(self) -> int:
        """This package's kernel launches per layer: the attention and the gated activation."""
        return 2


def packed_batch(n_seqs: int, lo: int, hi: int, vocab: int, seed: int = 0):
    """Seeded lengths ~U[lo, hi] (drawn first) and token ids uniform over the vocabulary."""
    g = torch.Generator().manual_seed(seed)
    lengths = torch.randint(lo, hi + 1, (n_seqs,), generator=g)
    ids = torch.randint(0, vocab, (int(lengths.sum()),), generator=g)
    return lengths, ids


def select_sequences(lengths: torch.Tensor, ids: torch.Tensor, which):
    """The packed ids and cu_seqlens of the sequences `which` (in that order)."""
    starts = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(lengths, 0)])
    parts = [ids[int(starts[i]):int(starts[i + 1])] for i in which]
    lens = [int(lengths[i]) for i in which]
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens, dtype=torch.long), 0).tolist()), dtype=torch.int32)
    return (torch.cat(parts) if parts else torch.zeros(0, dtype=torch.long)), cu, lens
