"""Encoder-stack glue on the CPU (fp32, the oracle's packed attention): packing invariance
(a packed forward equals the per-sequence forwards), the DeBERTa position scores, and the
sequence partition used by the C3 / C4 bench."""
import dataclasses

import torch
import torch.nn.functional as F

import oracle
from vf_b200 import dist as VD
from vf_b200 import encoders as EN


def _deb_attn(q, k, v, cu, ms, pk, pq, c, sm, pb, mr, lg):
    return oracle.deberta_attention_varlen_ref(q, k, v, cu, pk, pq, c, sm, pb, mr, lg, dtype=torch.float32)


def _deb_fused_attn(q, k, v, cu, ms, pk, pq, c, sm, pb, mr, lg, rel_key=None, rel_query=None):
    assert pk is None and pq is None
    return oracle.deberta_attention_fused_varlen_ref(q, k, v, cu, rel_key, rel_query, c, sm, pb, mr, lg,
                                                     dtype=torch.float32)


def _t5_attn(q, k, v, cu, ms, t, nb, md, dec, sc):
    return oracle.rpb_attention_varlen_ref(q, k, v, cu, t, nb, md, dec, sc, dtype=torch.float32)


def _gated_act(gate, up, act_fn):
    return oracle.gated_act_ref(gate, up, 0)


def _packing_invariance(model, vocab):
    lengths, ids = EN.packed_batch(4, 3, 40, vocab, seed=1)
    x, cu, lens = EN.select_sequences(lengths, ids, range(4))
    packed = model.forward(x, cu, max(lens))
    assert packed.shape == (x.shape[0], model.cfg.hidden) and torch.isfinite(packed).all()
    for i in range(4):
        xi, cui, li = EN.select_sequences(lengths, ids, [i])
        one = model.forward(xi, cui, li[0])
        a = int(cu[i])
        torch.testing.assert_close(packed[a:a + li[0]], one, atol=2e-5, rtol=2e-5)


def test_deberta_encoder_packing_invariance():
    cfg = dataclasses.replace(EN.DebertaConfig(), layers=2, hidden=128, heads=2, ffn=256, vocab=500,
                              position_buckets=16, max_relative_positions=64)
    _packing_invariance(EN.DebertaV3Encoder(cfg, device="cpu", dtype=torch.float32, attention_fn=_deb_attn,
                                            add_norm=EN.add_layer_norm_torch, act_fn=F.gelu,
                                            fused_positions=False), 500)


def test_deberta_encoder_fused_positions_match_products():
    """The fused mode's arguments (Kr, Qr as (H, 2S, D) views) give the same stack output as
    the caller-side products (the reference's way) through the oracle."""
    cfg = dataclasses.replace(EN.DebertaConfig(), layers=2, hidden=128, heads=2, ffn=256, vocab=500,
                              position_buckets=16, max_relative_positions=64)
    kw = dict(device="cpu", dtype=torch.float32, add_norm=EN.add_layer_norm_torch, act_fn=F.gelu)
    fused = EN.DebertaV3Encoder(cfg, attention_fn=_deb_fused_attn, **kw)
    compat = EN.DebertaV3Encoder(cfg, attention_fn=_deb_attn, fused_positions=False, **kw)
    lengths, ids = EN.packed_batch(4, 3, 40, 500, seed=1)
    x, cu, lens = EN.select_sequences(lengths, ids, range(4))
    torch.testing.assert_close(fused.forward(x, cu, max(lens)), compat.forward(x, cu, max(lens)), atol=2e-5,
                               rtol=2e-5)
    _packing_invariance(fused, 500)


def test_mt5_encoder_packing_invariance():
    cfg = dataclasses.replace(EN.MT5Config(), layers=2, hidden=128, heads=2, ffn=160, vocab=500)
    _packing_invariance(EN.MT5Encoder(cfg, device="cpu", dtype=torch.float32, attention_fn=_t5_attn,
                                       gated_act=_gated_act), 500)


def test_deberta_position_scores_are_q_dot_kr():
    """The pos_key / pos_query views handed to the op equal q . Kr and k . Qr row by row."""
    cfg = dataclasses.replace(EN.DebertaConfig(), layers=1, hidden=128, heads=2, ffn=256, vocab=100,
                              position_buckets=8, max_relative_positions=32)
    seen = {}

    def spy(q, k, v, cu, ms, pk, pq, *rest):
        seen.update(q=q, k=k, pk=pk, pq=pq)
        return _deb_attn(q, k, v, cu, ms, pk, pq, *rest)

    m = EN.DebertaV3Encoder(cfg, device="cpu", dtype=torch.float32, attention_fn=spy,
                            add_norm=EN.add_layer_norm_torch, act_fn=F.gelu, fused_positions=False)
    lengths, ids = EN.packed_batch(2, 5, 9, 100, seed=2)
    x, cu, lens = EN.select_sequences(lengths, ids, range(2))
    m.forward(x, cu, max(lens))
    E, H = cfg.hidden, cfg.heads
    rel = torch.nn.functional.layer_norm(m.rel, (E,), *m.rel_ln, cfg.eps)
    L0 = m.layers[0]
    rk = (rel @ L0["wqkv"][E:2 * E].t() + L0["bqkv"][E:2 * E]).view(-1, H, 64)
    rq = (rel @ L0["wqkv"][:E].t() + L0["bqkv"][:E]).view(-1, H, 64)
    torch.testing.assert_close(seen["pk"], torch.einsum("thd,shd->ths", seen["q"], rk), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(seen["pq"], torch.einsum("thd,shd->ths", seen["k"], rq), atol=1e-5, rtol=1e-5)


def test_c3_c4_partition_covers_every_sequence():
    for lo, hi in ((128, 768), (512, 768)):
        lengths, _ = EN.packed_batch(256, lo, hi, 1000, seed=0)
        costs = [VD.attention_cost(int(L)) + 5e7 * int(L) for L in lengths.tolist()]
        for world in (1, 2, 4, 8):
            shards = VD.lpt_shard(costs, world)
            assert sorted(i for s in shards for i in s) == list(range(256))
            loads = [sum(costs[i] for i in s) for s in shards]
            assert max(loads) <= 1.05 * sum(loads) / world   # 256 items: near-even makespan
