"""GPU parity of the DeBERTa disentangled attention op (kernels.flash_deberta_attention
drop-in) against the CPU oracle (fp64) and the reference's golden outputs.  Gates:
max-abs <= 2e-2 and per-row cosine >= 0.9999 on valid rows; rows past seq_len are 0."""
import math

import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle
from _util import assert_close, lens_mask

pytestmark = pytest.mark.gpu


def _op():
    from kernels.flash_deberta_attention import flash_deberta_attention
    return flash_deberta_attention


def make(B, H, M, N, S, dtype=torch.bfloat16, lens=None, seed=0, c2p=True, p2c=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, M, 64, generator=g).to(dtype)
    k = torch.randn(B, H, N, 64, generator=g).to(dtype)
    v = torch.randn(B, H, N, 64, generator=g).to(dtype)
    pk = (torch.randn(B, H, M, 2 * S, generator=g) * 3).to(dtype) if c2p else None
    pq = (torch.randn(B, H, N, 2 * S, generator=g) * 3).to(dtype) if p2c else None
    sl = None if lens is None else torch.tensor(lens, dtype=torch.int32)
    return q, k, v, pk, pq, sl


def run(q, k, v, pk, pq, sl, causal=False, sm_scale=None, pb=0, mr=0, log=False, what=""):
    dev = torch.device("cuda")
    cu = lambda t: None if t is None else t.to(dev)
    out = _op()(cu(q), cu(k), cu(v), cu(sl), cu(pk), cu(pq), causal, sm_scale, pb, mr, log)
    torch.cuda.synchronize()
    ref = oracle.deberta_attention_ref(q.float(), k.float(), v.float(), sl, None if pk is None else pk.float(),
                                       None if pq is None else pq.float(), causal, sm_scale, pb, mr, log)
    assert out.shape == q.shape and out.dtype == q.dtype
    assert torch.isfinite(out.float()).all(), what
    M = q.shape[2]
    valid = lens_mask(sl if sl is not None else [M] * q.shape[0], M)
    assert_close(out, ref, valid, what=what)
    if sl is not None:
        pad = ~valid
        assert (out.float().cpu()[pad[:, None, :].expand(out.shape[:3])] == 0).all(), f"{what}: padded rows must be 0"
    return out


@pytest.mark.parametrize("L", [1, 63, 128, 200, 256, 257, 512])
def test_deberta_v3_log_buckets(L):
    q, k, v, pk, pq, sl = make(2, 2, L, L, 256, lens=[L, max(1, (2 * L) // 3)], seed=L)
    run(q, k, v, pk, pq, sl, sm_scale=1 / math.sqrt(64 * 3), pb=256, mr=512, log=True, what=f"v3 L={L}")


def test_deberta_long_sequence_saturated_buckets():
    q, k, v, pk, pq, sl = make(1, 2, 1100, 1100, 256, lens=[1100], seed=3)
    run(q, k, v, pk, pq, sl, sm_scale=0.07, pb=256, mr=512, log=True, what="L=1100")


def test_deberta_v1_linear_positions():
    # models/deberta/deberta_encoder.py:258: att_span = min(max(M, N), max_rel)
    L = 300
    q, k, v, pk, pq, sl = make(2, 2, L, L, L, lens=[300, 150], seed=4)
    run(q, k, v, pk, pq, sl, sm_scale=1 / math.sqrt(64 * 3), pb=L, mr=512, log=False, what="v1 linear")


@pytest.mark.parametrize("c2p,p2c", [(True, False), (False, True), (False, False)])
def test_deberta_partial_terms(c2p, p2c):
    q, k, v, pk, pq, sl = make(2, 2, 192, 192, 64, lens=[192, 90], seed=5, c2p=c2p, p2c=p2c)
    run(q, k, v, pk, pq, sl, sm_scale=None, pb=64, mr=128, log=True, what=f"c2p={c2p} p2c={p2c}")


def test_deberta_no_seq_lengths_and_fp16():
    q, k, v, pk, pq, _ = make(2, 2, 300, 300, 128, dtype=torch.float16, seed=6)
    run(q, k, v, pk, pq, None, sm_scale=0.1, pb=128, mr=512, log=True, what="fp16 full")


def test_deberta_zero_length_rows():
    q, k, v, pk, pq, sl = make(3, 2, 160, 160, 64, lens=[160, 0, 1], seed=7)
    out = run(q, k, v, pk, pq, sl, pb=64, mr=128, log=True, what="zero length")
    assert (out[1].float() == 0).all()


def test_deberta_causal():
    q, k, v, pk, pq, sl = make(2, 2, 260, 260, 64, lens=[260, 200], seed=8)
    run(q, k, v, pk, pq, sl, causal=True, pb=64, mr=128, log=True, what="causal")


def test_deberta_cross_lengths():
    q, k, v, pk, pq, sl = make(2, 2, 100, 300, 64, lens=[90, 300], seed=9)
    run(q, k, v, pk, pq, sl, pb=64, mr=128, log=True, what="M!=N")


@pytest.mark.parametrize("name", ["deberta_log", "deberta_linear"])
def test_deberta_golden_reference_cases(name):
    G = np.load(gi.__file__.replace("golden_inputs.py", "golden.npz"))
    c = gi.deberta_op_case(name)
    bf = torch.bfloat16
    dev = torch.device("cuda")
    out = _op()(c["q"].to(bf).to(dev), c["k"].to(bf).to(dev), c["v"].to(bf).to(dev), c["seq_lengths"].to(dev),
                c["pos_key"].to(bf).to(dev), c["pos_query"].to(bf).to(dev), False, c["sm_scale"],
                c["position_buckets"], c["max_relative_distance"], c["use_log_bucket"])
    ref = torch.from_numpy(G[f"{name}_out"])
    assert_close(out, ref, lens_mask(c["seq_lengths"], out.shape[2]), what=f"golden {name}")


def test_deberta_layer_glue_matches_reference_layer():
    """The reference layer's _flash_forward glue (deberta_v2_encoder.py:246-328) restated
    around the op reproduces the reference's _pytorch_forward (golden) on valid rows."""
    G = np.load(gi.__file__.replace("golden_inputs.py", "golden.npz"))
    c = gi.deberta_layer_case()
    dev = torch.device("cuda")
    bf = torch.bfloat16
    H, pb, mr = c["num_heads"], c["position_buckets"], c["max_relative_positions"]
    hid = c["hidden"].to(dev).to(bf)
    lin = lambda x, w, b: x @ w.to(dev).to(bf).t() + b.to(dev).to(bf)
    B, L, E = hid.shape
    t4 = lambda x: x.view(x.shape[0], x.shape[1], H, -1).permute(0, 2, 1, 3)
    q, k, v = t4(lin(hid, c["wq"], c["bq"])), t4(lin(hid, c["wk"], c["bk"])), t4(lin(hid, c["wv"], c["bv"]))
    rel = c["rel"].to(dev).to(bf)[0:2 * pb].unsqueeze(0)
    pos_key = torch.matmul(q, t4(lin(rel, c["wk"], c["bk"])).transpose(-1, -2))
    pos_query = torch.matmul(k, t4(lin(rel, c["wq"], c["bq"])).transpose(-1, -2))
    seq = c["mask"].to(dev).sum(-1).int()
    ctx = _op()(q, k, v, seq, pos_key, pos_query, False, 1.0 / (64 * 3) ** 0.5, pb, mr, True)
    ctx = ctx.permute(0, 2, 1, 3).contiguous().view(B, L, E)
    ref = torch.from_numpy(G["deberta_layer_out"])
    valid = lens_mask(c["lens"], L)
    err = (ctx.float().cpu()[valid] - ref[valid]).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(ctx.float().cpu()[valid].double(), ref[valid].double(), dim=-1).min().item()
    assert err < 2e-2 and cos > 0.9999, (err, cos)


def test_deberta_c1_config_subset():
    from vf_b200.workloads import deberta_attention_inputs
    w = deberta_attention_inputs(seed=0, device="cuda")
    out = _op()(w["q"], w["k"], w["v"], w["seq_lengths"], w["pos_key"], w["pos_query"], False, w["sm_scale"],
                256, 512, True)
    for b in (0, 5):
        sl = w["seq_lengths"][b:b + 1].cpu()
        ref = oracle.deberta_attention_ref(*(w[n][b:b + 1].float().cpu() for n in ("q", "k", "v")), sl,
                                           w["pos_key"][b:b + 1].float().cpu(), w["pos_query"][b:b + 1].float().cpu(),
                                           False, w["sm_scale"], 256, 512, True)
        assert_close(out[b:b + 1], ref, lens_mask(sl, out.shape[2]), what=f"C1 batch {b}")


def test_deberta_fp32_inputs_tf32_level():
    """fp32 inputs (the C1 workload's dtype: 8 x 512, U[64,512]): fp16 operands, fp32 softmax/accumulation, fp32 out."""
    q, k, v, pk, pq, sl = make(2, 2, 320, 320, 256, dtype=torch.float32, lens=[320, 200], seed=23)
    dev = torch.device("cuda")
    cu = lambda t: None if t is None else t.to(dev)
    out = _op()(cu(q), cu(k), cu(v), cu(sl), cu(pk), cu(pq), False, 1.0 / math.sqrt(64 * 3), 256, 512, True)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == q.shape
    ref = oracle.deberta_attention_ref(q, k, v, sl, pk, pq, False, 1.0 / math.sqrt(64 * 3), 256, 512, True)
    valid = lens_mask(sl, 320)
    err, cos = assert_close(out, ref, valid, max_abs=2e-3, min_cos=0.99999, what="fp32 inputs")
    print(f"fp32 deberta: max_abs {err:.3e} min_cos {cos:.7f}")
    assert (out.float().cpu()[(~valid)[:, None, :].expand(out.shape[:3])] == 0).all()


def test_deberta_many_short_sequences_natural_order():
    """More (batch, query block) pairs than the cost-ordering table holds, some of length 0."""
    B, L = 1100, 64
    lens = [(29 * b) % (L + 1) for b in range(B)]
    q, k, v, pk, pq, sl = make(B, 1, L, L, 32, lens=lens, seed=33)
    run(q, k, v, pk, pq, sl, sm_scale=0.125, pb=32, mr=64, log=True, what="1100 sequences")


def test_deberta_position_views_strided_and_transposed():
    """Position tensors as views: sliced out of wider tensors (large row strides, gathered in
    place with 32-bit in-tile offsets) and with a non-unit last-dimension stride (the op
    makes those contiguous first)."""
    B, H, L, S = 2, 2, 300, 256
    g = torch.Generator().manual_seed(41)
    q, k, v = (torch.randn(B, H, L, 64, generator=g).to(torch.bfloat16) for _ in range(3))
    wide_k = (torch.randn(B, H, L, 3 * S, generator=g) * 3).to(torch.bfloat16)
    pk = wide_k[..., S:3 * S]                                  # row stride 3S, unit index stride
    pq = (torch.randn(B, H, 2 * S, L, generator=g) * 3).to(torch.bfloat16).transpose(-1, -2)
    sl = torch.tensor([300, 211], dtype=torch.int32)
    sm = 1 / math.sqrt(64 * 3)
    dev = torch.device("cuda")
    pk_dev = wide_k.to(dev)[..., S:3 * S]                      # slice on the device: strides kept
    assert pk_dev.stride(-2) == 3 * S and pq.to(dev).stride(-1) != 1
    out = _op()(q.to(dev), k.to(dev), v.to(dev), sl.to(dev), pk_dev, pq.to(dev), False, sm, S, 512, True)
    ref = oracle.deberta_attention_ref(q.float(), k.float(), v.float(), sl, pk.float(), pq.float(), False, sm, S,
                                       512, True)
    assert_close(out, ref, lens_mask(sl, L), what="strided / transposed position views")
