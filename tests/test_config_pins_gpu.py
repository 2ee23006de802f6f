"""Parity pins at the benchmark configurations themselves, on the exact inputs bench.py times
(same generators and seeds): every batch row of C1 (DeBERTa 8 x 512, bf16 and fp32) and of
C2 (mT5 16 x 768), and the C5 long-context cases L = 2048 and 4096 in both DeBERTa modes,
where the fp64 oracle checks one (sequence, head) slice at each end of the batch.
Gates: bf16 max-abs <= 2e-2 and per-row cosine >= 0.9999 on valid rows; fp32 inputs
max-abs <= 2e-3 and cosine >= 0.99999 (TF32-level)."""
import pytest
import torch

import oracle
from _util import assert_close, lens_mask
from kernels.flash_attention_rpb import flash_attention_rpb_final
from kernels.flash_deberta_attention import flash_deberta_attention
from vf_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _c(t):
    return t.float().cpu()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_c1_every_batch_row(dtype):
    x = W.deberta_attention_inputs(seed=2000, device="cuda", dtype=dtype)
    out = flash_deberta_attention(x["q"], x["k"], x["v"], x["seq_lengths"], x["pos_key"], x["pos_query"], False,
                                  x["sm_scale"], 256, 512, True)
    torch.cuda.synchronize()
    assert out.dtype == dtype
    lens = x["lengths"]
    valid = lens_mask(lens, 512)
    gate = dict(max_abs=2e-3, min_cos=0.99999) if dtype == torch.float32 else {}
    for b in range(8):
        sl = slice(b, b + 1)
        ref = oracle.deberta_attention_ref(_c(x["q"][sl]), _c(x["k"][sl]), _c(x["v"][sl]), lens[sl].to(torch.int32),
                                           _c(x["pos_key"][sl]), _c(x["pos_query"][sl]), False, x["sm_scale"], 256,
                                           512, True)
        assert_close(out[sl], ref, valid[sl], what=f"C1 {dtype} row {b}", **gate)
    pad = ~valid
    assert (out.float().cpu()[pad[:, None, :].expand(out.shape[:3])] == 0).all()


def test_c2_every_batch_row():
    x = W.mt5_attention_inputs(seed=1000, device="cuda")
    out = flash_attention_rpb_final(x["q"], x["k"], x["v"], x["rpb_table"], 32, 128, False, x["padding_mask"],
                                    0.0, 1.0)
    torch.cuda.synchronize()
    valid = lens_mask(x["lengths"], 768)
    for b in range(16):
        sl = slice(b, b + 1)
        ref = oracle.rpb_attention_ref(_c(x["q"][sl]), _c(x["k"][sl]), _c(x["v"][sl]), _c(x["rpb_table"]), 32, 128,
                                       False, _c(x["padding_mask"][sl]), 1.0)
        assert_close(out[sl], ref, valid[sl], what=f"C2 row {b} valid rows")
        assert_close(out[sl], ref, None, what=f"C2 row {b} all rows (padded rows are computed, as in the reference)")


@pytest.mark.parametrize("L", [2048, 4096])
@pytest.mark.parametrize("fused", [False, True], ids=["products", "fused"])
def test_c5_long_context(L, fused):
    B = 16384 // L
    x = W.deberta_attention_inputs(seed=3000, device="cuda", B=B, L=L, lengths=[L] * B)
    if fused:
        out = flash_deberta_attention(x["q"], x["k"], x["v"], x["seq_lengths"], None, None, False, x["sm_scale"], 256,
                                      512, True, rel_key=x["rel_key"], rel_query=x["rel_query"])
    else:
        out = flash_deberta_attention(x["q"], x["k"], x["v"], x["seq_lengths"], x["pos_key"], x["pos_query"], False,
                                      x["sm_scale"], 256, 512, True)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    for b, h in ((0, 0), (B - 1, 15)):
        s, hs = slice(b, b + 1), slice(h, h + 1)
        q, k, v = (_c(x[n][s, hs]) for n in ("q", "k", "v"))
        sl = torch.tensor([L], dtype=torch.int32)
        if fused:
            ref = oracle.deberta_attention_fused_ref(q, k, v, sl, _c(x["rel_key"][:, hs]), _c(x["rel_query"][:, hs]),
                                                     False, x["sm_scale"], 256, 512, True)
        else:
            ref = oracle.deberta_attention_ref(q, k, v, sl, _c(x["pos_key"][s, hs]), _c(x["pos_query"][s, hs]), False,
                                               x["sm_scale"], 256, 512, True)
        assert_close(out[s, hs], ref, None, what=f"C5 L={L} {'fused' if fused else 'products'} seq {b} head {h}")
