"""A flat vLLM batch of three requests through the drop-ins inside `varlen_glue.packed_batch`:
every request's rows must equal that request run alone (the oracle on its rows, and the
drop-in on the request alone), within the parity gates.  Covers the DeBERTa product mode,
the fused position mode and the T5 bias mode."""
import pytest
import torch

import oracle
from _util import assert_close
from kernels import varlen_glue
from kernels.flash_attention_rpb import flash_attention_rpb_final
from kernels.flash_deberta_attention import flash_deberta_attention

pytestmark = pytest.mark.gpu

LENS = (300, 129, 77)
H, S, MRD = 4, 256, 512


def _flat(seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(LENS)
    bf = torch.bfloat16
    q, k, v = (torch.randn(1, H, T, 64, generator=g).to(bf).cuda() for _ in range(3))
    rk, rq = ((torch.randn(1, H, 2 * S, 64, generator=g) * 0.4).to(bf).cuda() for _ in range(2))
    positions = torch.cat([torch.arange(n) for n in LENS]).cuda()
    return q, k, v, rk, rq, positions


def _requests():
    a = 0
    for n in LENS:
        yield a, a + n
        a += n


def test_deberta_products_flat_batch():
    q, k, v, rk, rq, positions = _flat(0)
    pk = (q @ rk.transpose(-1, -2))                    # the caller's c2p products, one row per token
    pq = (k @ rq.transpose(-1, -2))
    with varlen_glue.packed_batch(positions):
        out = flash_deberta_attention(q, k, v, None, pk, pq, False, 0.07, S, MRD, True)
    assert out.shape == q.shape
    for a, b in _requests():
        sl = lambda t: t[:, :, a:b]                     # noqa: E731
        ref = oracle.deberta_attention_ref(sl(q).cpu(), sl(k).cpu(), sl(v).cpu(), None, sl(pk).cpu(), sl(pq).cpu(),
                                           False, 0.07, S, MRD, True)
        assert_close(sl(out), ref, what=f"request rows {a}:{b} vs oracle")
        alone = flash_deberta_attention(sl(q), sl(k), sl(v), None, sl(pk), sl(pq), False, 0.07, S, MRD, True)
        assert_close(sl(out), alone.float(), what=f"request rows {a}:{b} vs the request alone")


def test_deberta_fused_flat_batch():
    q, k, v, rk, rq, positions = _flat(1)
    with varlen_glue.packed_batch(positions):
        out = flash_deberta_attention(q, k, v, None, causal=False, sm_scale=0.07, position_buckets=S,
                                      max_relative_distance=MRD, use_log_bucket=True, rel_key=rk, rel_query=rq)
    for a, b in _requests():
        sl = lambda t: t[:, :, a:b]                     # noqa: E731
        ref = oracle.deberta_attention_fused_ref(sl(q).cpu(), sl(k).cpu(), sl(v).cpu(), None, rk.cpu(), rq.cpu(),
                                                 False, 0.07, S, MRD, True)
        assert_close(sl(out), ref, what=f"request rows {a}:{b} vs oracle")


def test_t5_flat_batch():
    q, k, v, _, _, positions = _flat(2)
    table = torch.randn(32, H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16).cuda()
    mask = torch.zeros(1, 1, 1, q.size(2), dtype=torch.bfloat16, device="cuda")   # a flat batch: all valid
    with varlen_glue.packed_batch(positions):
        out = flash_attention_rpb_final(q, k, v, table, 32, 128, False, padding_mask=mask)
    for a, b in _requests():
        sl = lambda t: t[:, :, a:b]                     # noqa: E731
        ref = oracle.rpb_attention_ref(sl(q).cpu(), sl(k).cpu(), sl(v).cpu(), table.cpu(), 32, 128, False)
        assert_close(sl(out), ref, what=f"request rows {a}:{b} vs oracle")
    # Without the context the same flat call is one sequence, as the reference computes it.
    whole = flash_attention_rpb_final(q, k, v, table, 32, 128, False, padding_mask=mask)
    assert_close(whole, oracle.rpb_attention_ref(q.cpu(), k.cpu(), v.cpu(), table.cpu(), 32, 128, False),
                 what="flat call without a packed batch")
