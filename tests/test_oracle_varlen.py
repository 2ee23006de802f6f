"""The packed-batch oracle (each cu_seqlens sequence alone) against the padded oracle with
the reference's additive padding mask, on the valid rows: the two layouts describe the same
attention, so the packed form is pinned through the padded one (which tests/golden pins to
the reference)."""
import torch

import oracle
from _util import assert_close


def _padded_to_packed(x, lens):
    # (B, H, L, D) -> (sum(lens), H, D)
    return torch.cat([x[b, :, :L].permute(1, 0, 2) for b, L in enumerate(lens)], 0)


def test_varlen_oracle_matches_padded_oracle():
    g = torch.Generator().manual_seed(3)
    lens = [1, 37, 128, 129, 90, 0, 200]
    B, H, L = len(lens), 3, max(lens)
    q, k, v = (torch.randn(B, H, L, 64, generator=g) for _ in range(3))
    table = torch.randn(32, H, generator=g)
    valid = torch.arange(L)[None, :] < torch.tensor(lens)[:, None]
    mask = ((~valid).float() * torch.finfo(torch.float32).min)[:, None, None, :]
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32)
    for dec in (False, True):
        pad = oracle.rpb_attention_ref(q, k, v, table, 32, 128, dec, mask, 0.5)
        pk = oracle.rpb_attention_varlen_ref(_padded_to_packed(q, lens), _padded_to_packed(k, lens),
                                             _padded_to_packed(v, lens), cu, table, 32, 128, dec, 0.5)
        want = _padded_to_packed(pad, lens)
        assert_close(pk, want, None, max_abs=1e-9, min_cos=1 - 1e-12, what=f"decoder={dec}")


def test_varlen_oracle_leaves_rows_outside_sequences():
    q = torch.randn(10, 2, 64)
    out = oracle.rpb_attention_varlen_ref(q, q, q, [2, 5, 8], None, 32, 128, False, fill=7.0)
    assert torch.all(out[:2] == 7.0) and torch.all(out[8:] == 7.0)
    assert torch.isfinite(out[2:8]).all() and not torch.any(out[2:8] == 7.0)


def test_deberta_varlen_oracle_matches_padded_oracle():
    """Packed DeBERTa oracle against the padded oracle with seq_lengths (rows past a
    sequence are 0 there and absent here), log buckets, both position terms, causal too."""
    g = torch.Generator().manual_seed(4)
    lens = [1, 40, 129, 0, 200]
    B, H, L, S = len(lens), 2, max(lens), 32
    q, k, v = (torch.randn(B, H, L, 64, generator=g) for _ in range(3))
    pk, pq = (torch.randn(B, H, L, 2 * S, generator=g) for _ in range(2))
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0)), dtype=torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32)
    for causal in (False, True):
        pad = oracle.deberta_attention_ref(q, k, v, sl, pk, pq, causal, 0.1, S, 128, True)
        got = oracle.deberta_attention_varlen_ref(*(_padded_to_packed(t, lens) for t in (q, k, v)), cu,
                                                  _padded_to_packed(pk, lens), _padded_to_packed(pq, lens),
                                                  causal, 0.1, S, 128, True)
        assert_close(got, _padded_to_packed(pad, lens), None, max_abs=1e-9, min_cos=1 - 1e-12,
                     what=f"deberta causal={causal}")
