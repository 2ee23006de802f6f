"""Host logic of the packed-batch glue (kernels/varlen_glue.py), on CPU: request boundaries
from vLLM positions, the context stack, and which flat calls the drop-ins hand to the packed
operators, with what views.  The packed operators are replaced by spies here; the GPU
results are checked in test_varlen_glue_gpu.py."""
import pytest
import torch

import kernels.flash_attention_rpb as rpb_mod
import kernels.flash_deberta_attention as deb_mod
from kernels import varlen_glue as g


def _positions(lens):
    return torch.cat([torch.arange(n) for n in lens])


@pytest.mark.parametrize("lens", [[5], [3, 2, 4], [1, 1, 1], [7, 1], [128, 300, 17, 1]])
def test_cu_seqlens_from_positions(lens):
    cu, mx = g.cu_seqlens_from_positions(_positions(lens))
    assert cu.dtype == torch.int32
    assert cu.tolist() == [0] + torch.tensor(lens).cumsum(0).tolist()
    assert mx == max(lens)


def test_cu_seqlens_edge_cases():
    cu, mx = g.cu_seqlens_from_positions(torch.zeros(0, dtype=torch.long))
    assert cu.tolist() == [0] and mx == 0
    with pytest.raises(ValueError, match="first token"):
        g.cu_seqlens_from_positions(torch.tensor([3, 4, 0, 1]))
    with pytest.raises(ValueError, match="1-D"):
        g.cu_seqlens_from_positions(torch.zeros(2, 3, dtype=torch.long))


def test_context_stack_and_routing_rule():
    assert g.current() is None
    q_flat = torch.zeros(1, 2, 9, 64)
    with g.packed_batch(_positions([3, 2, 4])) as outer:
        assert g.current() is outer and outer.num_seqs == 3 and outer.total == 9
        assert g.routes(q_flat) is outer
        assert g.routes(torch.zeros(2, 2, 9, 64)) is None          # a padded batch is left alone
        assert g.routes(torch.zeros(1, 2, 8, 64)) is None          # not this batch's tokens
        with g.packed_batch(cu_seqlens=torch.tensor([0, 4], dtype=torch.int32), max_seqlen=4) as inner:
            assert g.current() is inner
            assert g.routes(torch.zeros(1, 2, 4, 64)) is None      # one request: the flat call is already right
        assert g.current() is outer
    assert g.current() is None and g.routes(q_flat) is None


def test_context_argument_errors():
    with pytest.raises(ValueError):
        with g.packed_batch():
            pass
    with pytest.raises(ValueError):
        with g.packed_batch(_positions([2]), cu_seqlens=torch.tensor([0, 2], dtype=torch.int32), max_seqlen=2):
            pass
    with pytest.raises(ValueError, match="max_seqlen"):
        with g.packed_batch(cu_seqlens=torch.tensor([0, 2], dtype=torch.int32)):
            pass
    with pytest.raises(ValueError, match="int32"):
        with g.packed_batch(cu_seqlens=torch.tensor([0, 2]), max_seqlen=2):
            pass


def test_context_closes_on_error():
    with pytest.raises(RuntimeError):
        with g.packed_batch(_positions([2, 2])):
            raise RuntimeError("layer failed")
    assert g.current() is None


class _Spy:
    def __init__(self):
        self.calls = []

    def __call__(self, *args, **kwargs):
        self.calls.append((args, kwargs))
        q = args[0]
        return torch.full_like(q, 7.0)


def test_deberta_flat_call_goes_to_the_packed_operator(monkeypatch):
    spy = _Spy()
    monkeypatch.setattr(deb_mod, "flash_deberta_attention_varlen", spy)
    H, T, S = 2, 9, 4
    q = torch.randn(1, T, H, 64).permute(0, 2, 1, 3)                 # the reference's _transpose_4d view
    k, v = torch.randn(1, H, T, 64), torch.randn(1, H, T, 64)
    pk, pq = torch.randn(1, H, T, 2 * S), torch.randn(1, H, T, 2 * S)
    with g.packed_batch(_positions([3, 2, 4])) as batch:
        out = deb_mod.flash_deberta_attention(q, k, v, torch.tensor([T], dtype=torch.int32), pk, pq, False, 0.1,
                                              S, 8, True)
    (args, kwargs), = spy.calls
    assert args[0].shape == (T, H, 64) and args[0].data_ptr() == q.data_ptr()
    assert torch.equal(args[0], q[0].transpose(0, 1))
    assert args[3] is batch.cu_seqlens and args[4] == 4
    assert torch.equal(args[5], pk[0].transpose(0, 1)) and torch.equal(args[6], pq[0].transpose(0, 1))
    assert args[7:] == (False, 0.1, S, 8, True)
    assert kwargs == {"rel_key": None, "rel_query": None}
    assert out.shape == (1, H, T, 64) and bool((out == 7.0).all())


def test_deberta_fused_flat_call_keeps_the_tables(monkeypatch):
    spy = _Spy()
    monkeypatch.setattr(deb_mod, "flash_deberta_attention_varlen", spy)
    H, T = 2, 5
    q = torch.randn(1, H, T, 64)
    rk, rq = torch.randn(1, H, 8, 64), torch.randn(1, H, 8, 64)
    with g.packed_batch(_positions([2, 3])):
        deb_mod.flash_deberta_attention(q, q, q, None, rel_key=rk, rel_query=rq, position_buckets=4)
    (args, kwargs), = spy.calls
    assert args[5] is None and args[6] is None
    assert kwargs["rel_key"] is rk and kwargs["rel_query"] is rq


def test_rpb_flat_call_goes_to_the_packed_operator(monkeypatch):
    spy = _Spy()
    monkeypatch.setattr(rpb_mod, "flash_attention_rpb_varlen", spy)
    H, T = 2, 6
    q = torch.randn(1, H, T, 64)
    table = torch.randn(32, H)
    mask = torch.zeros(1, 1, 1, T)
    with g.packed_batch(_positions([4, 2])) as batch:
        out = rpb_mod.flash_attention_rpb_final(q, q, q, table, 32, 128, False, padding_mask=mask)
        with pytest.raises(ValueError, match="dropout"):
            rpb_mod.flash_attention_rpb_final(q, q, q, table, 32, 128, False, dropout_p=0.1)
    (args, kwargs), = spy.calls
    assert args[0].shape == (T, H, 64) and args[3] is batch.cu_seqlens and args[4] == 4
    assert args[5] is table and args[6:] == (32, 128, False, 1.0)
    assert out.shape == (1, H, T, 64)


def test_install_fused_positions_is_idempotent():
    class Layer:
        def _flash_forward(self, *a):
            return "reference"
    original = Layer._flash_forward
    g.install_fused_positions(Layer)
    g.install_fused_positions(Layer)
    assert Layer._flash_forward is g.deberta_v2_flash_forward
    assert Layer._vf_reference_flash_forward is original


def test_fused_forward_keeps_the_reference_method_without_both_terms():
    class Layer:
        pos_att_type = ["c2p"]

        def _vf_reference_flash_forward(self, *a):
            return ("reference", a)
    assert g.deberta_v2_flash_forward(Layer(), 1, 2, 3, 4, 5) == ("reference", (1, 2, 3, 4, 5))
