"""GPU parity of the packed variable-length DeBERTa op (kernels.flash_deberta_attention
.flash_deberta_attention_varlen -> vf_deberta_attention_varlen_fwd) against the CPU oracle
(each cu_seqlens sequence alone, fp64).  Gates: max-abs <= 2e-2 and per-row cosine >= 0.9999."""
import ctypes
import math

import pytest
import torch

import oracle
from _util import assert_close

pytestmark = pytest.mark.gpu

V3 = dict(pb=256, mr=512, log=True)


def _op():
    from kernels.flash_deberta_attention import flash_deberta_attention_varlen
    return flash_deberta_attention_varlen


def make_packed(lens, H=2, S=256, dtype=torch.bfloat16, seed=0, lead=0, tail=0, c2p=True, p2c=True):
    g = torch.Generator().manual_seed(seed)
    total = lead + sum(lens) + tail
    q, k, v = (torch.randn(total, H, 64, generator=g).to(dtype) for _ in range(3))
    pk = (torch.randn(total, H, 2 * S, generator=g) * 3).to(dtype) if c2p else None
    pq = (torch.randn(total, H, 2 * S, generator=g) * 3).to(dtype) if p2c else None
    cu = torch.tensor([lead] + [lead + int(x) for x in torch.cumsum(torch.tensor(lens), 0)], dtype=torch.int32)
    return q, k, v, pk, pq, cu


def run_check(lens, H=2, S=256, pb=256, mr=512, log=True, causal=False, sm_scale=1 / math.sqrt(64 * 3),
              dtype=torch.bfloat16, seed=0, c2p=True, p2c=True, what=""):
    q, k, v, pk, pq, cu = make_packed(lens, H, S, dtype, seed, c2p=c2p, p2c=p2c)
    d = lambda t: None if t is None else t.cuda()
    f = lambda t: None if t is None else t.float()
    out = _op()(d(q), d(k), d(v), cu.cuda(), max(max(lens), 1), d(pk), d(pq), causal, sm_scale, pb, mr, log)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = oracle.deberta_attention_varlen_ref(f(q), f(k), f(v), cu, f(pk), f(pq), causal, sm_scale, pb, mr, log)
    valid = torch.zeros(q.shape[0], dtype=torch.bool)
    for a, b in zip(cu[:-1].tolist(), cu[1:].tolist()):
        valid[a:b] = True
    assert torch.isfinite(out.float()[valid]).all(), f"{what}: non-finite output"
    return assert_close(out[valid], ref[valid], None, what=what)


@pytest.mark.parametrize("lens", [[1], [128], [129], [1, 63, 128, 129, 255, 256, 257, 512], [512] * 3, [5, 300, 17]])
def test_deberta_varlen_lengths(lens):
    run_check(lens, seed=len(lens) + lens[0], what=f"lens={lens}")


def test_deberta_varlen_empty_sequences_between():
    run_check([0, 50, 0, 300, 0, 1, 0], what="empty sequences")


def test_deberta_varlen_long_sequence_saturated():
    run_check([1100, 37], what="L=1100")


def test_deberta_varlen_v1_linear_positions():
    run_check([300, 150], S=300, pb=300, mr=512, log=False, what="v1 linear")


@pytest.mark.parametrize("c2p,p2c", [(True, False), (False, True), (False, False)])
def test_deberta_varlen_partial_terms(c2p, p2c):
    run_check([192, 90], S=64, pb=64, mr=128, sm_scale=None, c2p=c2p, p2c=p2c, what=f"c2p={c2p} p2c={p2c}")


def test_deberta_varlen_causal_fp16():
    run_check([300, 1, 129], dtype=torch.float16, causal=True, what="causal fp16")


def test_deberta_varlen_many_short_sequences_natural_order():
    lens = [1 + (37 * b) % 64 for b in range(1500)]
    run_check(lens, H=1, S=32, pb=32, mr=64, seed=5, what="1500 sequences")


def test_deberta_varlen_matches_padded_op_on_c1():
    """C1 (8 x 512, lengths U[64, 512]) packed vs. padded with seq_lengths: both GPU outputs
    meet the gate against each other on the valid rows."""
    from kernels.flash_deberta_attention import flash_deberta_attention
    from vf_b200.workloads import deberta_attention_inputs
    w = deberta_attention_inputs(seed=0, device="cuda")
    lens = [int(x) for x in w["lengths"].tolist()]
    pad = flash_deberta_attention(w["q"], w["k"], w["v"], w["seq_lengths"], w["pos_key"], w["pos_query"], False,
                                  w["sm_scale"], 256, 512, True)
    pack = lambda x: torch.cat([x[b, :, :n].permute(1, 0, 2) for b, n in enumerate(lens)], 0)
    cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0).tolist()), dtype=torch.int32, device="cuda")
    out = _op()(pack(w["q"]), pack(w["k"]), pack(w["v"]), cu, max(lens), pack(w["pos_key"]), pack(w["pos_query"]),
                False, w["sm_scale"], 256, 512, True)
    err, _ = assert_close(out, pack(pad).float(), None, what="packed vs padded C1")
    print(f"packed vs padded C1: max_abs {err:.3e}")


def test_deberta_varlen_fp32_inputs():
    q, k, v, pk, pq, cu = make_packed([300, 170], dtype=torch.float32, seed=21)
    sm = 1 / math.sqrt(64 * 3)
    out = _op()(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), 300, pk.cuda(), pq.cuda(), False, sm, 256, 512, True)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    ref = oracle.deberta_attention_varlen_ref(q, k, v, cu, pk, pq, False, sm, 256, 512, True)
    assert_close(out, ref, None, max_abs=2e-3, min_cos=0.99999, what="fp32 packed")


def _t4(x):
    from vf_b200 import _lib
    d = _lib.Tensor4d()
    d.data = x.data_ptr()
    for i, (sz, st) in enumerate(((1, x.shape[0] * x.stride(0)), (x.shape[1], x.stride(1)),
                                  (x.shape[0], x.stride(0)), (x.shape[2], x.stride(2)))):
        d.size[i] = sz
        d.stride[i] = st
    return d


def _abi_call(q, k, v, out, pk, pq, cu, num_seqs, max_seqlen, sm_scale):
    from vf_b200 import _lib
    lib = _lib.load()
    a = _lib.DebertaArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    a.q, a.k, a.v, a.out = _t4(q), _t4(k), _t4(v), _t4(out)
    a.pos_key, a.pos_query = _t4(pk), _t4(pq)
    a.causal = 0
    a.has_sm_scale, a.sm_scale = 1, sm_scale
    a.position_buckets, a.max_relative_distance, a.use_log_bucket = 256, 512, 1
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.vf_deberta_attention_varlen_fwd(ctypes.byref(a), ctypes.c_void_p(cu.data_ptr()), num_seqs,
                                             max_seqlen, ctypes.c_void_p(stream))
    assert rc == 0, lib.vf_last_error().decode()


def test_deberta_varlen_c_abi_leaves_rows_outside_sequences():
    lens = [130, 1, 200]
    q, k, v, pk, pq, cu = make_packed(lens, seed=4, lead=3, tail=5)
    dq, dk, dv, dpk, dpq = q.cuda(), k.cuda(), v.cuda(), pk.cuda(), pq.cuda()
    out = torch.full_like(dq, 7.0)
    sm = 1 / math.sqrt(64 * 3)
    _abi_call(dq, dk, dv, out, dpk, dpq, cu.cuda(), len(lens), 200, sm)
    torch.cuda.synchronize()
    o = out.cpu()
    assert torch.all(o[:3] == 7.0) and torch.all(o[-5:] == 7.0)
    ref = oracle.deberta_attention_varlen_ref(q.float(), k.float(), v.float(), cu, pk.float(), pq.float(), False,
                                              sm, 256, 512, True)
    assert_close(o[3:-5], ref[3:-5], None, what="C ABI packed rows")


def test_deberta_varlen_bad_offsets_set_error_bit_and_stay_in_bounds():
    import vf_b200
    lens = [100, 60]
    q, k, v, pk, pq, cu = make_packed(lens, seed=6, tail=8)
    dq, dk, dv, dpk, dpq = q.cuda(), k.cuda(), v.cuda(), pk.cuda(), pq.cuda()
    vf_b200.device_error(clear=True)
    out = torch.full_like(dq, 7.0)
    _abi_call(dq, dk, dv, out, dpk, dpq, cu.cuda(), 2, 64, 0.1)        # 100 > max_seqlen 64
    assert vf_b200.device_error(clear=True) & 4
    assert torch.all(out[-8:].cpu() == 7.0)
    bad = torch.tensor([100, 40, 160], dtype=torch.int32)           # decreasing
    out2 = torch.full_like(dq, 7.0)
    _abi_call(dq, dk, dv, out2, dpk, dpq, bad.cuda(), 2, 100, 0.1)
    assert vf_b200.device_error(clear=True) & 4
    o2 = out2.cpu()
    assert torch.all(o2[:40] == 7.0) and torch.all(o2[-8:] == 7.0)
