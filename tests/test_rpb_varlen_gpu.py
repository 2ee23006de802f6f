"""GPU parity of the packed variable-length T5-RPB op (kernels.flash_attention_rpb
.flash_attention_rpb_varlen -> vf_rpb_attention_varlen_fwd) against the CPU oracle (each
cu_seqlens sequence alone, fp64).  Gates: max-abs <= 2e-2 and per-row cosine >= 0.9999."""
import ctypes

import pytest
import torch

import oracle
from _util import assert_close

pytestmark = pytest.mark.gpu


def _op():
    from kernels.flash_attention_rpb import flash_attention_rpb_varlen
    return flash_attention_rpb_varlen


def make_packed(lens, H=2, dtype=torch.bfloat16, nb=32, seed=0, lead=0, tail=0):
    g = torch.Generator().manual_seed(seed)
    total = lead + sum(lens) + tail
    # q at half scale: scores of std ~4 at softmax_scale 1.0.  With unit q and k (std 8) the
    # softmax is nearly one-hot and bf16 rounding of P and O alone reaches the 2e-2 gate
    # over a few thousand rows (seen at 3 x 768: 2.2e-2 with cosine 0.999993).
    q, k, v = (torch.randn(total, H, 64, generator=g) for _ in range(3))
    q, k, v = (0.5 * q).to(dtype), k.to(dtype), v.to(dtype)
    table = (torch.randn(nb, H, generator=g) * 2.0).to(dtype)
    cu = torch.tensor([lead] + [lead + int(x) for x in torch.cumsum(torch.tensor(lens), 0)], dtype=torch.int32)
    return q, k, v, table, cu


def run_check(lens, H=2, dtype=torch.bfloat16, nb=32, md=128, is_decoder=False, scale=1.0, table=True, seed=0,
              what=""):
    q, k, v, t, cu = make_packed(lens, H, dtype, nb, seed)
    dev = torch.device("cuda")
    out = _op()(q.to(dev), k.to(dev), v.to(dev), cu.to(dev), max(max(lens), 1), t.to(dev) if table else None,
                nb, md, is_decoder, scale)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = oracle.rpb_attention_varlen_ref(q.float(), k.float(), v.float(), cu, t.float() if table else None, nb, md,
                                          is_decoder, scale)
    assert torch.isfinite(out.float()).all(), f"{what}: non-finite output"
    return assert_close(out, ref, None, what=what)


@pytest.mark.parametrize("lens", [
    [1], [128], [129], [1, 127, 128, 129, 255, 256, 257, 700], [768] * 3, [5, 300, 17, 513],
])
def test_varlen_lengths(lens):
    run_check(lens, seed=len(lens) + lens[0], what=f"lens={lens}")


def test_varlen_empty_sequences_between():
    run_check([0, 50, 0, 300, 0, 1, 0], what="empty sequences")


def test_varlen_fp16_scale_no_table():
    run_check([200, 333, 64], dtype=torch.float16, scale=0.125, table=False, what="fp16 no table")


def test_varlen_decoder_causal():
    run_check([300, 1, 129, 256], is_decoder=True, what="decoder")


def test_varlen_other_bucket_config_more_heads():
    run_check([700, 90], H=4, nb=64, md=256, what="64/256, 4 heads")


def test_varlen_many_short_sequences_natural_order():
    # 1500 sequences: more (sequence, query block) pairs than the cost-ordering table holds.
    lens = [1 + (37 * b) % 64 for b in range(1500)]
    run_check(lens, H=1, seed=5, what="1500 sequences")


def test_varlen_matches_padded_op_on_c2():
    """C2 (16 x 768, lengths U[256, 768]) packed vs. padded + additive mask: the same
    attention; both GPU outputs must meet the gate against each other, and two sequences
    against the oracle."""
    from kernels.flash_attention_rpb import flash_attention_rpb_final
    from vf_b200.workloads import mt5_attention_inputs, mt5_varlen_inputs
    w = mt5_attention_inputs(seed=0, device="cuda")
    p = mt5_varlen_inputs(seed=0, device="cuda")
    pad = flash_attention_rpb_final(w["q"], w["k"], w["v"], w["rpb_table"], 32, 128, False, w["padding_mask"], 0.0, 1.0)
    out = _op()(p["q"], p["k"], p["v"], p["cu_seqlens"], p["max_seqlen"], p["rpb_table"], 32, 128)
    lens = [int(x) for x in w["lengths"].tolist()]
    want = torch.cat([pad[b, :, :n].permute(1, 0, 2) for b, n in enumerate(lens)], 0)
    err, _ = assert_close(out, want.float(), None, what="packed vs padded")
    print(f"packed vs padded C2: max_abs {err:.3e}")
    cu = p["cu_seqlens"].cpu()
    for b in (0, 9):
        a, e = int(cu[b]), int(cu[b + 1])
        sub = [0, e - a]
        ref = oracle.rpb_attention_varlen_ref(p["q"][a:e].float().cpu(), p["k"][a:e].float().cpu(),
                                              p["v"][a:e].float().cpu(), sub, p["rpb_table"].float().cpu(), 32, 128,
                                              False)
        assert_close(out[a:e], ref, None, what=f"C2 packed sequence {b}")


def test_varlen_strided_views_from_packed_qkv():
    # q, k, v as slices of one [total, 3, H, 64] projection (row stride 3*H*64).
    lens = [100, 257, 31]
    H = 4
    g = torch.Generator().manual_seed(9)
    total = sum(lens)
    qkv = torch.randn(total, 3, H, 64, generator=g).to(torch.bfloat16)
    t = torch.randn(32, H, generator=g).to(torch.bfloat16)
    cu = torch.tensor([0, 100, 357, 388], dtype=torch.int32)
    d = qkv.cuda()
    out = _op()(d[:, 0], d[:, 1], d[:, 2], cu.cuda(), 257, t.cuda(), 32, 128)
    ref = oracle.rpb_attention_varlen_ref(qkv[:, 0].float(), qkv[:, 1].float(), qkv[:, 2].float(), cu, t.float(),
                                          32, 128, False)
    assert_close(out, ref, None, what="strided qkv views")


def test_varlen_fp32_inputs():
    q, k, v, t, cu = make_packed([300, 170], dtype=torch.float32, seed=21)
    out = _op()(q.cuda(), k.cuda(), v.cuda(), cu.cuda(), 300, t.cuda(), 32, 128, False, 0.125)
    torch.cuda.synchronize()
    assert out.dtype == torch.float32
    ref = oracle.rpb_attention_varlen_ref(q, k, v, cu, t, 32, 128, False, 0.125)
    assert_close(out, ref, None, max_abs=2e-3, min_cos=0.99999, what="fp32 packed")


def _t4(x):
    # [total, H, 64] -> (1, H, total, 64) view for the C ABI
    from vf_b200 import _lib
    d = _lib.Tensor4d()
    d.data = x.data_ptr()
    for i, (sz, st) in enumerate(((1, x.shape[0] * x.stride(0)), (x.shape[1], x.stride(1)),
                                  (x.shape[0], x.stride(0)), (x.shape[2], x.stride(2)))):
        d.size[i] = sz
        d.stride[i] = st
    return d


def _abi_call(q, k, v, out, table, cu, num_seqs, max_seqlen):
    from vf_b200 import _lib
    lib = _lib.load()
    a = _lib.RpbArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    a.q, a.k, a.v, a.out = _t4(q), _t4(k), _t4(v), _t4(out)
    a.rpb_table = table.data_ptr()
    a.table_rows, a.table_cols = table.shape
    a.table_stride_row, a.table_stride_col = table.stride()
    a.table_dtype = _lib.VF_DTYPE_BF16
    a.num_buckets, a.max_distance, a.is_decoder = 32, 128, 0
    a.softmax_scale = 1.0
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.vf_rpb_attention_varlen_fwd(ctypes.byref(a), ctypes.c_void_p(cu.data_ptr()), num_seqs, max_seqlen,
                                         ctypes.c_void_p(stream))
    assert rc == 0, lib.vf_last_error().decode()


def test_varlen_c_abi_leaves_rows_outside_sequences():
    """Through the C ABI: sequences start at row 3 and end 5 rows before the end; rows
    outside them keep what the caller put there."""
    lens = [130, 1, 200]
    q, k, v, t, cu = make_packed(lens, H=2, seed=4, lead=3, tail=5)
    dq, dk, dv, dt, dcu = q.cuda(), k.cuda(), v.cuda(), t.cuda(), cu.cuda()
    out = torch.full_like(dq, 7.0)
    _abi_call(dq, dk, dv, out, dt, dcu, len(lens), 200)
    torch.cuda.synchronize()
    o = out.cpu()
    assert torch.all(o[:3] == 7.0) and torch.all(o[-5:] == 7.0)
    ref = oracle.rpb_attention_varlen_ref(q.float(), k.float(), v.float(), cu, t.float(), 32, 128, False)
    assert_close(o[3:-5], ref[3:-5], None, what="C ABI packed rows")


def test_varlen_bad_offsets_set_error_bit_and_stay_in_bounds():
    """A sequence longer than max_seqlen and decreasing offsets set bit 2 of the device error
    word; the rows used are clamped into the views (nothing outside them is written)."""
    import vf_b200
    lens = [100, 60]
    q, k, v, t, cu = make_packed(lens, H=2, seed=6, tail=8)
    dq, dk, dv, dt = q.cuda(), k.cuda(), v.cuda(), t.cuda()
    vf_b200.device_error(clear=True)
    out = torch.full_like(dq, 7.0)
    _abi_call(dq, dk, dv, out, dt, cu.cuda(), 2, 64)             # 100 > max_seqlen 64
    assert vf_b200.device_error(clear=True) & 4
    assert torch.all(out[-8:].cpu() == 7.0)
    bad = torch.tensor([100, 40, 160], dtype=torch.int32)         # decreasing
    out2 = torch.full_like(dq, 7.0)
    _abi_call(dq, dk, dv, out2, dt, bad.cuda(), 2, 100)
    assert vf_b200.device_error(clear=True) & 4
    o2 = out2.cpu()
    assert torch.all(o2[:40] == 7.0) and torch.all(o2[-8:] == 7.0)


def test_varlen_repeat_is_deterministic():
    q, k, v, t, cu = make_packed([300, 200, 5], seed=13)
    args = (q.cuda(), k.cuda(), v.cuda(), cu.cuda(), 300, t.cuda(), 32, 128)
    a = _op()(*args)
    b = _op()(*args)
    assert torch.equal(a, b)
