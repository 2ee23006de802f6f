"""The fused DeBERTa entry points' argument rules (include/vf_b200.h): checks that fire on the
host before any CUDA call, with fake device addresses, so they run without a GPU."""
import ctypes

import pytest

from vf_b200 import _lib

H, L, S = 2, 256, 256


def view(data, size, stride):
    t = _lib.Tensor4d()
    t.data = data
    for i in range(4):
        t.size[i] = size[i]
        t.stride[i] = stride[i]
    return t


def contig(data, size):
    st = [size[1] * size[2] * size[3], size[2] * size[3], size[3], 1]
    return view(data, size, st)


def args(**kw):
    a = _lib.DebertaFusedArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    a.q = contig(0x100000, (1, H, L, 64))
    a.k = contig(0x200000, (1, H, L, 64))
    a.v = contig(0x300000, (1, H, L, 64))
    a.out = contig(0x400000, (1, H, L, 64))
    a.rel_key = contig(0x500000, (1, H, 2 * S, 64))
    a.rel_query = contig(0x600000, (1, H, 2 * S, 64))
    a.has_sm_scale = 1
    a.sm_scale = 0.07
    a.position_buckets = S
    a.max_relative_distance = 512
    a.use_log_bucket = 1
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def ws_bytes(b=1, h=H, m=L, n=L):
    return _lib.load().vf_deberta_fused_workspace_bytes(b, h, m, n)


def call(a, ws=0x10000000, nbytes=None):
    lib = _lib.load()
    if nbytes is None:
        nbytes = ws_bytes(a.q.size[0], a.q.size[1], a.q.size[2], a.k.size[2])
    return lib.vf_deberta_attention_fused_fwd(ctypes.byref(a), ctypes.c_void_p(ws), nbytes, None)


def test_workspace_size_formula():
    # 2 expanded tables of H x (ceil128(M) + ceil128(N)) rows x 64 x 2 bytes, plus the unit
    # order (4 bytes per (batch row, 128-row query block)), each rounded up to 256 bytes
    assert ws_bytes(8, 16, 512, 512) == 2 * 16 * 1024 * 128 + 256
    assert ws_bytes(3, 2, 200, 300) == 2 * (2 * (256 + 384) * 128) + 256
    assert ws_bytes(-1, 2, 3, 4) == _lib.VF_EINVAL


@pytest.mark.parametrize("kw,code,msg", [
    (dict(rel_key=contig(0x500000, (2, H, 2 * S, 64))), _lib.VF_EUNSUPPORTED, "shared by the batch"),
    (dict(rel_key=contig(0x500000, (1, H + 1, 2 * S, 64))), _lib.VF_EINVAL, "rel_key must be"),
    (dict(rel_query=contig(0x600000, (1, H, 2 * S - 2, 64))), _lib.VF_EINVAL, "rel_query must be"),
    (dict(rel_key=view(0x500008, (1, H, 2 * S, 64), (H * 2 * S * 64, 2 * S * 64, 64, 1))), _lib.VF_EINVAL,
     "16-byte aligned"),
    (dict(dtype=_lib.VF_DTYPE_F32), _lib.VF_EUNSUPPORTED, "dtype"),
    (dict(position_buckets=0, max_relative_distance=0), _lib.VF_EINVAL, "position_buckets"),
    (dict(position_buckets=256, max_relative_distance=100), _lib.VF_EUNSUPPORTED, "log-bucket"),
])
def test_fused_validation_rejects_before_launch(kw, code, msg):
    assert call(args(**kw)) == code
    assert msg in _lib.load().vf_last_error().decode()


def test_fused_workspace_rules():
    lib = _lib.load()
    assert call(args(), ws=0) == _lib.VF_EINVAL
    assert "workspace" in lib.vf_last_error().decode()
    assert call(args(), ws=0x10000010) == _lib.VF_EINVAL          # not 256-byte aligned
    assert call(args(), nbytes=ws_bytes() - 1) == _lib.VF_EINVAL
    assert "too small" in lib.vf_last_error().decode()
    assert lib.vf_deberta_attention_fused_fwd(None, None, 0, None) == _lib.VF_EINVAL


def test_fused_varlen_rules():
    lib = _lib.load()
    a = args(seq_lengths=0x700000)
    cu = ctypes.c_void_p(0x800000)
    assert lib.vf_deberta_attention_fused_varlen_fwd(ctypes.byref(a), cu, 1, L, ctypes.c_void_p(0x10000000),
                                                     ws_bytes(1, H, L, L), None) == _lib.VF_EUNSUPPORTED
    assert "seq_lengths" in lib.vf_last_error().decode()
    a = args()
    assert lib.vf_deberta_attention_fused_varlen_fwd(ctypes.byref(a), cu, 0, L, ctypes.c_void_p(0x10000000),
                                                     ws_bytes(1, H, L, L), None) == _lib.VF_EINVAL


def test_fused_sequence_limit():
    big = 65536 + 128
    a = args(q=contig(0x100000, (1, H, big, 64)), k=contig(0x200000, (1, H, big, 64)),
             v=contig(0x300000, (1, H, big, 64)), out=contig(0x400000, (1, H, big, 64)))
    assert call(a) == _lib.VF_EUNSUPPORTED
    assert "65536" in _lib.load().vf_last_error().decode()
