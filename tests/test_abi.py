"""The C ABI library: loads, exports every symbol include/vf_b200.h declares, host-side
bucket functions are bit-exact with the reference, and argument validation rejects bad
inputs before any GPU work (no compute call is made here)."""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import golden_inputs as gi
from vf_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "vf_b200.h"
G = np.load(Path(gi.__file__).with_name("golden.npz"))


def header_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vf_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    declared = header_functions()
    assert declared, "no functions parsed from the header"
    missing = [name for name in declared if not hasattr(lib, name)]
    assert not missing, f"declared but not exported: {missing}"
    assert set(declared) == set(_lib.EXPORTED_SYMBOLS)
    assert lib.vf_abi_version() == _lib.ABI_VERSION


def test_struct_sizes_match_c_layout():
    # 8-byte pointer + 2 x 4 int64
    assert ctypes.sizeof(_lib.Tensor4d) == 72
    assert ctypes.sizeof(_lib.RpbArgs) % 8 == 0
    assert ctypes.sizeof(_lib.DebertaArgs) % 8 == 0


@pytest.mark.parametrize("bs,mp", gi.DEBERTA_BUCKET_CONFIGS)
def test_c_deberta_bucket_matches_reference(bs, mp):
    ours = np.array(_lib.deberta_log_bucket(bs, mp, -gi.R_SWEEP, gi.R_SWEEP))
    assert np.array_equal(ours, G[f"deberta_bucket_{bs}_{mp}"].astype(np.int64))


@pytest.mark.parametrize("nb,md,bidir", gi.T5_BUCKET_CONFIGS)
def test_c_t5_bucket_matches_reference(nb, md, bidir):
    ours = np.array(_lib.t5_relative_bucket(nb, md, bidir, -gi.R_SWEEP, gi.R_SWEEP))
    assert np.array_equal(ours, G[f"t5_bucket_{nb}_{md}_{int(bidir)}"].astype(np.int64))


def test_bucket_domain_errors():
    with pytest.raises(_lib.VfError):
        _lib.t5_relative_bucket(2, 128, True, 0, 4)      # max_exact == 0
    with pytest.raises(_lib.VfError):
        _lib.deberta_log_bucket(256, 100, 0, 4)          # log of a ratio < 1


def _fake_t4(shape, ptr=0x10000):
    t = _lib.Tensor4d()
    t.data = ptr
    strides = [shape[1] * shape[2] * shape[3], shape[2] * shape[3], shape[3], 1]
    for i in range(4):
        t.size[i] = shape[i]
        t.stride[i] = strides[i]
    return t


def _rpb_args(D=64, dtype=_lib.VF_DTYPE_BF16, dropout=0.0):
    a = _lib.RpbArgs()
    a.dtype = dtype
    shape = (2, 4, 256, D)
    a.q, a.k, a.v, a.out = (_fake_t4(shape, 0x10000 * (i + 1)) for i in range(4))
    a.num_buckets, a.max_distance = 32, 128
    a.dropout_p = dropout
    a.softmax_scale = 1.0
    return a


@pytest.mark.parametrize("kwargs,code", [
    (dict(D=128), _lib.VF_EUNSUPPORTED),
    (dict(dtype=_lib.VF_DTYPE_F32), _lib.VF_EUNSUPPORTED),
    (dict(dropout=0.1), _lib.VF_EUNSUPPORTED),
])
def test_rpb_validation_rejects_before_launch(kwargs, code):
    lib = _lib.load()
    rc = lib.vf_rpb_attention_fwd(ctypes.byref(_rpb_args(**kwargs)), None)
    assert rc == code
    assert lib.vf_last_error().decode()


@pytest.mark.parametrize("mshape,msg", [((2, 1, 7, 256), "query dim"), ((2, 1, 256, 255), "last dim"),
                                         ((3, 1, 256, 256), "batch dim"), ((2, 3, 1, 256), "head dim")])
def test_rpb_mask_shapes_rejected_before_launch(mshape, msg):
    """A padding mask broadcasts over (B|1, H|1, 1|M, N); other shapes fail before any launch."""
    lib = _lib.load()
    a = _rpb_args()
    a.padding_mask = _fake_t4(mshape, 0x80000)
    a.mask_dtype = _lib.VF_DTYPE_BF16
    assert lib.vf_rpb_attention_fwd(ctypes.byref(a), None) == _lib.VF_EINVAL
    assert msg in lib.vf_last_error().decode()


def test_rpb_null_and_shape_mismatch():
    lib = _lib.load()
    assert lib.vf_rpb_attention_fwd(None, None) == _lib.VF_EINVAL
    a = _rpb_args()
    a.k.size[1] = 3
    assert lib.vf_rpb_attention_fwd(ctypes.byref(a), None) == _lib.VF_EINVAL
    assert "batch and heads" in lib.vf_last_error().decode()


def test_deberta_validation_rejects_before_launch():
    lib = _lib.load()
    a = _lib.DebertaArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    shape = (2, 4, 256, 64)
    a.q, a.k, a.v, a.out = (_fake_t4(shape, 0x10000 * (i + 1)) for i in range(4))
    a.pos_key = _fake_t4((2, 4, 256, 512), 0x90000)
    a.position_buckets = 0
    a.max_relative_distance = 0
    assert lib.vf_deberta_attention_fwd(ctypes.byref(a), None) == _lib.VF_EINVAL
    assert "position" in lib.vf_last_error().decode()


def _varlen_args(total=300, H=4):
    a = _rpb_args()
    a.q, a.k, a.v, a.out = (_fake_t4((1, H, total, 64), 0x10000 * (i + 1)) for i in range(4))
    return a


@pytest.mark.parametrize("mutate,cu,num_seqs,max_seqlen,code,msg", [
    (None, None, 2, 100, _lib.VF_EINVAL, "cu_seqlens"),
    (None, 0x20003, 2, 100, _lib.VF_EINVAL, "cu_seqlens"),          # misaligned
    (None, 0x20000, 0, 100, _lib.VF_EINVAL, "num_seqs"),
    (None, 0x20000, 2, 0, _lib.VF_EINVAL, "max_seqlen"),
    (None, 0x20000, 2, 301, _lib.VF_EINVAL, "max_seqlen"),
    ("batch2", 0x20000, 2, 100, _lib.VF_EINVAL, "packed views"),
    ("k_rows", 0x20000, 2, 100, _lib.VF_EINVAL, "packed rows"),
    ("mask", 0x20000, 2, 100, _lib.VF_EUNSUPPORTED, "padding_mask"),
])
def test_rpb_varlen_validation_rejects_before_launch(mutate, cu, num_seqs, max_seqlen, code, msg):
    lib = _lib.load()
    a = _varlen_args()
    if mutate == "batch2":
        a.q.size[0] = 2
    elif mutate == "k_rows":
        a.k.size[2] = 299
    elif mutate == "mask":
        a.padding_mask = _fake_t4((1, 1, 1, 300), 0x80000)
    rc = lib.vf_rpb_attention_varlen_fwd(ctypes.byref(a), cu, num_seqs, max_seqlen, None)
    assert rc == code
    assert msg in lib.vf_last_error().decode()


def test_deberta_varlen_validation_rejects_before_launch():
    lib = _lib.load()
    a = _lib.DebertaArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    a.q, a.k, a.v, a.out = (_fake_t4((1, 4, 300, 64), 0x10000 * (i + 1)) for i in range(4))
    a.position_buckets, a.max_relative_distance = 256, 512
    a.seq_lengths = 0x30000
    assert lib.vf_deberta_attention_varlen_fwd(ctypes.byref(a), 0x20000, 2, 100, None) == _lib.VF_EUNSUPPORTED
    assert "seq_lengths" in lib.vf_last_error().decode()
    a.seq_lengths = None
    assert lib.vf_deberta_attention_varlen_fwd(ctypes.byref(a), None, 2, 100, None) == _lib.VF_EINVAL
    assert lib.vf_deberta_attention_varlen_fwd(ctypes.byref(a), 0x20000, 2, 301, None) == _lib.VF_EINVAL
    assert "max_seqlen" in lib.vf_last_error().decode()


def test_deberta_position_strides_beyond_32_bit_offsets_rejected():
    """The gathers use 32-bit offsets inside a key tile; views whose strides could overflow
    them are refused before any launch."""
    lib = _lib.load()
    a = _lib.DebertaArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    shape = (2, 4, 256, 64)
    a.q, a.k, a.v, a.out = (_fake_t4(shape, 0x10000 * (i + 1)) for i in range(4))
    a.position_buckets, a.max_relative_distance, a.use_log_bucket = 256, 512, 1
    a.pos_query = _fake_t4((2, 4, 256, 512), 0x90000)
    a.pos_query.stride[2] = 1 << 25            # 127 * 2^25 > 2^31
    assert lib.vf_deberta_attention_fwd(ctypes.byref(a), None) == _lib.VF_EUNSUPPORTED
    assert "32-bit" in lib.vf_last_error().decode()
    a.pos_query = _lib.Tensor4d()
    a.pos_key = _fake_t4((2, 4, 256, 512), 0x90000)
    a.pos_key.stride[3] = 1 << 23              # 511 * 2^23 > 2^31
    assert lib.vf_deberta_attention_fwd(ctypes.byref(a), None) == _lib.VF_EUNSUPPORTED
