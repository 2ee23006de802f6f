"""The gated feed-forward activation on the CPU: the oracle pinned to the reference's own
unfused path (models/mt5/mt5_encoder.py:427-437: F.gelu / F.relu / F.silu then `* up`),
the C-ABI's argument checks (no launch), and the drop-in's inference-only contract."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

import oracle
from vf_b200 import _lib

FALLBACK = {
    0: lambda g: F.gelu(g, approximate="tanh"),
    1: lambda g: F.gelu(g, approximate="none"),
    2: F.relu,
    3: F.silu,
}


@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_oracle_matches_reference_fallback_fp32(act):
    g = torch.Generator().manual_seed(act)
    gate, up = torch.randn(64, 300, generator=g) * 3, torch.randn(64, 300, generator=g)
    torch.testing.assert_close(oracle.gated_act_ref(gate, up, act), FALLBACK[act](gate) * up, rtol=2e-6, atol=1e-5)


def test_act_name_map_matches_reference():
    from kernels.ff_fused import _act_type_map
    for name, code in (("gelu", 0), ("gelu_new", 0), ("gelu_fast", 0), ("gelu_pytorch_tanh", 0),
                       ("gelu_accurate", 1), ("relu", 2), ("silu", 3), ("swish", 3), ("unknown", 0), ("GELU_NEW", 0)):
        assert _act_type_map(name) == code


def test_dropout_in_training_is_refused():
    from kernels.ff_fused import fused_gelu_mul_dropout
    x = torch.zeros(2, 8)
    with pytest.raises(NotImplementedError):
        fused_gelu_mul_dropout(x, x, "gelu", dropout_p=0.1, training=True)


def _args(**kw):
    a = _lib.GatedActArgs()
    a.dtype, a.gate, a.up, a.out = _lib.VF_DTYPE_BF16, 0x10000, 0x20000, 0x30000
    a.rows, a.cols = 4, 64
    a.gate_row_stride = a.up_row_stride = a.out_row_stride = 64
    a.act = 0
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code,msg", [
    (dict(act=7), _lib.VF_EINVAL, "activation"),
    (dict(rows=-1), _lib.VF_EINVAL, "negative"),
    (dict(gate=None), _lib.VF_EINVAL, "non-null"),
    (dict(up_row_stride=32), _lib.VF_EINVAL, "row strides"),
    (dict(dtype=9), _lib.VF_EUNSUPPORTED, "dtype"),
])
def test_gated_act_validation_rejects_before_launch(kw, code, msg):
    lib = _lib.load()
    assert lib.vf_gated_act_fwd(ctypes.byref(_args(**kw)), None) == code
    assert msg in lib.vf_last_error().decode()


def test_gated_act_empty_is_a_no_op():
    lib = _lib.load()
    assert lib.vf_gated_act_fwd(ctypes.byref(_args(rows=0)), None) == _lib.VF_OK
    assert lib.vf_gated_act_fwd(None, None) == _lib.VF_EINVAL


@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_oracle_without_up_is_the_activation(act):
    """up = None: the plain activation (the DeBERTa feed-forward uses the exact GELU)."""
    g = torch.randn(64, 96, generator=torch.Generator().manual_seed(act)) * 3
    torch.testing.assert_close(oracle.gated_act_ref(g, None, act), FALLBACK[act](g), rtol=2e-6, atol=1e-5)


def test_gated_act_without_up_argument_rules():
    """up = NULL (activation only): any up_row_stride is accepted (it is not read), an empty
    call returns VF_OK, and a NULL gate or out is still refused before any launch."""
    lib = _lib.load()
    assert lib.vf_gated_act_fwd(ctypes.byref(_args(up=None, up_row_stride=0, rows=0)), None) == _lib.VF_OK
    assert lib.vf_gated_act_fwd(ctypes.byref(_args(up=None, up_row_stride=-5, rows=0)), None) == _lib.VF_OK
    assert lib.vf_gated_act_fwd(ctypes.byref(_args(gate=None, up=None)), None) == _lib.VF_EINVAL
    assert "non-null" in lib.vf_last_error().decode()
    assert lib.vf_gated_act_fwd(ctypes.byref(_args(out=None, up=None)), None) == _lib.VF_EINVAL
