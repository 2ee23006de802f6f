"""The DeBERTa residual add + LayerNorm on the CPU: the oracle pinned to the reference's own
call (models/deberta_v2/deberta_v2_encoder.py:507 / :566, nn.LayerNorm of the tensor sum),
and the C-ABI's argument checks (no launch)."""
import ctypes
import math

import pytest
import torch
import torch.nn.functional as F

import oracle
from vf_b200 import _lib
from vf_b200 import encoders as EN


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cols", [1024, 768, 37])
def test_oracle_matches_reference_layer_norm_call(dtype, cols):
    g = torch.Generator().manual_seed(cols)
    x = torch.randn(64, cols, generator=g).to(dtype)
    r = (3.0 * torch.randn(64, cols, generator=g) + 0.5).to(dtype)
    w = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(dtype)
    b = (0.1 * torch.randn(cols, generator=g)).to(dtype)
    ln = torch.nn.LayerNorm(cols, eps=1e-7).to(dtype)
    with torch.no_grad():
        ln.weight.copy_(w)
        ln.bias.copy_(b)
        ref = ln(x + r)                               # the reference's two calls
    ours = oracle.add_layer_norm_ref(x, r, w, b, 1e-7)
    assert ours.dtype == dtype
    # The oracle normalises in float64: one unit in the last place of a 16-bit dtype at most;
    # torch's fp32 norm itself carries a few units of fp32 rounding (8 allowed).
    ulp = {torch.float32: 2.0 ** -20, torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}[dtype]
    torch.testing.assert_close(ours.float(), ref.float(), rtol=ulp, atol=ulp)
    assert torch.equal(EN.add_layer_norm_torch(x, r, w, b, 1e-7), F.layer_norm(x + r, (cols,), w, b, 1e-7))


def test_oracle_without_bias_and_constant_rows():
    x = torch.zeros(3, 16, dtype=torch.float64)
    r = torch.full((3, 16), 2.5, dtype=torch.float64)
    w = torch.ones(16, dtype=torch.float64)
    out = oracle.add_layer_norm_ref(x, r, w, None, 1e-7)
    assert torch.equal(out, torch.zeros_like(out))    # a constant row normalises to zero
    y = oracle.add_layer_norm_ref(torch.arange(8.0).view(1, 8), torch.zeros(1, 8), torch.ones(8), None, 0.0)
    assert math.isclose(float(y.mean()), 0.0, abs_tol=1e-6) and math.isclose(float(y.var(unbiased=False)), 1.0,
                                                                             rel_tol=1e-5)


def _args(**kw):
    a = _lib.AddLayerNormArgs()
    a.dtype, a.x, a.residual, a.weight, a.bias, a.out = _lib.VF_DTYPE_BF16, 0x10000, 0x20000, 0x30000, 0x40000, 0x50000
    a.rows, a.cols = 4, 64
    a.x_row_stride = a.residual_row_stride = a.out_row_stride = 64
    a.eps = 1e-7
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code,msg", [
    (dict(rows=-1), _lib.VF_EINVAL, "negative"),
    (dict(x=None), _lib.VF_EINVAL, "non-null"),
    (dict(weight=None), _lib.VF_EINVAL, "non-null"),
    (dict(residual_row_stride=32), _lib.VF_EINVAL, "row strides"),
    (dict(eps=float("nan")), _lib.VF_EINVAL, "eps"),
    (dict(eps=-1.0), _lib.VF_EINVAL, "eps"),
    (dict(dtype=9), _lib.VF_EUNSUPPORTED, "dtype"),
])
def test_add_layer_norm_validation_rejects_before_launch(kw, code, msg):
    lib = _lib.load()
    assert lib.vf_add_layer_norm_fwd(ctypes.byref(_args(**kw)), None) == code
    assert msg in lib.vf_last_error().decode()


def test_add_layer_norm_empty_is_a_no_op():
    lib = _lib.load()
    assert lib.vf_add_layer_norm_fwd(ctypes.byref(_args(rows=0)), None) == _lib.VF_OK
    assert lib.vf_add_layer_norm_fwd(ctypes.byref(_args(cols=0)), None) == _lib.VF_OK
    assert lib.vf_add_layer_norm_fwd(None, None) == _lib.VF_EINVAL


@pytest.mark.parametrize("kw,exc,msg", [
    (dict(weight=torch.ones(32)), ValueError, "weight must be"),
    (dict(bias=torch.ones(3, 64)), ValueError, "bias must be"),
    (dict(input_tensor=torch.zeros(4, 32)), ValueError, "identical shape"),
    (dict(weight=torch.ones(64, dtype=torch.float64)), TypeError, "dtype"),
    (dict(), RuntimeError, "CUDA"),
])
def test_drop_in_checks_arguments_before_the_op(kw, exc, msg):
    """The drop-in's own checks (shapes, dtypes, CUDA device) raise before the op is called."""
    from kernels.fused_add_layernorm import fused_add_layer_norm
    args = dict(hidden_states=torch.zeros(4, 64), input_tensor=torch.zeros(4, 64), weight=torch.ones(64),
                bias=torch.zeros(64))
    args.update(kw)
    with pytest.raises(exc, match=msg):
        fused_add_layer_norm(**args)
