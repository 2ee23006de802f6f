"""Linear + activation (vf_linear_act_fwd: exact GELU + bias, or GELU-tanh times a second operand), CPU side: the C entry point rejects bad arguments
before any CUDA call, the torch op's fake / CPU registrations, the drop-in's activation check
and installer."""
import ctypes

import pytest
import torch

from vf_b200 import _lib


def _args(**kw):
    a = _lib.LinearActArgs(dtype=_lib.VF_DTYPE_BF16, x=0x10000, weight=0x20000, bias=0x30000, mul=None, out=0x40000,
                           rows=100, K=1024, N=4096, x_row_stride=1024, weight_row_stride=1024, mul_row_stride=0,
                           out_row_stride=4096, act=1)
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,code,msg", [
    (dict(dtype=_lib.VF_DTYPE_F32), _lib.VF_EUNSUPPORTED, "dtype"),
    (dict(act=2), _lib.VF_EUNSUPPORTED, "built forms"),
    (dict(act=0), _lib.VF_EINVAL, "takes a bias and no mul"),                         # gated form without mul
    (dict(act=0, bias=None, mul=0x50000, mul_row_stride=100), _lib.VF_EINVAL, "at least"),
    (dict(act=1, mul=0x50000, mul_row_stride=4096), _lib.VF_EINVAL, "takes a bias and no mul"),
    (dict(act=0, bias=None, mul=0x50008, mul_row_stride=4096), _lib.VF_EINVAL, "16-byte"),
    (dict(K=0), _lib.VF_EINVAL, "K > 0"),
    (dict(rows=-1), _lib.VF_EINVAL, "rows >= 0"),
    (dict(weight=None), _lib.VF_EINVAL, "non-null"),
    (dict(bias=None), _lib.VF_EINVAL, "takes a bias"),
    (dict(x_row_stride=512), _lib.VF_EINVAL, "at least"),
    (dict(N=4100, out_row_stride=4100), _lib.VF_EINVAL, "multiples of 8"),
    (dict(x=0x10004), _lib.VF_EINVAL, "16-byte"),
])
def test_linear_act_rejects_before_launch(kw, code, msg):
    lib = _lib.load()
    a = _args(**kw)
    assert lib.vf_linear_act_fwd(ctypes.byref(a), None) == code
    assert msg in lib.vf_last_error().decode()


def test_linear_act_no_rows_is_ok_without_cuda():
    lib = _lib.load()
    assert lib.vf_linear_act_fwd(None, None) == _lib.VF_EINVAL
    a = _args(rows=0, x=None)
    assert lib.vf_linear_act_fwd(ctypes.byref(a), None) == _lib.VF_OK


def test_linear_act_op_fake_and_cpu():
    import vf_b200.ops  # noqa: F401
    x = torch.empty(3, 7, 64, dtype=torch.bfloat16, device="meta")
    w = torch.empty(256, 64, dtype=torch.bfloat16, device="meta")
    assert torch.ops.vf_b200.linear_act(x, w, None, None, 1).shape == (3, 7, 256)
    with pytest.raises(RuntimeError, match="no CPU implementation"):
        torch.ops.vf_b200.linear_act(torch.zeros(4, 64, dtype=torch.bfloat16), torch.zeros(8, 64, dtype=torch.bfloat16),
                                     None, None, 1)


def test_intermediate_dropin_activation_check_and_installer():
    import torch.nn.functional as F
    from kernels import linear_act
    import transformers.activations as A
    assert linear_act._exact_gelu(A.ACT2FN["gelu"]) and linear_act._exact_gelu(F.gelu)
    assert not linear_act._exact_gelu(A.ACT2FN["gelu_new"]) and not linear_act._exact_gelu(torch.nn.GELU("tanh"))

    class Inter:
        def forward(self, hidden_states):
            return "reference"

    linear_act.install_fused_intermediate(Inter)
    linear_act.install_fused_intermediate(Inter)
    assert Inter.forward is linear_act.deberta_intermediate_forward
    assert Inter._vf_reference_forward(None, None) == "reference"
    with pytest.raises(RuntimeError, match="CUDA"):
        Inter().forward(torch.zeros(2, 8))
