"""GPU parity of the DeBERTa residual add + LayerNorm (kernels.fused_add_layernorm ->
vf_add_layer_norm_fwd) against the CPU oracle (float64 normalisation of the dtype-rounded
sum): within one unit in the last place of a 16-bit dtype (8 units for fp32, whose fp32
reductions round a few times), and against torch's own two calls on the GPU to twice that.  Covers the register-held widths (NV = 1, 2, 4, 8 vectors per
lane), the scalar kernel (odd widths, misaligned views, rows too wide for registers),
strided and 3-D views, no bias, and a call through the C ABI."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

import oracle
from vf_b200 import _lib

pytestmark = pytest.mark.gpu

ULP = {torch.float32: 2.0 ** -20, torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}


def _inputs(shape, dtype, seed, bias=True):
    g = torch.Generator().manual_seed(seed)
    cols = shape[-1]
    x = torch.randn(*shape, generator=g).to(dtype)
    r = (2.0 * torch.randn(*shape, generator=g) + 0.25).to(dtype)
    w = (1.0 + 0.1 * torch.randn(cols, generator=g)).to(dtype)
    b = (0.1 * torch.randn(cols, generator=g)).to(dtype) if bias else None
    return x, r, w, b


def _op():
    from kernels.fused_add_layernorm import fused_add_layer_norm
    return fused_add_layer_norm


def _check(x, r, w, b, eps=1e-7, what=""):
    dev = lambda t: None if t is None else t.cuda()
    out = _op()(dev(x), dev(r), dev(w), dev(b), eps)
    torch.cuda.synchronize()
    assert out.shape == x.shape and out.dtype == x.dtype and out.is_contiguous()
    ref = oracle.add_layer_norm_ref(x.cpu(), r.cpu(), w.cpu(), None if b is None else b.cpu(), eps,
                                    dtype=torch.float64)
    u = ULP[x.dtype]
    # one unit in the last place of the result, relative, plus the same absolute near zero
    torch.testing.assert_close(out.cpu().double(), ref, rtol=u, atol=u * 2, msg=what)
    # torch's own unfused calls on the GPU (the reference's path) to the same bound
    torch_out = F.layer_norm(dev(x) + dev(r), (x.shape[-1],), dev(w), dev(b), eps)
    torch.testing.assert_close(out.float(), torch_out.float(), rtol=2 * u, atol=2 * u, msg=what)
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("rows,cols", [(1, 1024), (4097, 1024), (300, 768), (77, 256), (64, 2048), (5, 64)])
def test_add_layer_norm_matches_oracle(dtype, rows, cols):
    _check(*_inputs((rows, cols), dtype, rows * 7 + cols), what=f"{dtype} {rows}x{cols}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("cols", [1001, 4096, 7])
def test_add_layer_norm_scalar_kernel(dtype, cols):
    """Odd widths and rows wider than the register-held form use the scalar kernel."""
    _check(*_inputs((129, cols), dtype, cols), what=f"{dtype} cols {cols}")


def test_add_layer_norm_views_and_no_bias():
    x, r, w, b = _inputs((3, 50, 2048), torch.bfloat16, 11)
    # the left halves of wider rows (row stride 2048, 1024 columns) and a 3-D shape
    _check(x[..., :1024], r[..., 1024:], w[:1024], b[:1024], what="strided halves")
    _check(x[..., :1024], r[..., :1024], w[:1024], None, what="no bias")
    # a view misaligned by one element goes through the scalar kernel
    _check(x[..., 1:1025], r[..., :1024], w[:1024], b[:1024], what="misaligned")
    # eps as the DeBERTa config gives it, and a larger one
    _check(*_inputs((40, 1024), torch.bfloat16, 12), eps=1e-5, what="eps 1e-5")


def test_add_layer_norm_constant_rows_are_bias():
    x = torch.zeros(8, 1024, dtype=torch.bfloat16)
    r = torch.full((8, 1024), 3.0, dtype=torch.bfloat16)
    w = torch.ones(1024, dtype=torch.bfloat16)
    b = torch.linspace(-1, 1, 1024).to(torch.bfloat16)
    out = _op()(x.cuda(), r.cuda(), w.cuda(), b.cuda(), 1e-7)
    assert torch.equal(out.cpu(), b.expand(8, -1))


def test_add_layer_norm_empty():
    x = torch.empty(0, 1024, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(1024, dtype=torch.bfloat16, device="cuda")
    assert _op()(x, x, w, None).shape == (0, 1024)


def test_add_layer_norm_through_c_abi():
    """The C entry point with device pointers from torch, on the current stream."""
    lib = _lib.load()
    x, r, w, b = (t.cuda() for t in _inputs((513, 1024), torch.bfloat16, 21))
    out = torch.empty_like(x)
    a = _lib.AddLayerNormArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    a.x, a.residual, a.weight, a.bias, a.out = x.data_ptr(), r.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr()
    a.rows, a.cols = 513, 1024
    a.x_row_stride = a.residual_row_stride = a.out_row_stride = 1024
    a.eps = 1e-7
    assert lib.vf_add_layer_norm_fwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    torch.cuda.synchronize()
    ref = oracle.add_layer_norm_ref(x.cpu(), r.cpu(), w.cpu(), b.cpu(), 1e-7, dtype=torch.float64)
    torch.testing.assert_close(out.cpu().double(), ref, rtol=2.0 ** -7, atol=2.0 ** -6)
