"""Linear + activation GEMMs on the GPU (csrc/vf_gemm.cu through torch.ops.vf_b200.linear_act and
the C ABI) against the plain PyTorch fp32 reference of the same op on the same 16-bit inputs:
F.gelu(F.linear(x, W, b)) (DeBERTa), gelu_tanh(x W0^T) * up (mT5).  Gate: max-abs <= 2e-2 (of
the output scale where outputs exceed 1) and cosine >= 0.9999 per row, and no further from fp32
than 1.5x the two-step 16-bit path the reference takes (GEMM, rounding, then the activation)."""
import ctypes

import pytest
import torch
import torch.nn.functional as F

from kernels.linear_act import gated_gelu_tanh, linear_gelu
from vf_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _case(rows, K, N, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(rows, K, generator=g, device=DEV).to(dtype)
    w = (torch.randn(N, K, generator=g, device=DEV) * K ** -0.5).to(dtype)
    b = (torch.randn(N, generator=g, device=DEV) * 0.5).to(dtype)
    return x, w, b


def _check(out, x, w, b, what):
    ref = F.gelu(F.linear(x.float(), w.float(), b.float()))
    theirs = F.gelu(F.linear(x, w, b)).float()
    err = (out.float() - ref).abs().max().item()
    err_t = (theirs - ref).abs().max().item()
    cos = F.cosine_similarity(out.float().reshape(-1, ref.shape[-1]), ref.reshape(-1, ref.shape[-1]), dim=-1)
    assert err <= 2e-2, f"{what}: max_abs {err:.3e}"
    assert err <= 1.5 * err_t + 1e-3, f"{what}: {err:.3e} vs torch's 16-bit path {err_t:.3e}"
    assert cos.min().item() >= 0.9999, f"{what}: min row cosine {cos.min().item():.6f}"


@pytest.mark.parametrize("rows,K,N", [
    (1, 64, 8), (100, 1024, 4096), (1000, 768, 3072), (8192, 1024, 4096), (257, 4096, 1024), (333, 72, 136),
])
def test_linear_gelu_matches_torch_fp32(rows, K, N):
    x, w, b = _case(rows, K, N, torch.bfloat16, rows + K)
    _check(linear_gelu(x, w, b), x, w, b, f"{rows}x{K}x{N}")


def test_linear_gelu_fp16_views_and_no_bias():
    x, w, b = _case(300, 1024, 2048, torch.float16, 7)
    wide = torch.cat([x, x], 1)[:, :1024]                         # row stride 2048
    _check(linear_gelu(wide, w, b), x, w, b, "fp16 strided")
    x3 = x.view(3, 100, 1024)
    out = linear_gelu(x3, w, None)
    assert out.shape == (3, 100, 2048)
    _check(out.view(300, 2048), x, w, torch.zeros_like(b), "3-D, no bias")


def test_linear_act_through_c_abi_twice():
    lib = _lib.load()
    x, w, b = _case(500, 1024, 4096, torch.bfloat16, 3)
    out = torch.full((500, 4096), float("nan"), device=DEV, dtype=torch.bfloat16)
    a = _lib.LinearActArgs(dtype=_lib.VF_DTYPE_BF16, x=x.data_ptr(), weight=w.data_ptr(), bias=b.data_ptr(),
                           mul=None, out=out.data_ptr(), rows=500, K=1024, N=4096, x_row_stride=1024,
                           weight_row_stride=1024, mul_row_stride=0, out_row_stride=4096, act=1)
    for _ in range(2):
        rc = lib.vf_linear_act_fwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.vf_last_error().decode()
        torch.cuda.synchronize()
        _check(out, x, w, b, "c abi")


def _gelu_tanh_ref(z):
    return 0.5 * z * (1.0 + torch.tanh(0.7978845608028654 * (z + 0.044715 * z ** 3)))


@pytest.mark.parametrize("rows,K,N,dtype", [
    (1, 64, 8, torch.bfloat16), (777, 1024, 2816, torch.bfloat16), (8192, 1024, 2816, torch.bfloat16),
    (300, 512, 1024, torch.float16),
])
def test_gated_gelu_tanh_matches_torch_fp32(rows, K, N, dtype):
    """gelu_tanh(x W0^T) * up (the mT5 gated feed-forward, up = x W1^T) against fp32 torch on
    the same inputs, and no further from it than the reference's two-step 16-bit path
    (16-bit projections, then the activation kernel's fp32 arithmetic on them)."""
    g = torch.Generator(device=DEV).manual_seed(rows + N)
    x = torch.randn(rows, K, generator=g, device=DEV).to(dtype)
    w0 = (torch.randn(N, K, generator=g, device=DEV) * K ** -0.5).to(dtype)
    w1 = (torch.randn(N, K, generator=g, device=DEV) * K ** -0.5).to(dtype)
    up = x @ w1.t()
    out = gated_gelu_tanh(x, w0, up)
    ref = _gelu_tanh_ref(x.float() @ w0.float().t()) * up.float()
    theirs = (_gelu_tanh_ref((x @ w0.t()).float()) * up.float()).to(dtype).float()
    err = (out.float() - ref).abs().max().item()
    err_t = (theirs - ref).abs().max().item()
    scale = max(ref.abs().max().item(), 1.0)     # outputs reach ~10: one bf16 half-ulp there is 0.03
    cos = F.cosine_similarity(out.float(), ref, dim=-1)
    assert err <= 2e-2 * scale and err <= 1.5 * err_t + 1e-3, (err, err_t, scale)
    assert cos.min().item() >= 0.9999


def test_gated_gelu_tanh_strided_up_through_c_abi():
    lib = _lib.load()
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(256, 1024, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(2 * 2816, 1024, generator=g, device=DEV) * 1024 ** -0.5).to(torch.bfloat16)   # wi_0; wi_1 stacked
    gu = x @ w.t()                                   # [256, 2F]: up is the strided right half
    up = gu[:, 2816:]
    out = torch.empty(256, 2816, device=DEV, dtype=torch.bfloat16)
    a = _lib.LinearActArgs(dtype=_lib.VF_DTYPE_BF16, x=x.data_ptr(), weight=w.data_ptr(), bias=None,
                           mul=up.data_ptr(), out=out.data_ptr(), rows=256, K=1024, N=2816, x_row_stride=1024,
                           weight_row_stride=1024, mul_row_stride=2 * 2816, out_row_stride=2816, act=0)
    rc = lib.vf_linear_act_fwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.vf_last_error().decode()
    torch.cuda.synchronize()
    ref = _gelu_tanh_ref(x.float() @ w[:2816].float().t()) * up.float()
    assert (out.float() - ref).abs().max().item() <= 2e-2 * max(ref.abs().max().item(), 1.0)
