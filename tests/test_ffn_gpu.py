"""GPU parity of the gated feed-forward activation (kernels.ff_fused.fused_gelu_mul_dropout
-> vf_gated_act_fwd) against the CPU oracle of the reference's kernel arithmetic: fp32 to
1e-5, 16-bit outputs to within rounding of the fp32 result (one unit in the last place)."""
import pytest
import torch

import oracle
import vf_b200.ops  # noqa: F401  (registers torch.ops.vf_b200)

pytestmark = pytest.mark.gpu

TOL = {torch.float32: dict(rtol=1e-5, atol=1e-6), torch.float16: dict(rtol=1e-3, atol=1e-4),
       torch.bfloat16: dict(rtol=8e-3, atol=1e-3)}
NAMES = {0: "gelu_new", 1: "gelu_accurate", 2: "relu", 3: "silu"}


def _op():
    from kernels.ff_fused import fused_gelu_mul_dropout
    return fused_gelu_mul_dropout


def _check(gate, up, act, what):
    out = _op()(gate.cuda(), up.cuda(), NAMES[act])
    torch.cuda.synchronize()
    assert out.shape == gate.shape and out.dtype == gate.dtype
    ref = oracle.gated_act_ref(gate.cpu(), up.cpu(), act)
    torch.testing.assert_close(out.cpu().float(), ref.float(), **TOL[gate.dtype], msg=what)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_gated_act_parity(dtype, act):
    g = torch.Generator().manual_seed(act)
    gate, up = (torch.randn(333, 2816, generator=g) * 3).to(dtype), torch.randn(333, 2816, generator=g).to(dtype)
    _check(gate, up, act, f"{dtype} act={act}")


def test_stacked_projection_halves_read_in_place():
    # gate / up as the two column halves of one [T, 2F] projection (row stride 2F).
    gu = (torch.randn(1000, 2 * 2816) * 2).to(torch.bfloat16)
    _check(gu[:, :2816], gu[:, 2816:], 0, "halves")


@pytest.mark.parametrize("cols", [1, 7, 13, 2817])
def test_widths_without_16_byte_vectors(cols):
    gate, up = torch.randn(5, 3, cols).to(torch.bfloat16), torch.randn(5, 3, cols).to(torch.bfloat16)
    _check(gate, up, 0, f"cols={cols}")


def test_strided_and_transposed_operands():
    x = torch.randn(64, 96)
    gate = x.t().to(torch.float16)                 # last-dim stride != 1 -> copied
    up = torch.randn(2, 96, 64).to(torch.float16)[1]
    _check(gate, up, 3, "transposed")


def test_mt5_c4_shape_and_empty():
    gate = (torch.randn(4096, 2816) * 3).to(torch.bfloat16)
    _check(gate, torch.randn(4096, 2816).to(torch.bfloat16), 0, "mT5 shape")
    e = torch.empty(0, 2816, dtype=torch.bfloat16, device="cuda")
    assert _op()(e, e).shape == (0, 2816)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_activation_without_up(dtype, act):
    """torch.ops.vf_b200.gated_act(x, None, act): out = act(x) (vector and scalar kernels)."""
    for shape in ((1024, 4096), (37, 101)):
        x = (torch.randn(*shape, generator=torch.Generator().manual_seed(act)) * 3).to(dtype)
        out = torch.ops.vf_b200.gated_act(x.cuda(), None, act)
        torch.cuda.synchronize()
        ref = oracle.gated_act_ref(x, None, act)
        torch.testing.assert_close(out.cpu().float(), ref.float(), **TOL[dtype], msg=f"{dtype} act {act} {shape}")


def test_exact_gelu_matches_torch_gelu():
    """The DeBERTa stack's activation against torch's own exact GELU on the GPU."""
    import torch.nn.functional as F
    from vf_b200.encoders import exact_gelu_kernel
    x = (torch.randn(4096, 4096, generator=torch.Generator().manual_seed(5)) * 2).to(torch.bfloat16).cuda()
    torch.testing.assert_close(exact_gelu_kernel(x).float(), F.gelu(x).float(), **TOL[torch.bfloat16])
