"""Failure detection on the GPU without a fault: a bounded in-kernel wait on a barrier
that nothing arrives at must give up, report through the device error word, and leave
the context usable."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_timeout_and_context_survives():
    import vf_b200
    from vf_b200 import _lib
    assert vf_b200.device_error(clear=True) == 0
    _lib.selftest_wait_timeout(limit_cycles=2_000_000)       # ~1 ms of SM cycles
    word = vf_b200.device_error(clear=True)
    assert word & 1, f"timeout bit not set: {word}"
    assert vf_b200.device_error(clear=True) == 0
    # the context still runs the real kernels
    from kernels.flash_attention_rpb import flash_attention_rpb_final
    q, k, v = (torch.randn(1, 2, 130, 64, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    table = torch.randn(32, 2, device="cuda", dtype=torch.bfloat16)
    out = flash_attention_rpb_final(q, k, v, table, 32, 128, False)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert vf_b200.device_error(clear=True) == 0
