"""Argument checks inside the CUDA implementations of the torch ops raise RuntimeError.

Each case calls a torch.ops.vf_b200 op with CUDA tensors and one bad argument.  The check
fires on the host, before any kernel launch: a TORCH_CHECK in csrc/vf_torch_ops.cpp, or a
negative code from the C ABI turned into a TORCH_CHECK by check_rc.  Each case runs in a
child process, so a crash of the host process on the throw (rather than a Python
RuntimeError) fails the test without taking the test session with it.
"""
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

PRELUDE = f"""
import sys
sys.path[:0] = [{str(ROOT / 'vllm-factory_b200')!r}]
import torch
import vf_b200.ops  # noqa: F401
dev = torch.device("cuda:0")
bf = torch.bfloat16
"""

CASES = {
    # TORCH_CHECK in add_layer_norm: weight length differs from the row width
    "add_layer_norm_weight": """
x = torch.zeros(4, 64, dtype=bf, device=dev)
torch.ops.vf_b200.add_layer_norm(x, x, torch.ones(32, dtype=bf, device=dev), None, 1e-7)
""",
    # TORCH_CHECK in gated_act: gate and up differ in shape
    "gated_act_shapes": """
torch.ops.vf_b200.gated_act(torch.zeros(4, 64, dtype=bf, device=dev), torch.zeros(4, 32, dtype=bf, device=dev), 0)
""",
    # TORCH_CHECK in rpb_attention: a 3-D bias table
    "rpb_table_rank": """
q = torch.zeros(1, 2, 16, 64, dtype=bf, device=dev)
torch.ops.vf_b200.rpb_attention(q, q, q, torch.zeros(32, 2, 1, dtype=bf, device=dev), 32, 128, False, None, 0.0, 1.0)
""",
    # C ABI VF_EINVAL (pos_key shape) through check_rc
    "deberta_pos_key_shape": """
q = torch.zeros(1, 2, 16, 64, dtype=bf, device=dev)
pk = torch.zeros(1, 2, 15, 512, dtype=bf, device=dev)
torch.ops.vf_b200.deberta_attention(q, q, q, None, pk, None, False, None, 256, 512, True)
""",
    # C ABI VF_EUNSUPPORTED (head_dim 32) through check_rc
    "rpb_head_dim": """
q = torch.zeros(1, 2, 16, 32, dtype=bf, device=dev)
torch.ops.vf_b200.rpb_attention(q, q, q, None, 32, 128, False, None, 0.0, 1.0)
""",
}


@pytest.mark.gpu
@pytest.mark.parametrize("case", sorted(CASES))
def test_argument_check_in_cuda_impl_raises(case):
    code = PRELUDE + textwrap.dedent(f"""
try:
{textwrap.indent(textwrap.dedent(CASES[case]).strip(), '    ')}
    print("RETURNED")
except RuntimeError as e:
    print("RAISED", str(e).splitlines()[0])
torch.cuda.synchronize()
""")
    res = subprocess.run([sys.executable, "-X", "faulthandler", "-c", code], cwd=ROOT, capture_output=True,
                         text=True, timeout=300)
    assert res.returncode == 0, f"exit {res.returncode}\n{res.stdout[-2000:]}\n{res.stderr[-4000:]}"
    assert "RAISED" in res.stdout, res.stdout


@pytest.mark.gpu
def test_device_error_check_mode_raises_on_bad_packed_offsets():
    """With VF_B200_CHECK_DEVICE_ERRORS=1 every op synchronises after its launch and raises
    when a kernel set the device error word: here decreasing packed offsets (bit 2; the kernel
    clamps the rows it uses into the views and returns).  Without the variable the same call
    returns and only vf_device_error reports it."""
    import os
    call = """
q = torch.randn(200, 2, 64, dtype=bf, device=dev)
t = torch.randn(32, 2, dtype=bf, device=dev)
bad = torch.tensor([100, 40, 160], dtype=torch.int32, device=dev)
torch.ops.vf_b200.rpb_attention_varlen(q, q, q, bad, 100, t, 32, 128, False, 1.0)
"""
    code = PRELUDE + textwrap.dedent(f"""
import vf_b200
vf_b200.device_error(clear=True)
try:
{textwrap.indent(textwrap.dedent(call).strip(), '    ')}
    torch.cuda.synchronize()
    print("RETURNED", vf_b200.device_error(clear=True) & 4)
except RuntimeError as e:
    print("RAISED", str(e).splitlines()[0])
""")
    for flag, want in (("1", "RAISED vf_b200: a kernel reported device error word"), ("0", "RETURNED 4")):
        env = dict(os.environ, VF_B200_CHECK_DEVICE_ERRORS=flag)
        res = subprocess.run([sys.executable, "-X", "faulthandler", "-c", code], cwd=ROOT, capture_output=True,
                             text=True, timeout=300, env=env)
        assert res.returncode == 0, f"exit {res.returncode}\n{res.stdout[-2000:]}\n{res.stderr[-4000:]}"
        assert want in res.stdout, res.stdout
