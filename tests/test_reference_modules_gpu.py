"""The reference's own attention modules, run with their kernel imports bound to this repository.

tests/reference_modules_run.py builds DisentangledSelfAttentionV2 (DeBERTa v2/v3),
DisentangledSelfAttention (DeBERTa v1) and T5SelfAttention (mT5) from the reference install,
with `kernels.*` resolved here, and runs each layer through its flash path (this repository's
CUDA operators), its own bf16 PyTorch path and an fp32 copy of that PyTorch path.  Also, per
layer, the requests as one flat vLLM batch inside `varlen_glue.packed_batch` ("packed"), and
for DeBERTa v2 the fused position mode installed on the reference's class, padded ("fused")
and packed ("fused_packed"); each request's rows are compared with the padded fp32 result.

Gates, over the valid query rows: the flash path against the fp32 PyTorch path within
max-abs 2e-2 and per-row cosine 0.9995 (the layer's bf16 projections round before and after
the kernel; the kernel alone is held to 0.9999 by the operator tests), and no further from
the fp32 result than 1.5x the reference's own bf16 PyTorch path.  Needs a reference install
(VF_REFERENCE, or baseline/_ref); skipped without one."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
pytestmark = pytest.mark.gpu


def _reference_root():
    env = os.environ.get("VF_REFERENCE")
    for cand in ([Path(env)] if env else []) + [ROOT / "baseline" / "_ref"]:
        if (cand / "models" / "deberta_v2" / "deberta_v2_encoder.py").exists():
            return cand
    return None


@pytest.fixture(scope="module")
def results():
    ref = _reference_root()
    if ref is None:
        pytest.skip("no reference install (VF_REFERENCE or baseline/_ref)")
    proc = subprocess.run([sys.executable, str(ROOT / "tests" / "reference_modules_run.py"),
                           "--reference", str(ref), "--device", "cuda"],
                          capture_output=True, text=True, timeout=900, cwd=str(ROOT))
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")]
    assert proc.returncode == 0 and line, proc.stdout[-3000:] + proc.stderr[-3000:]
    return json.loads(line[-1][len("RESULT "):])


@pytest.mark.parametrize("layer", ["deberta_v2", "deberta_v1", "mt5"])
def test_reference_layer_flash_path_matches_its_pytorch_path(results, layer):
    r = results[layer]
    assert r["kernel_module"].startswith("kernels."), r["kernel_module"]
    assert Path(r["kernel_file"]).resolve().is_relative_to(ROOT / "vllm-factory_b200"), r["kernel_file"]
    theirs = r["torch_bf16"]
    expected = {"deberta_v2": ("flash", "packed", "fused", "fused_packed"),
                "deberta_v1": ("flash", "packed"), "mt5": ("flash", "packed")}[layer]
    for mode in expected:
        ours = r[mode]
        assert ours["max_abs"] <= 2e-2, (mode, r)
        assert ours["min_row_cos"] >= 0.9995, (mode, r)
        assert ours["max_abs"] <= 1.5 * theirs["max_abs"] + 1e-3, (mode, r)
        assert 1.0 - ours["min_row_cos"] <= 1.5 * (1.0 - theirs["min_row_cos"]) + 1e-5, (mode, r)


def test_reference_deberta_intermediate_with_fused_gelu(results):
    """DebertaV2Intermediate (models/deberta_v2/deberta_v2_encoder.py:535-550) with the dense
    layer and exact GELU as one GEMM (kernels.linear_act installed on the class), against its
    fp32 twin: within max-abs 2e-2 / cosine 0.9995 and no further than 1.5x its own bf16 path."""
    r = results["deberta_v2_intermediate"]
    assert r["kernel_module"] == "kernels.linear_act", r
    assert Path(r["kernel_file"]).resolve().is_relative_to(ROOT / "vllm-factory_b200"), r
    ours, theirs = r["fused"], r["torch_bf16"]
    assert ours["max_abs"] <= 2e-2 and ours["min_row_cos"] >= 0.9995, r
    assert ours["max_abs"] <= 1.5 * theirs["max_abs"] + 1e-3, r
