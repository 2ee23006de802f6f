"""The drop-in modules against the reference's own ones: every reference parameter keeps its
name, kind, default and position (extra parameters are keyword-only), and the reference's
exports exist here.  Needs a reference install (VF_REFERENCE, or baseline/_ref from
`pip install --target baseline/_ref <reference checkout>`); skipped without one."""
import importlib
import inspect
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _reference_root():
    env = os.environ.get("VF_REFERENCE")
    for cand in ([Path(env)] if env else []) + [ROOT / "baseline" / "_ref"]:
        if (cand / "kernels" / "flash_deberta_attention.py").exists():
            return cand
    return None


REF = _reference_root()
pytestmark = pytest.mark.skipif(REF is None, reason="no reference install (VF_REFERENCE or baseline/_ref)")

CASES = [
    ("flash_deberta_attention", "flash_deberta_attention"),
    ("flash_deberta_attention", "clear_config_cache"),
    ("flash_attention_rpb", "flash_attention_rpb_final"),
    ("ff_fused", "fused_gelu_mul_dropout"),
]


def _load_reference(module):
    """The reference's kernels.<module>, loaded from its file under a private name so that it
    never shadows this repository's `kernels` package."""
    spec = importlib.util.spec_from_file_location(f"_vf_reference_kernels_{module}", REF / "kernels" / f"{module}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("module,fn", CASES)
def test_signature_keeps_every_reference_parameter(module, fn):
    ours = inspect.signature(getattr(importlib.import_module(f"kernels.{module}"), fn))
    theirs = inspect.signature(getattr(_load_reference(module), fn))
    ours_p, theirs_p = list(ours.parameters.values()), list(theirs.parameters.values())
    assert len(ours_p) >= len(theirs_p)
    for a, b in zip(ours_p, theirs_p):
        assert (a.name, a.kind, a.default) == (b.name, b.kind, b.default), f"{fn}: {a} != {b}"
    for extra in ours_p[len(theirs_p):]:
        assert extra.kind == inspect.Parameter.KEYWORD_ONLY and extra.default is None, f"{fn}: extra {extra}"


def test_reference_exports_exist():
    ref = _load_reference("flash_deberta_attention")
    ours = importlib.import_module("kernels.flash_deberta_attention")
    for name in ref.__all__:
        assert hasattr(ours, name), name
        assert name in ours.__all__, name
    assert ours.HAS_TRITON is True
