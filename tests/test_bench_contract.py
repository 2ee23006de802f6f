"""bench.py's CPU-side contract: the reference arm (the oracle on the host cores) prints
one JSON line with the keys the driver reads, only rank 0 prints under torchrun, and every
workload with a committed ncu capture has its DRAM traffic in profiles/traffic.json."""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(args, env_extra=None, timeout=240):
    env = dict(os.environ, **(env_extra or {}))
    res = subprocess.run([sys.executable, "bench.py", *args], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=timeout)
    assert res.returncode == 0, res.stderr[-2000:]
    return [l for l in res.stdout.splitlines() if l.startswith("{")]


@pytest.mark.parametrize("workload", ["mt5_c2", "deberta_add_ln", "deberta_ffn_gemm"])
def test_reference_arm_line(workload):
    lines = _run(["--impl", "reference", "--workload", workload, "--steps", "3", "--warmup", "3"])
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    for k in ("metric", "unit", "n_gpus", "steps", "warmup", "config", "dtype", "data"):
        assert k in d
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"] and cb["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    assert _run(["--impl", "reference", "--gpus", "2", "--steps", "3", "--warmup", "3"],
                {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"}) == []


def test_traffic_entries_for_captured_workloads():
    t = json.loads((ROOT / "profiles" / "traffic.json").read_text())
    for w in ("mt5_c2", "deberta_c1", "mt5_c2_varlen", "deberta_c1_varlen", "deberta_c1_fused", "mt5_ffn_act",
              "deberta_add_ln"):
        assert isinstance(t.get(w), int) and t[w] > 0, w


def test_reference_arm_default_has_same_configs_and_sub_results():
    """The default run's reference line carries the headline and both sub-results, each with
    the `config` object the GPU arm prints for the same workload."""
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "vllm-factory_b200"))
    import bench
    lines = _run(["--impl", "reference", "--steps", "3", "--warmup", "3"], timeout=400)
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["config"] == bench.attention_config("mt5_c2")
    subs = d["sub_results"]
    assert subs["deberta_c1"]["config"] == bench.attention_config("deberta_c1_fused")
    assert subs["deberta_c3"]["config"] == bench.attention_config("deberta_c3")
    assert subs["deberta_c3"]["unit"] == "tokens/s per layer" and subs["deberta_c3"]["scaling"] == "strong"
    for s in subs.values():
        assert s["impl"] == "reference" and s["value"] > 0
