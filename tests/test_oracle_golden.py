"""Pins the CPU oracle to the reference: every check compares oracle/ against outputs that
tests/golden/make_golden.py produced by running the reference's own functions."""
import numpy as np
import pytest
import torch

import golden_inputs as gi
import oracle
from oracle.rpb import deberta_position_index_ref
from _util import assert_close, lens_mask

G = np.load(gi.__file__.replace("golden_inputs.py", "golden.npz"))
R = torch.arange(-gi.R_SWEEP, gi.R_SWEEP + 1)


@pytest.mark.parametrize("bs,mp", gi.DEBERTA_BUCKET_CONFIGS)
def test_deberta_bucket_sweep_bit_exact(bs, mp):
    ours = oracle.deberta_log_bucket_ref(R, bs, mp).numpy()
    ref = G[f"deberta_bucket_{bs}_{mp}"].astype(np.int64)
    assert np.array_equal(ours, ref)


@pytest.mark.parametrize("nb,md,bidir", gi.T5_BUCKET_CONFIGS)
def test_t5_bucket_sweep_bit_exact(nb, md, bidir):
    ours = oracle.t5_relative_bucket_ref(R, bidir, nb, md).numpy()
    ref = G[f"t5_bucket_{nb}_{md}_{int(bidir)}"].astype(np.int64)
    assert np.array_equal(ours, ref)


def test_exact_integer_hazards():
    # DeBERTa |r| = 511 at (256, 512): log ratio is exactly 1 -> bucket 255 (512 -> 256).
    b = oracle.deberta_log_bucket_ref(torch.tensor([511, -511, 512, 510]), 256, 512)
    assert b.tolist() == [255, -255, 256, 255]
    # T5 |r| = 16/32/64 at (32, 128): log ratio hits 2.0/4.0/6.0 exactly before truncation.
    t = oracle.t5_relative_bucket_ref(torch.tensor([16, 32, 64, -16, -32, -64]), True, 32, 128)
    assert t.tolist() == [16 + 8 + 2, 16 + 8 + 4, 16 + 8 + 6, 8 + 2, 8 + 4, 8 + 6]


@pytest.mark.parametrize("name", ["deberta_log", "deberta_linear"])
def test_deberta_op_oracle_matches_reference(name):
    c = gi.deberta_op_case(name)
    for key in ("q", "k", "v", "pos_key", "pos_query"):
        assert gi.sha(c[key]) == str(G[f"{name}_sha_{key}"]), f"regenerated input {key} differs"
    out = oracle.deberta_attention_ref(c["q"], c["k"], c["v"], c["seq_lengths"], c["pos_key"], c["pos_query"],
                                       False, c["sm_scale"], c["position_buckets"], c["max_relative_distance"],
                                       c["use_log_bucket"], dtype=torch.float32)
    ref = torch.from_numpy(G[f"{name}_out"])
    # the reference fallback computes padded rows; compare valid rows only
    assert_close(out, ref, lens_mask(c["seq_lengths"], out.shape[2]), max_abs=2e-5, min_cos=0.999999, what=name)


def test_t5_oracle_matches_reference():
    c = gi.t5_case("t5_enc")
    for key in ("q", "k", "v", "table", "mask"):
        assert gi.sha(c[key]) == str(G[f"t5_enc_sha_{key}"])
    out = oracle.rpb_attention_ref(c["q"], c["k"], c["v"], c["table"], c["num_buckets"], c["max_distance"],
                                   False, c["mask"], 1.0, dtype=torch.float32)
    ref = torch.from_numpy(G["t5_enc_out"])
    # every row (padded ones included) is defined by the reference's T5 path
    assert_close(out, ref, None, max_abs=2e-5, min_cos=0.999999, what="t5_enc")


def test_t5_oracle_matches_reference_with_query_varying_mask():
    """A [B, 1, L, L] mask (varies over query rows) through the reference's own bias helper
    and SDPA: the oracle the query-row-mask kernel instance is checked against."""
    c = gi.t5_case("t5_qmask")
    for key in ("q", "k", "v", "table", "mask"):
        assert gi.sha(c[key]) == str(G[f"t5_qmask_sha_{key}"])
    out = oracle.rpb_attention_ref(c["q"], c["k"], c["v"], c["table"], c["num_buckets"], c["max_distance"],
                                   False, c["mask"], 1.0, dtype=torch.float32)
    ref = torch.from_numpy(G["t5_qmask_out"])
    assert_close(out, ref, None, max_abs=2e-5, min_cos=0.999999, what="t5_qmask")


def test_deberta_layer_oracle_matches_reference():
    c = gi.deberta_layer_case()
    for key in ("hidden", "wq", "wk", "wv", "rel"):
        assert gi.sha(c[key]) == str(G[f"deberta_layer_sha_{key}"])
    out = oracle.deberta_layer_ref(c["hidden"], c["mask"], c["wq"], c["bq"], c["wk"], c["bk"], c["wv"], c["bv"],
                                   c["rel"], c["num_heads"], c["position_buckets"], c["max_relative_positions"])
    ref = torch.from_numpy(G["deberta_layer_out"])
    valid = lens_mask(c["lens"], out.shape[1])
    o = out[valid]
    r = ref[valid]
    assert (o - r).abs().max().item() < 2e-5


def test_deberta_position_index_symmetry():
    # p2c in the HF layer (clamp(-bucket(n - m) + S)) equals the op's clamp(bucket(m - n) + S)
    idx = deberta_position_index_ref(300, 300, 64, 64, 128, True)
    rel = torch.arange(300)[:, None] - torch.arange(300)[None, :]
    hf = torch.clamp(-oracle.deberta_log_bucket_ref(-rel, 64, 128) + 64, 0, 127)
    assert torch.equal(idx, hf)


def test_gliner_span_oracle_matches_reference():
    c = gi.span_case()
    for key in ("h", "pe", "span_idx"):
        assert gi.sha(c[key]) == str(G[f"gliner_span_sha_{key}"])
    for key, t in c["weights"].items():
        assert gi.sha(t) == str(G[f"gliner_span_sha_{key}"])
    ref = torch.from_numpy(G["gliner_span_out"])
    out = oracle.span_scores_ref(c["h"], c["span_idx"], c["weights"], c["pe"], c["max_width"])
    assert (out - ref).abs().max().item() < 1e-12
    # The factored form the GPU kernel evaluates equals the reference's order of operations.
    fac = oracle.span_scores_factored_ref(c["h"], c["span_idx"], c["weights"], c["pe"], c["max_width"])
    assert (fac - ref).abs().max().item() < 1e-12


def test_deberta_intermediate_oracle_matches_reference():
    c = gi.intermediate_case()
    for key in ("x", "weight", "bias"):
        assert gi.sha(c[key]) == str(G[f"deberta_intermediate_sha_{key}"])
    out = oracle.linear_gelu_ref(c["x"], c["weight"], c["bias"])
    ref = torch.from_numpy(G["deberta_intermediate_out"]).double()
    assert (out - ref).abs().max().item() < 2e-5
