"""Generates tests/golden/golden.npz by running the REFERENCE's own code on the CPU.

Run in a container that has the reference checkout (it is read-only input here and is
not needed anywhere else):

    python tests/golden/make_golden.py --reference /path/to/vllm-factory

What it records (all from reference functions, never from this repository's code):
  * DeBERTa log buckets: models/deberta_v2/deberta_v2_encoder.py:70 make_log_bucket_position
    over r in [-8191, 8191], and build_relative_position_v2 (:92) on a 1024 x 1024 grid
    (checked equal to the sweep);
  * T5 buckets: models/mt5/mt5_encoder.py:125 T5RelativePositionBias._relative_position_bucket
    over the same sweep;
  * DeBERTa op outputs: kernels/flash_deberta_attention.py:375 _pytorch_flash_deberta_fwd;
  * mT5 attention outputs: T5RelativePositionBias.forward (:150) +
    _make_contiguous_additive_bias (:75) + SDPA with scale 1.0, the fallback math of
    T5SelfAttention.forward (:285-316);
  * DeBERTa-v2 layer context: DisentangledSelfAttentionV2._pytorch_forward (:332) built on
    vLLM's CPU linears with the case's weights;
  * DebertaV2Intermediate.forward (:547-550): the dense layer + exact GELU, fp32;
  * GLiNER span scores: poolers/gliner.py SpanMarkerV0.forward (:133-140) with the case's
    weights, in float64, and the pooler's einsum (:289).
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import golden_inputs as gi  # noqa: E402


def _bootstrap_vllm_cpu():
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29531")
    from vllm.config import DeviceConfig, VllmConfig, set_current_vllm_config
    from vllm.distributed.parallel_state import (ensure_model_parallel_initialized,
                                                 init_distributed_environment)
    cfg = VllmConfig(device_config=DeviceConfig(device="cpu"))
    ctx = set_current_vllm_config(cfg)
    ctx.__enter__()
    init_distributed_environment(world_size=1, rank=0, local_rank=0,
                                 distributed_init_method="tcp://127.0.0.1:29531", backend="gloo")
    ensure_model_parallel_initialized(1, 1)
    return ctx


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VF_REFERENCE"),
                    help="path of a vllm-factory checkout (default: $VF_REFERENCE)")
    ap.add_argument("--out", default=str(HERE / "golden.npz"))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("make_golden.py needs a reference checkout: pass --reference or set VF_REFERENCE")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    out = {}

    # ---------------- buckets
    from models.deberta_v2.deberta_v2_encoder import (build_relative_position_v2,
                                                      make_log_bucket_position)
    from models.mt5.mt5_encoder import T5RelativePositionBias, _make_contiguous_additive_bias
    r = torch.arange(-gi.R_SWEEP, gi.R_SWEEP + 1, dtype=torch.long)
    for bs, mp in gi.DEBERTA_BUCKET_CONFIGS:
        sweep = make_log_bucket_position(r, bs, mp).to(torch.long)
        grid = build_relative_position_v2(1024, 1024, torch.device("cpu"), bucket_size=bs, max_position=mp)[0]
        # grid[i, j] = bucket(i - j): row 1023 covers r in [0, 1023], column 1023 covers [-1023, 0]
        assert torch.equal(grid[1023].flip(0), sweep[gi.R_SWEEP:gi.R_SWEEP + 1024])
        assert torch.equal(grid[:, 1023].flip(0), sweep[gi.R_SWEEP - 1023:gi.R_SWEEP + 1].flip(0))
        out[f"deberta_bucket_{bs}_{mp}"] = sweep.to(torch.int16).numpy()
    for nb, md, bidir in gi.T5_BUCKET_CONFIGS:
        b = T5RelativePositionBias._relative_position_bucket(r, bidirectional=bidir, num_buckets=nb,
                                                             max_distance=md)
        out[f"t5_bucket_{nb}_{md}_{int(bidir)}"] = b.to(torch.int16).numpy()

    # ---------------- DeBERTa op (torch fallback of the reference op), fp32
    from kernels.flash_deberta_attention import _pytorch_flash_deberta_fwd
    for name in ("deberta_log", "deberta_linear"):
        c = gi.deberta_op_case(name)
        o = _pytorch_flash_deberta_fwd(c["q"], c["k"], c["v"], c["seq_lengths"], c["pos_key"], c["pos_query"],
                                       False, c["sm_scale"], c["position_buckets"],
                                       c["max_relative_distance"], c["use_log_bucket"])
        out[f"{name}_out"] = o.float().numpy()
        for key in ("q", "k", "v", "pos_key", "pos_query"):
            out[f"{name}_sha_{key}"] = np.array(gi.sha(c[key]))

    # ---------------- mT5 attention (reference fallback math), fp32
    c = gi.t5_case("t5_enc")
    B, H, L, _ = c["q"].shape
    rpb = T5RelativePositionBias(c["num_buckets"], c["max_distance"], H)
    with torch.no_grad():
        rpb.relative_attention_bias.weight.copy_(c["table"])
        dense = rpb(L, L, torch.device("cpu"), bidirectional=True)
        bias = _make_contiguous_additive_bias(dense, c["mask"], B, H, L, L, torch.float32, torch.device("cpu"))
        o = torch.nn.functional.scaled_dot_product_attention(c["q"], c["k"], c["v"], attn_mask=bias, scale=1.0)
    out["t5_enc_out"] = o.float().numpy()
    for key in ("q", "k", "v", "table", "mask"):
        out[f"t5_enc_sha_{key}"] = np.array(gi.sha(c[key]))
    # The same path with a mask that varies over query rows ([B, 1, L, L]).
    c = gi.t5_case("t5_qmask")
    B, H, L, _ = c["q"].shape
    rpb = T5RelativePositionBias(c["num_buckets"], c["max_distance"], H)
    with torch.no_grad():
        rpb.relative_attention_bias.weight.copy_(c["table"])
        dense = rpb(L, L, torch.device("cpu"), bidirectional=True)
        bias = _make_contiguous_additive_bias(dense, c["mask"].float(), B, H, L, L, torch.float32,
                                              torch.device("cpu"))
        o = torch.nn.functional.scaled_dot_product_attention(c["q"], c["k"], c["v"], attn_mask=bias, scale=1.0)
    out["t5_qmask_out"] = o.float().numpy()
    for key in ("q", "k", "v", "table", "mask"):
        out[f"t5_qmask_sha_{key}"] = np.array(gi.sha(c[key]))

    # ---------------- DeBERTa-v2 layer (_pytorch_forward), fp32
    ctx = _bootstrap_vllm_cpu()
    from transformers import DebertaV2Config
    from models.deberta_v2.deberta_v2_encoder import DisentangledSelfAttentionV2
    c = gi.deberta_layer_case()
    E = c["hidden"].shape[-1]
    cfg = DebertaV2Config(hidden_size=E, num_attention_heads=c["num_heads"], intermediate_size=4 * E,
                          position_buckets=c["position_buckets"], max_relative_positions=c["max_relative_positions"],
                          relative_attention=True, pos_att_type=["c2p", "p2c"], share_att_key=True,
                          hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    att = DisentangledSelfAttentionV2(cfg, prefix="golden").eval()
    with torch.no_grad():
        for proj, wn, bn in ((att.query_proj, "wq", "bq"), (att.key_proj, "wk", "bk"), (att.value_proj, "wv", "bv")):
            proj.weight.copy_(c[wn])
            proj.bias.copy_(c[bn])
        hid = c["hidden"]
        qo, _ = att.query_proj(hid)
        ko, _ = att.key_proj(hid)
        vo, _ = att.value_proj(hid)
        m = c["mask"].to(torch.float32)[:, None, None, :]
        mask4 = m * m.squeeze(-2).unsqueeze(-1)  # DebertaV2Encoder.get_attention_mask
        rel_pos = build_relative_position_v2(hid.shape[1], hid.shape[1], torch.device("cpu"),
                                             bucket_size=c["position_buckets"],
                                             max_position=c["max_relative_positions"])
        ctx_out = att._pytorch_forward(qo, ko, vo, mask4, rel_pos, c["rel"])
    out["deberta_layer_out"] = ctx_out.float().numpy()
    for key in ("hidden", "wq", "wk", "wv", "rel"):
        out[f"deberta_layer_sha_{key}"] = np.array(gi.sha(c[key]))
    # ---------------- DebertaV2Intermediate (dense + ACT2FN["gelu"]), fp32
    from models.deberta_v2.deberta_v2_encoder import DebertaV2Intermediate
    c = gi.intermediate_case()
    E = c["x"].shape[-1]
    icfg = DebertaV2Config(hidden_size=E, num_attention_heads=1, intermediate_size=4 * E, hidden_act="gelu")
    inter = DebertaV2Intermediate(icfg, prefix="golden.intermediate").eval()
    with torch.no_grad():
        inter.dense.weight.copy_(c["weight"])
        inter.dense.bias.copy_(c["bias"])
        out["deberta_intermediate_out"] = inter(c["x"]).float().numpy()
    for key in ("x", "weight", "bias"):
        out[f"deberta_intermediate_sha_{key}"] = np.array(gi.sha(c[key]))
    del ctx

    # ---------------- GLiNER span marker + class einsum, float64
    from poolers.gliner import SpanMarkerV0
    c = gi.span_case()
    D = c["h"].shape[-1]
    marker = SpanMarkerV0(D, c["max_width"], dropout=0.0).double().eval()
    with torch.no_grad():
        for pre, seq in (("start", marker.project_start), ("end", marker.project_end), ("out", marker.out_project)):
            seq[0].weight.copy_(c["weights"][f"{pre}_w1"])
            seq[0].bias.copy_(c["weights"][f"{pre}_b1"])
            seq[3].weight.copy_(c["weights"][f"{pre}_w2"])
            seq[3].bias.copy_(c["weights"][f"{pre}_b2"])
        rep = marker(c["h"].double(), c["span_idx"])
        scores = torch.einsum("BLKD,BCD->BLKC", rep, c["pe"].double()).squeeze(0)
    out["gliner_span_out"] = scores.numpy()
    for key in ("h", "pe", "span_idx"):
        out[f"gliner_span_sha_{key}"] = np.array(gi.sha(c[key]))
    for key, t in sorted(c["weights"].items()):
        out[f"gliner_span_sha_{key}"] = np.array(gi.sha(t))

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {sorted(out)}")


if __name__ == "__main__":
    main()
