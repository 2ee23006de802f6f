"""Runs the reference's own attention modules with `kernels.*` resolved to this repository.

The reference's model files import their kernels as `from kernels.flash_deberta_attention
import ...` and `from kernels.flash_attention_rpb import flash_attention_rpb_final`.  With this
repository's package directory ahead of the reference install on sys.path, those imports bind
the drop-ins here, while `models.*` still comes from the reference.  Each layer is then run
three ways on the same seeded weights and inputs:

  flash       the module as shipped, whose kernel path calls this repository's CUDA operator
              (DisentangledSelfAttentionV2._flash_forward, deberta_encoder.py
              DisentangledSelfAttention._flash_forward, mt5_encoder.py T5SelfAttention.forward);
  torch_bf16  the same bf16 module forced onto the reference's own PyTorch path
              (use_flash_kernel = False; for mT5 the module-level kernel name is withdrawn,
              which is the reference's own switch to its SDPA fallback);
  torch_fp32  an fp32 copy of the module (the bf16 weights upcast) on the PyTorch path.

Prints one JSON object: per layer, the max-abs difference and the minimum per-row cosine
over the valid (unpadded) query rows of flash and torch_bf16, each against torch_fp32.

Run as a separate process (it initialises vLLM's distributed state):
    python tests/reference_modules_run.py --reference <reference install> [--device cuda]
`--device cpu` replaces the CUDA operators by the oracle (test infrastructure only), which
checks this script's plumbing without a GPU.
"""
import argparse
import contextlib
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _paths(reference):
    for p in (ROOT / "vllm-factory_b200", ROOT):
        if str(p) not in sys.path:
            sys.path.insert(0, str(p))
    sys.path.append(str(reference))


def _bootstrap_vllm(device, port):
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", str(port))
    from vllm.config import DeviceConfig, VllmConfig, set_current_vllm_config
    from vllm.distributed.parallel_state import (ensure_model_parallel_initialized,
                                                 init_distributed_environment)
    ctx = set_current_vllm_config(VllmConfig(device_config=DeviceConfig(device=device)))
    ctx.__enter__()
    init_distributed_environment(world_size=1, rank=0, local_rank=0,
                                 distributed_init_method=f"tcp://127.0.0.1:{port}", backend="gloo")
    ensure_model_parallel_initialized(1, 1)
    return ctx


def _init(module, gen, std):
    import torch
    with torch.no_grad():
        for p in module.parameters():
            p.copy_(torch.randn(p.shape, generator=gen) * std)


def _compare(out, ref, lens):
    import torch
    worst, cos_min = 0.0, 1.0
    for b, n in enumerate(lens):
        a = out[b, :n].float().cpu()
        r = ref[b, :n].float().cpu()
        worst = max(worst, (a - r).abs().max().item())
        cos_min = min(cos_min, torch.nn.functional.cosine_similarity(a, r, dim=-1).min().item())
    return {"max_abs": worst, "min_row_cos": cos_min}


def _oracle_patches():
    """CPU stand-ins for the CUDA operators, for a plumbing check without a GPU."""
    import oracle

    def deberta(q, k, v, seq_lengths, pos_key, pos_query, causal=False, sm_scale=None,
                position_buckets=256, max_relative_distance=512, use_log_bucket=True):
        return oracle.deberta_attention_ref(q, k, v, seq_lengths, pos_key, pos_query, causal, sm_scale,
                                            position_buckets, max_relative_distance, use_log_bucket).to(q.dtype)

    def rpb(q, k, v, rpb_table, num_buckets, max_distance, is_decoder, padding_mask=None,
            dropout_p=0.0, softmax_scale=1.0, use_autotune=True):
        return oracle.rpb_attention_ref(q, k, v, rpb_table, num_buckets, max_distance, is_decoder,
                                        padding_mask, softmax_scale).to(q.dtype)
    return deberta, rpb


def run(device, lens, seed=0, oracle_kernels=None):
    """`oracle_kernels` (default: on CPU) binds the oracle in place of the drop-ins, which
    skips the packed-batch and fused checks: that glue lives in the drop-ins."""
    import torch
    dev = torch.device(device)
    bf = torch.bfloat16
    B, L, T = len(lens), max(lens), sum(lens)
    mask2 = (torch.arange(L)[None, :] < torch.tensor(lens)[:, None]).to(torch.int64).to(dev)
    gen = torch.Generator().manual_seed(seed)
    results = {}
    if oracle_kernels is None:
        oracle_kernels = device == "cpu"
    patches = _oracle_patches() if oracle_kernels else None
    packed = patches is None
    if packed:
        from kernels import varlen_glue
        positions = torch.cat([torch.arange(n) for n in lens]).to(dev)

    def flatten(x):
        """(B, L, E) -> (1, T, E): the valid rows back to back, the way vLLM batches requests."""
        return torch.cat([x[b, :n] for b, n in enumerate(lens)]).unsqueeze(0)

    def compare_flat(out_flat, ref):
        padded = torch.zeros(B, L, out_flat.size(-1), dtype=out_flat.dtype, device=out_flat.device)
        for b, piece in enumerate(torch.split(out_flat[0], list(lens))):
            padded[b, :lens[b]] = piece
        return _compare(padded, ref, lens)

    def three_ways(make, layer, call, flash_on, flash_off):
        flash_on(layer)
        with torch.no_grad():
            out_flash = call(layer, bf)
        flash_off(layer)
        with torch.no_grad():
            out_bf16 = call(layer, bf)
        flash_on(layer)
        ref = make()                       # vLLM parameters do not deep-copy: build a twin
        with torch.no_grad():
            src = dict(layer.named_parameters())
            for name, p in ref.named_parameters():
                p.copy_(src[name].float().cpu())
        ref = ref.to(dev, torch.float32)
        flash_off(ref)
        with torch.no_grad():
            out_fp32 = call(ref, torch.float32)
        flash_on(ref)
        return {"flash": _compare(out_flash, out_fp32, lens), "torch_bf16": _compare(out_bf16, out_fp32, lens)}, out_fp32

    def kernel_source(res, fn):
        res["kernel_module"] = fn.__module__
        res["kernel_file"] = getattr(sys.modules[fn.__module__], "__file__", None)

    # --- DeBERTa v2 / v3 (log buckets, shared attention key)
    import models.deberta_v2.deberta_v2_encoder as v2
    from transformers import DebertaV2Config
    if patches:
        v2.flash_deberta_attention = patches[0]
        v2.HAS_FLASH_DEBERTA = True
    E, H, PB, MRP = 768, 12, 256, 512
    cfg = DebertaV2Config(hidden_size=E, num_attention_heads=H, intermediate_size=4 * E,
                          position_buckets=PB, max_relative_positions=MRP, max_position_embeddings=MRP,
                          relative_attention=True, pos_att_type=["c2p", "p2c"], share_att_key=True,
                          hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    make = lambda: v2.DisentangledSelfAttentionV2(cfg, prefix="check.v2").eval()  # noqa: E731
    att = make()
    _init(att, gen, 0.03)
    att = att.to(dev, bf)
    hid = torch.randn(B, L, E, generator=gen).to(dev)
    rel = torch.randn(2 * PB, E, generator=gen).to(dev)
    ext = mask2[:, None, None, :]
    mask4 = ext * ext.squeeze(-2).unsqueeze(-1)        # DebertaV2Encoder.get_attention_mask
    rel_pos = v2.build_relative_position_v2(L, L, dev, bucket_size=PB, max_position=MRP)
    assert att.use_flash_kernel, "the reference module did not bind a kernel"
    res, ref_v2 = three_ways(
        make, att, lambda m, dt: m(hid.to(dt), mask4, rel_pos, rel.to(dt)),
        lambda m: setattr(m, "use_flash_kernel", True), lambda m: setattr(m, "use_flash_kernel", False))
    kernel_source(res, v2.flash_deberta_attention)
    if packed:
        # A flat batch (mask all ones) inside packed_batch: the requests are kept apart.
        ones4 = torch.ones(1, 1, T, T, dtype=torch.int64, device=dev)
        rel_pos_t = v2.build_relative_position_v2(T, T, dev, bucket_size=PB, max_position=MRP)
        flat_call = lambda: att(flatten(hid).to(bf), ones4, rel_pos_t, rel.to(bf))  # noqa: E731
        with torch.no_grad(), varlen_glue.packed_batch(positions):
            res["packed"] = compare_flat(flat_call(), ref_v2)
        # The fused position mode installed on the reference's class: padded, then packed.
        varlen_glue.install_fused_positions(v2.DisentangledSelfAttentionV2)
        try:
            with torch.no_grad():
                res["fused"] = _compare(att(hid.to(bf), mask4, rel_pos, rel.to(bf)), ref_v2, lens)
                with varlen_glue.packed_batch(positions):
                    res["fused_packed"] = compare_flat(flat_call(), ref_v2)
        finally:
            v2.DisentangledSelfAttentionV2._flash_forward = v2.DisentangledSelfAttentionV2._vf_reference_flash_forward
            del v2.DisentangledSelfAttentionV2._vf_reference_flash_forward
    results["deberta_v2"] = res

    if packed:
        # DebertaV2Intermediate (dense + exact GELU) with the GEMM-epilogue GELU installed on the
        # reference's class, against its own bf16 forward and an fp32 twin.
        from kernels import linear_act
        make_i = lambda: v2.DebertaV2Intermediate(cfg, prefix="check.intermediate").eval()  # noqa: E731
        inter = make_i()
        _init(inter, gen, 0.03)
        inter = inter.to(dev, bf)
        x_i = torch.randn(B, L, E, generator=gen).to(dev)
        twin = make_i()
        with torch.no_grad():
            src = dict(inter.named_parameters())
            for name, p in twin.named_parameters():
                p.copy_(src[name].float().cpu())
            twin = twin.to(dev, torch.float32)
            ref_i = twin(x_i)
            theirs = inter(x_i.to(bf))
            linear_act.install_fused_intermediate(v2.DebertaV2Intermediate)
            try:
                ours = inter(x_i.to(bf))
            finally:
                v2.DebertaV2Intermediate.forward = v2.DebertaV2Intermediate._vf_reference_forward
                del v2.DebertaV2Intermediate._vf_reference_forward
        results["deberta_v2_intermediate"] = {"fused": _compare(ours, ref_i, lens),
                                              "torch_bf16": _compare(theirs, ref_i, lens),
                                              "kernel_module": linear_act.linear_gelu.__module__,
                                              "kernel_file": linear_act.__file__}

    # --- DeBERTa v1 (linear positions, separate position projections)
    import models.deberta.deberta_encoder as v1
    from transformers import DebertaConfig
    if patches:
        v1.flash_deberta_attention = patches[0]
        v1.HAS_FLASH_DEBERTA = True
    cfg1 = DebertaConfig(hidden_size=E, num_attention_heads=H, intermediate_size=4 * E,
                         max_position_embeddings=MRP, relative_attention=True, max_relative_positions=-1,
                         pos_att_type=["c2p", "p2c"], hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    make1 = lambda: v1.DisentangledSelfAttention(cfg1, prefix="check.v1").eval()  # noqa: E731
    att1 = make1()
    _init(att1, gen, 0.03)
    att1 = att1.to(dev, bf)
    rel1 = torch.randn(2 * MRP, E, generator=gen).to(dev)
    rel_pos1 = v1.build_relative_position(L, L, dev)
    assert att1.use_flash_kernel, "the reference module did not bind a kernel"
    res, ref_v1 = three_ways(
        make1, att1, lambda m, dt: m(hid.to(dt), mask4, rel_pos1, rel1.to(dt)),
        lambda m: setattr(m, "use_flash_kernel", True), lambda m: setattr(m, "use_flash_kernel", False))
    kernel_source(res, v1.flash_deberta_attention)
    if packed:
        ones4 = torch.ones(1, 1, T, T, dtype=torch.int64, device=dev)
        with torch.no_grad(), varlen_glue.packed_batch(positions):
            out = att1(flatten(hid).to(bf), ones4, v1.build_relative_position(T, T, dev), rel1.to(bf))
        res["packed"] = compare_flat(out, ref_v1)
    results["deberta_v1"] = res

    # --- mT5 encoder self-attention (T5 buckets, additive padding mask, output projection)
    import models.mt5.mt5_encoder as t5
    if patches:
        t5.flash_attention_rpb_final = patches[1]
    if device == "cpu":
        # The fallback's sdpa_kernel(EFFICIENT_ATTENTION, MATH) passes MATH as torch's
        # `set_priority` flag, leaving only the memory-efficient backend, which has no CPU
        # kernel; the plumbing check lets torch pick its backend instead.
        t5.sdpa_kernel = lambda *a, **k: contextlib.nullcontext()
    kernel = t5.flash_attention_rpb_final
    D_MODEL, TH = 512, 8
    make5 = lambda: t5.T5SelfAttention(D_MODEL, TH, 64, 0.0, None, None, prefix="check.t5",  # noqa: E731
                                       use_rpb=True, rpb_num_buckets=32, rpb_max_distance=128,
                                       is_decoder=False).eval()
    att5 = make5()
    _init(att5, gen, 0.03)
    with torch.no_grad():
        att5.rpb.relative_attention_bias.weight.normal_(0.0, 1.0, generator=gen)
    att5 = att5.to(dev, bf)
    hid5 = torch.randn(B, L, D_MODEL, generator=gen).to(dev)

    def call5(m, dt):
        pad = mask2[:, None, None, :].to(dt)
        pad = (1.0 - pad) * torch.finfo(dt).min            # T5Stack.forward's broadcast mask
        return m(hid5.to(dt), rpb_table=m.rpb.relative_attention_bias.weight.contiguous(), attention_mask=pad)

    def t5_on(_m):
        t5.flash_attention_rpb_final = kernel

    def t5_off(_m):
        t5.__dict__.pop("flash_attention_rpb_final", None)

    res, ref_t5 = three_ways(make5, att5, call5, t5_on, t5_off)
    kernel_source(res, kernel)
    if packed:
        zero = torch.zeros(1, 1, 1, T, dtype=bf, device=dev)   # mt5_gliner's flat call: mask all ones
        with torch.no_grad(), varlen_glue.packed_batch(positions):
            out = att5(flatten(hid5).to(bf), rpb_table=att5.rpb.relative_attention_bias.weight.contiguous(),
                       attention_mask=zero)
        res["packed"] = compare_flat(out, ref_t5)
    results["mt5"] = res
    return results


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("VF_REFERENCE", str(ROOT / "baseline" / "_ref")))
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--lens", default="384,250,17")
    ap.add_argument("--port", type=int, default=29547)
    args = ap.parse_args()
    _paths(args.reference)
    import torch
    torch.manual_seed(0)
    ctx = _bootstrap_vllm(args.device, args.port)
    res = run(args.device, [int(x) for x in args.lens.split(",")])
    print("RESULT " + json.dumps(res))
    del ctx


if __name__ == "__main__":
    main()
