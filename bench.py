"""Benchmark of the relative-position attention hot path (one JSON line on rank 0).

Default run: the headline is one mT5-large encoder self-attention layer with the T5
relative-position bias, bf16, 16 sequences x 768 positions (valid lengths ~ U[256, 768],
right padding), 16 heads x 64.  A "step" is one call of the drop-in
`kernels.flash_attention_rpb.flash_attention_rpb_final` on that batch.  The same run adds
two sub-results with the same keys: the DeBERTa-v3-large disentangled attention layer
(8 x 512, U[64, 512]; the fused mode, whose position contractions run inside the kernel,
when the build has it) and the 24-layer DeBERTa-v3-large encoder stack over 256 packed
sequences (encoder tokens/s).

  value        attention TFLOP/s over the whole job (valid work: 4*H*D*sum L_i^2, plus the
               position contractions 4*H*D*sum L_i*P(L_i) where the kernel does them),
               inputs resident in HBM; each step reads a different input set (the rotation
               spans > 3x the 126 MB L2), so no step is served from L2.
  e2e          the same metric through the same public call with pinned HOST buffers:
               every step copies the inputs host->device and the output device->host
               inside the timed region; copies of neighbouring steps overlap the compute
               (upload, compute and download streams, two device slots).
  roofline     dominant kernel vs the measured dense bf16 peak (MEASURED_PEAKS.json).
  cpu_baseline the oracle (CPU restatement of the reference's torch path) on this host.

Multi-GPU (torchrun, one process per GPU): for the attention lines every rank runs its own
batch with the same valid lengths as rank 0's (weak scaling); the encoder stack splits one
256-sequence batch over the ranks by LPT on estimated FLOPs (strong scaling).  NCCL carries
only the barrier and the max-time / summed-work reductions.  `--impl reference` times the
reference's CPU implementation (the oracle port) on rank 0 and prints the same metric with
the same `config`.  `--impl reference_triton` times the reference's own Triton kernels on
one GPU on the same input sets (a secondary bar beside the CPU reference arm).

Named workloads (`--workload`): mt5_c2, mt5_c2_varlen, deberta_c1[_fused], deberta_c1_fp32,
deberta_c1_varlen[_fused], deberta_c5_<L>[_fused] (L = 1024, 2048, 4096), the encoder
stacks deberta_c3 / mt5_c4, the HBM-bound ops beside the path, mt5_ffn_act /
deberta_add_ln (value = GB/s), the feed-forward GEMMs with the activation in the
epilogue, deberta_ffn_gemm / mt5_ffn_gemm (TFLOP/s), and the GLiNER span head downstream
of the encoder, gliner_span (value = spans/s).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "vllm-factory_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

L2_BYTES = 126 * 1024 * 1024
METRIC = "RPB attention TFLOP/s (% bf16 peak); encoder tokens/s at 1/2/4/8 B200"


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return dict(bf16=d["bf16_tflops"], bf16_sustained=d["bf16_tflops_sustained"], hbm=d["hbm_gbs"],
                    source="measured")
    return dict(bf16=1590.0, bf16_sustained=1400.0, hbm=6650.0, source="fallback")


def committed_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d.get(workload)
    return None


def pipelined_e2e(dev, host: dict, call, n_steps: int, world: int):
    """End-to-end time of `n_steps` calls through the public op with host buffers: every
    step copies its inputs (the tensors of `host`, pinned) to the device and its result
    back to pinned host memory, inside the timed region.  As a serving loop would, the
    copies of neighbouring steps overlap the compute: uploads on one stream into two
    device slots, compute on the current stream, downloads on a third; events order each
    slot's upload after the compute that last read it, each compute after its upload and
    each download after its compute.  Returns (max-over-ranks ms, h2d bytes, d2h bytes)."""
    cur = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    keys = [k for k, v in host.items() if isinstance(v, torch.Tensor)]
    # Device slots and pinned outputs take the strides of their source (the DeBERTa inputs are
    # permuted views of a projection, as the reference's caller builds them), so each copy is
    # one asynchronous memcpy of the dense block, not a host-side transpose through pageable
    # memory.
    slots = [{k: torch.empty_strided(host[k].size(), host[k].stride(), dtype=host[k].dtype, device=dev)
              for k in keys} for _ in range(2)]
    probe = call({**host, **{k: slots[0][k].copy_(host[k]) for k in keys}})
    outs = [torch.empty_strided(probe.size(), probe.stride(), dtype=probe.dtype, pin_memory=True) for _ in range(2)]
    torch.cuda.synchronize()
    h2d = sum(host[k].numel() * host[k].element_size() for k in keys)
    d2h = outs[0].numel() * outs[0].element_size()

    def run(n):
        done = [None, None]                        # compute event of the last step per slot
        copied = [None, None]                      # download event of the last step per output
        for i in range(n):
            s = i % 2
            with torch.cuda.stream(up):
                if done[s] is not None:
                    up.wait_event(done[s])
                for k in keys:
                    slots[s][k].copy_(host[k], non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(up)
            cur.wait_event(ready)
            o = call({**host, **slots[s]})
            done[s] = torch.cuda.Event()
            done[s].record(cur)
            with torch.cuda.stream(down):
                down.wait_event(done[s])
                if copied[s] is not None:
                    down.wait_event(copied[s])
                outs[s].copy_(o, non_blocking=True)
                o.record_stream(down)
                copied[s] = torch.cuda.Event()
                copied[s].record(down)
        for ev in copied:
            if ev is not None:
                cur.wait_event(ev)

    run(2)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    up.wait_event(e0)
    down.wait_event(e0)
    run(n_steps)
    e1.record(cur)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    return ms.item(), h2d, d2h


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- workloads
ATTN_WORKLOADS = ("mt5_c2", "mt5_c2_varlen", "deberta_c1", "deberta_c1_fp32", "deberta_c1_varlen",
                  "deberta_c1_fused", "deberta_c1_varlen_fused", "deberta_c5_1024", "deberta_c5_2048",
                  "deberta_c5_4096", "deberta_c5_1024_fused", "deberta_c5_2048_fused", "deberta_c5_4096_fused")
COMPAT_NOTE = ("compat: the caller's pos_key = Q.Kr^T / pos_query = K.Qr^T products (cuBLAS) are inputs, "
               "made outside the kernel; FLOPs count QK^T + PV only")
FUSED_NOTE = ("fused: rel_key / rel_query in, Q.Kr^T and K.Qr^T on tcgen05 inside the kernel; "
              "FLOPs count QK^T + PV + both position contractions at their distinct-index width")


def attention_config(name: str) -> dict:
    """The `config` object of an attention workload; both arms print the same one."""
    if name.startswith("mt5_c2"):
        cfg = {"workload": "mT5-large encoder self-attention layer, T5 RPB 32 buckets / max_distance 128",
               "global_batch": 16, "seq_len": 768, "heads": 16, "head_dim": 64,
               "lengths": "U[256,768] right-padded"}
        if name == "mt5_c2_varlen":
            cfg["workload"] += ", packed (cu_seqlens)"
            cfg["lengths"] = "U[256,768] packed, no padding"
        return cfg
    if name.startswith("deberta_c1"):
        cfg = {"workload": "DeBERTa-v3-large disentangled self-attention layer, c2p|p2c, 256 buckets / max_rel 512",
               "global_batch": 8, "seq_len": 512, "heads": 16, "head_dim": 64, "lengths": "U[64,512] right-padded"}
        if name == "deberta_c1_fp32":
            cfg["workload"] += ", fp32 tensors in and out"
        if "varlen" in name:
            cfg["workload"] += ", packed (cu_seqlens)"
            cfg["lengths"] = "U[64,512] packed, no padding"
        cfg["mode"] = FUSED_NOTE if name.endswith("_fused") else COMPAT_NOTE
        return cfg
    if name.startswith("deberta_c5"):
        L = int(name.split("_")[2])
        return {"workload": f"DeBERTa long-context disentangled attention, seq {L}, full length",
                "global_batch": 16384 // L, "seq_len": L, "heads": 16, "head_dim": 64,
                "mode": FUSED_NOTE if name.endswith("_fused") else COMPAT_NOTE}
    if name in ENCODER_NAMES:
        from vf_b200 import encoders as EN
        tokens = int(encoder_setup(name)[2].sum())
        return {"workload": ENCODER_NAMES[name], "sequences": 256, "layers": 24, "tokens": tokens,
                "lengths": "U[128,768]" if name == "deberta_c3" else "U[512,768]",
                "partition": "packed batch, LPT by estimated FLOPs over ranks"}
    raise SystemExit(f"unknown workload {name}")


def build_workload(name: str, rank: int, device):
    """Returns (list of input dicts, call(inputs) -> out, flops per step, tokens per step, config,
    keys copied per step, lengths, launches per step).  Weak scaling: rank r's batch has the
    valid lengths of rank 0's batch (rotated) and its own seeded values."""
    from vf_b200 import workloads as W

    cfg = attention_config(name)
    launches = 1
    if name == "mt5_c2":
        from kernels.flash_attention_rpb import flash_attention_rpb_final
        base = W.mt5_attention_inputs(seed=1000 + rank, device=device, lengths=W.rank_lengths("mt5", rank))
        lens = base["lengths"].tolist()
        flops = W.core_flops(lens)

        def call(x):
            return flash_attention_rpb_final(x["q"], x["k"], x["v"], x["rpb_table"], 32, 128, False,
                                             x["padding_mask"], 0.0, 1.0)

        per_set = sum(base[k].numel() * base[k].element_size() for k in ("q", "k", "v")) * 4 // 3
        keys = ("q", "k", "v", "rpb_table", "padding_mask")
    elif name == "mt5_c2_varlen":
        from kernels.flash_attention_rpb import flash_attention_rpb_varlen
        base = W.mt5_varlen_inputs(seed=1000 + rank, device=device, lengths=W.rank_lengths("mt5", rank))
        lens = base["lengths"].tolist()
        flops = W.core_flops(lens)

        def call(x):
            return flash_attention_rpb_varlen(x["q"], x["k"], x["v"], x["cu_seqlens"], x["max_seqlen"],
                                              x["rpb_table"], 32, 128, False, 1.0)

        per_set = sum(base[k].numel() * base[k].element_size() for k in ("q", "k", "v")) * 4 // 3
        keys = ("q", "k", "v", "rpb_table", "cu_seqlens")
    elif name.startswith("deberta_c1_varlen"):
        from kernels.flash_deberta_attention import flash_deberta_attention_varlen
        fused = name.endswith("_fused")
        base = W.deberta_varlen_inputs(seed=2000 + rank, device=device, lengths=W.rank_lengths("deberta", rank))
        lens = base["lengths"].tolist()
        flops = W.core_flops(lens) + (W.deberta_pos_flops(lens) if fused else 0.0)
        if fused:
            keys = ("q", "k", "v", "rel_key", "rel_query", "cu_seqlens")
            launches = 2

            def call(x):
                return flash_deberta_attention_varlen(x["q"], x["k"], x["v"], x["cu_seqlens"], x["max_seqlen"],
                                                      None, None, False, x["sm_scale"], 256, 512, True,
                                                      rel_key=x["rel_key"], rel_query=x["rel_query"])
        else:
            keys = ("q", "k", "v", "pos_key", "pos_query", "cu_seqlens")

            def call(x):
                return flash_deberta_attention_varlen(x["q"], x["k"], x["v"], x["cu_seqlens"], x["max_seqlen"],
                                                      x["pos_key"], x["pos_query"], False, x["sm_scale"], 256, 512,
                                                      True)
        per_set = sum(base[k].numel() * base[k].element_size() for k in keys if k != "cu_seqlens")
    elif name.startswith("deberta_c1") or name.startswith("deberta_c5"):
        from kernels.flash_deberta_attention import flash_deberta_attention
        fused = name.endswith("_fused")
        if name.startswith("deberta_c1"):
            dt = torch.float32 if name == "deberta_c1_fp32" else torch.bfloat16
            base = W.deberta_attention_inputs(seed=2000 + rank, device=device, dtype=dt,
                                              lengths=W.rank_lengths("deberta", rank))
            if dt == torch.float32:
                cfg["_dtype"] = "f32"
        else:
            L = int(name.split("_")[2])
            base = W.deberta_attention_inputs(seed=3000 + rank, device=device, B=16384 // L, L=L,
                                              lengths=[L] * (16384 // L))
        lens = base["lengths"].tolist()
        flops = W.core_flops(lens) + (W.deberta_pos_flops(lens) if fused else 0.0)
        if fused:
            keys = ("q", "k", "v", "rel_key", "rel_query", "seq_lengths")
            launches = 2

            def call(x):
                return flash_deberta_attention(x["q"], x["k"], x["v"], x["seq_lengths"], None, None, False,
                                               x["sm_scale"], 256, 512, True, rel_key=x["rel_key"],
                                               rel_query=x["rel_query"])
        else:
            keys = ("q", "k", "v", "pos_key", "pos_query", "seq_lengths")

            def call(x):
                return flash_deberta_attention(x["q"], x["k"], x["v"], x["seq_lengths"], x["pos_key"],
                                               x["pos_query"], False, x["sm_scale"], 256, 512, True)
        per_set = sum(base[k].numel() * base[k].element_size() for k in keys if k != "seq_lengths")
    else:
        raise SystemExit(f"unknown workload {name}")

    n_sets = max(1, math.ceil(3 * L2_BYTES / per_set))
    sets = [base]
    for _ in range(n_sets - 1):
        sets.append({k: (v.clone() if isinstance(v, torch.Tensor) and v.is_cuda and k in keys else v)
                     for k, v in base.items()})
    cfg["_l2"] = f"{n_sets} rotating input sets ({per_set / 2**20:.0f} MiB each) > 3x L2; no flush"
    return sets, call, flops, float(sum(lens)), cfg, keys, lens, launches


def cpu_baseline(name: str, lens, budget_s: float = 12.0):
    """Times the oracle (CPU restatement of the reference's torch path) on a bounded sample."""
    import oracle
    from vf_b200 import workloads as W
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    if name.startswith("mt5_c2"):
        x = W.mt5_attention_inputs(seed=1000, device="cpu")
        flops_done, t0, n = 0.0, time.perf_counter(), 0
        while True:
            b = n % x["q"].shape[0]
            sl = slice(b, b + 1)
            oracle.rpb_attention_ref(x["q"][sl].float(), x["k"][sl].float(), x["v"][sl].float(),
                                     x["rpb_table"].float(), 32, 128, False, x["padding_mask"][sl].float(), 1.0,
                                     dtype=torch.float32)
            flops_done += W.core_flops([int(x["lengths"][b])])
            n += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
        sample = f"{n} sequences of the C2 batch, one at a time, fp32 torch on CPU (oracle port of the reference's SDPA path)"
    else:
        # Compat lines: the op's own work (pos_key / pos_query are inputs), core FLOPs only.
        # Fused lines: the position products Q.Kr^T and K.Qr^T run inside the timed loop too
        # (as the reference's caller does them), core + position FLOPs.
        fused = name.endswith("_fused")
        x = W.deberta_attention_inputs(seed=2000, device="cpu")
        flops_done, t0, n = 0.0, time.perf_counter(), 0
        while True:
            b = n % x["q"].shape[0]
            sl = slice(b, b + 1)
            q, k = x["q"][sl].float(), x["k"][sl].float()
            if fused:
                pk = torch.matmul(q, x["rel_key"].float().transpose(-1, -2))
                pq = torch.matmul(k, x["rel_query"].float().transpose(-1, -2))
            else:
                pk, pq = x["pos_key"][sl].float(), x["pos_query"][sl].float()
            oracle.deberta_attention_ref(q, k, x["v"][sl].float(), x["seq_lengths"][sl], pk, pq,
                                         False, x["sm_scale"], 256, 512, True, dtype=torch.float32)
            L = int(x["lengths"][b])
            flops_done += W.core_flops([L]) + (W.deberta_pos_flops([L]) if fused else 0.0)
            n += 1
            if time.perf_counter() - t0 > budget_s:
                break
        dt = time.perf_counter() - t0
        sample = (f"{n} sequences of the C1 batch, fp32 torch on CPU (oracle port of the reference's op fallback"
                  + (", with the caller's two position products)" if fused else ")"))
    return {"value": flops_done / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": sample}


# ----------------------------------------------------------------------------- encoder stacks
ENCODER_WORKLOADS = ("deberta_c3", "mt5_c4")
ENCODER_NAMES = {"deberta_c3": "DeBERTa-v3-large 24-layer encoder stack, 256 packed sequences",
                 "mt5_c4": "mT5-large 24-layer encoder stack, 256 packed sequences"}


def encoder_setup(name: str):
    """(model class, config, lengths, ids, attention FLOPs per layer of one sequence)."""
    from vf_b200 import encoders as EN
    from vf_b200 import workloads as W
    if name == "deberta_c3":
        cfg = EN.DebertaConfig()
        lengths, ids = EN.packed_batch(256, 128, 768, cfg.vocab, seed=0)
        attn = lambda L: W.core_flops([L]) + W.deberta_pos_flops([L])
        return EN.DebertaV3Encoder, cfg, lengths, ids, attn
    cfg = EN.MT5Config()
    lengths, ids = EN.packed_batch(256, 512, 768, cfg.vocab, seed=0)
    return EN.MT5Encoder, cfg, lengths, ids, lambda L: W.core_flops([L])


def encoder_cpu_baseline(name: str, budget_s: float = 15.0):
    """The stack's layers on the host cores (fp32, the oracle's attention), on the first
    sequences of the batch, 2 layers: encoder tokens/s per layer, as a reported baseline."""
    import dataclasses

    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    cls, cfg, lengths, ids, _ = encoder_setup(name)
    from vf_b200 import encoders as EN
    small = dataclasses.replace(cfg, layers=2)
    if name == "deberta_c3":
        fn = lambda q, k, v, cu, ms, pk, pq, c, sm, pb, mr, lg: oracle.deberta_attention_varlen_ref(
            q, k, v, cu, pk, pq, c, sm, pb, mr, lg, dtype=torch.float32)
    else:
        fn = lambda q, k, v, cu, ms, t, nb, md, dec, sc: oracle.rpb_attention_varlen_ref(
            q, k, v, cu, t, nb, md, dec, sc, dtype=torch.float32)
    extra = ({"add_norm": lambda x, r, w, b, eps: oracle.add_layer_norm_ref(x, r, w, b, eps),
              "act_fn": lambda x: oracle.gated_act_ref(x, None, 1)} if name == "deberta_c3"
             else {"gated_act": lambda g, u, a: oracle.gated_act_ref(g, u, 0)})
    if name == "deberta_c3":
        extra["fused_positions"] = False   # the reference's caller forms q . Kr and k . Qr itself
    model = cls(small, device="cpu", dtype=torch.float32, seed=0, attention_fn=fn, **extra)
    done, n, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s and n < len(lengths):
        x, cu, lens = EN.select_sequences(lengths, ids, [n])
        model.forward(x, cu, lens[0])
        done += lens[0]
        n += 1
    dt = time.perf_counter() - t0
    return {"value": done * small.layers / dt, "unit": "tokens/s per layer", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"first {n} sequences, 2 layers, fp32 torch on CPU with the oracle's attention"}


def run_encoder(args, name: str, steps: int, world: int, rank: int, dev, warmup: int, cpu_base: bool):
    """C3 / C4: the 256-sequence packed batch is partitioned by sequence over the ranks
    (LPT on estimated FLOPs), each rank runs the 24-layer stack on its shard; value =
    encoder tokens/s of the whole job (total valid tokens / max rank time).  Every rank
    takes the same collective steps; rank 0 gets the line, the others None."""
    from vf_b200 import dist as VD
    from vf_b200 import encoders as EN
    cls, cfg, lengths, ids, attn = encoder_setup(name)
    model = cls(cfg, device=dev, seed=0)
    gemm_tok = model.flops_per_token_gemm()
    costs = [gemm_tok * int(L) + cfg.layers * attn(int(L)) for L in lengths.tolist()]
    mine = VD.lpt_shard(costs, world)[rank]
    x_ids, cu, lens = EN.select_sequences(lengths, ids, mine)
    x_dev, cu_dev, max_len = x_ids.to(dev), cu.to(dev), max(lens)
    flops = sum(costs[i] for i in mine)
    tokens = float(sum(lens))
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for _ in range(warmup):
        model.forward(x_dev, cu_dev, max_len)
    torch.cuda.synchronize()
    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        model.forward(x_dev, cu_dev, max_len)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    ms_max, flops_all, tokens_all = VD.reduce_timing(ms, flops, tokens, dev)
    value = tokens_all * steps / (ms_max * 1e-3)

    e2e = None
    if not args.no_e2e:
        host = {"ids": x_ids.pin_memory(), "cu": cu.pin_memory()}
        n_e2e = max(3, min(steps, 10))
        ems, h2d, d2h = pipelined_e2e(dev, host, lambda x: model.forward(x["ids"], x["cu"], max_len), n_e2e, world)
        barrier()
        e2e = {"value": tokens_all * n_e2e / (ems * 1e-3), "unit": "tokens/s", "pipelined": True,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": n_e2e}
    if rank != 0:
        return None
    peaks = measured_peaks()
    achieved = flops / (ms / steps * 1e-3) / 1e12
    cfg_line = attention_config(name)
    cfg_line["tokens"] = int(lengths.sum())
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg_line,
            "l2": "weights (>0.8 GB) and activations exceed L2; no flush",
            "attention_flops_share": sum(cfg.layers * attn(int(lengths[i])) for i in mine) / flops,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_sustained"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16_sustained"], "traffic": None,
                         "peak_source": f"{peaks['source']} bf16 dense (sustained: a 24-layer step runs for seconds)",
                         "what": "whole stack: GEMM + attention algorithmic FLOPs of rank 0's shard per second"},
            "gpu_launches": steps * cfg.layers * model.own_launches_per_layer(), "clocks": clocks, "e2e": e2e}
    if world == 1 and cpu_base:
        line["cpu_baseline"] = encoder_cpu_baseline(name)
    return line


# ----------------------------------------------------------------------------- FFN activation
def gated_act_cpu_baseline(budget_s: float = 10.0):
    """The oracle of the reference's kernel arithmetic (fp32 torch) on the host cores over
    a 2048-row slice of the workload, repeated for ~10 s: GB/s of the same bytes."""
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(4000)
    gu = (torch.randn(2048, 2 * 2816, generator=g) * 2).to(torch.bfloat16)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        oracle.gated_act_ref(gu[:, :2816], gu[:, 2816:], 0)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n * 3 * 2048 * 2816 * 2 / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} x 2048 rows of the 16384 x 2816 workload, fp32 torch on CPU (oracle)"}


def add_layer_norm_cpu_baseline(budget_s: float = 10.0):
    """The oracle of the reference's two calls (float64 torch) on the host cores over a
    2048-row slice of the workload, repeated for ~10 s: GB/s of the same bytes."""
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(5000)
    x, r = (torch.randn(2048, 1024, generator=g).to(torch.bfloat16) for _ in range(2))
    w, b = torch.ones(1024, dtype=torch.bfloat16), torch.zeros(1024, dtype=torch.bfloat16)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        oracle.add_layer_norm_ref(x, r, w, b, 1e-7)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n * 3 * 2048 * 1024 * 2 / dt / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} x 2048 rows of the 65536 x 1024 workload, float64 torch on CPU (oracle)"}


def _run_hbm_op(args, world: int, rank: int, dev, warmup: int, sets, call, nbytes: int, cfg: dict, cpu_fn,
                bound: str = "hbm"):
    """Shared timing of the ops beside the path: `call(*sets[i % len(sets)])` per step.
    bound "hbm": value = algorithmic bytes (`nbytes`) / time in GB/s against the measured
    HBM copy; bound "tensor": `nbytes` holds the algorithmic FLOPs, value in TFLOP/s against
    the measured bf16 GEMM peak.  The host time of one op call (Python, dispatch, output
    allocation) exceeds the elementwise kernels' device time, so the K timed steps are
    captured once in a CUDA graph and the replay is timed: all K launches run, back to back.
    e2e: eager calls, the first input set from pinned host memory in, the result out, every
    step."""
    stream = torch.cuda.current_stream(dev)
    for i in range(warmup):
        call(*sets[i % len(sets)])
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(args.steps):
            call(*sets[i % len(sets)])
    graph.replay()                                   # one untimed replay
    torch.cuda.synchronize()
    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    graph.replay()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)
    from vf_b200 import dist as VD
    ms_max, bytes_all, _ = VD.reduce_timing(ms, float(nbytes), 0.0, dev)
    div, unit = (1e9, "GB/s") if bound == "hbm" else (1e12, "TFLOP/s")
    value = bytes_all * args.steps / (ms_max * 1e-3) / div
    e2e = None
    if not args.no_e2e:
        host = {str(j): t.cpu().pin_memory() for j, t in enumerate(sets[0])}
        n_e2e = max(3, min(args.steps, 10))
        ems, h2d, d2h = pipelined_e2e(dev, host, lambda x: call(*(x[str(j)] for j in range(len(host)))), n_e2e, world)
        e2e = {"value": bytes_all * n_e2e / (ems * 1e-3) / div, "unit": unit, "pipelined": True,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": n_e2e}
    if rank != 0:
        return None
    peaks = measured_peaks()
    achieved = nbytes / (ms / args.steps * 1e-3) / div
    if bound == "hbm":
        peak, src, work = peaks.get("hbm", 6650.0), f"{peaks['source']} HBM copy", "algorithmic_bytes_per_launch"
    else:
        peak, src, work = peaks["bf16"], f"{peaks['source']} bf16 GEMM (burst)", "algorithmic_flops_per_launch"
    return {"metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": cfg,
            "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                         "frac": achieved / peak, "traffic": committed_traffic(args.workload),
                         "peak_source": src, work: nbytes},
            "gpu_launches": args.steps, "clocks": clocks, "e2e": e2e,
            **({"cpu_baseline": cpu_fn()} if world == 1 and not args.no_cpu_baseline else {})}


def run_gated_act(args, world: int, rank: int, dev, warmup: int):
    """mt5_ffn_act: the gated-GELU of one mT5-large FFN (kernels.ff_fused drop-in) on the
    two halves of a stacked [16384, 2 x 2816] bf16 projection, read in place.  HBM-bound:
    value = bytes moved (gate + up read, out written) / time, in GB/s."""
    from kernels.ff_fused import fused_gelu_mul_dropout
    T, Fd = 16384, 2816
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    sets = [((torch.randn(T, 2 * Fd, generator=g, device=dev) * 2).to(torch.bfloat16),) for _ in range(3)]
    call = lambda gu: fused_gelu_mul_dropout(gu[:, :Fd], gu[:, Fd:], "gelu_new")
    cfg = {"workload": "mT5-large FFN gated-GELU (kernels/ff_fused.py drop-in), 16384 x 2816, halves of a stacked projection",
           "l2": "3 rotating 185 MB input sets > L2; no flush", "launch": "K steps in one CUDA graph"}
    return _run_hbm_op(args, world, rank, dev, warmup, sets, call, 3 * T * Fd * 2, cfg, gated_act_cpu_baseline)


def run_add_layer_norm(args, world: int, rank: int, dev, warmup: int):
    """deberta_add_ln: LayerNorm(x + residual) of a DeBERTa-v3-large layer output
    (kernels.fused_add_layernorm drop-in for deberta_v2_encoder.py:507 / :566) over 65536
    packed tokens x 1024, bf16.  HBM-bound: value = bytes moved (x, residual read, out
    written) / time, in GB/s."""
    from kernels.fused_add_layernorm import fused_add_layer_norm
    T, E = 65536, 1024
    g = torch.Generator(device=dev).manual_seed(5000 + rank)
    sets = [tuple(torch.randn(T, E, generator=g, device=dev).to(torch.bfloat16) for _ in range(2)) for _ in range(2)]
    w = (1.0 + 0.1 * torch.randn(E, generator=g, device=dev)).to(torch.bfloat16)
    b = (0.1 * torch.randn(E, generator=g, device=dev)).to(torch.bfloat16)
    call = lambda x, r: fused_add_layer_norm(x, r, w, b, 1e-7)
    cfg = {"workload": "DeBERTa-v3-large residual add + LayerNorm (kernels/fused_add_layernorm.py), 65536 x 1024",
           "l2": "2 rotating 256 MB input sets > L2; no flush", "launch": "K steps in one CUDA graph"}
    return _run_hbm_op(args, world, rank, dev, warmup, sets, call, 3 * T * E * 2, cfg, add_layer_norm_cpu_baseline)


FFN_GEMM_SHAPES = {"deberta_ffn_gemm": (65536, 1024, 4096), "mt5_ffn_gemm": (65536, 1024, 2816)}


def ffn_gemm_cpu_baseline(name: str, budget_s: float = 10.0):
    """The oracle's unfused arithmetic (float64 torch: projection, then the activation) on
    the host cores over a 256-row slice of the workload, repeated for ~10 s: TFLOP/s of the
    same GEMM work."""
    import oracle
    torch.set_num_threads(os.cpu_count() or 1)
    M, K, N = FFN_GEMM_SHAPES[name]
    rows = 256
    g = torch.Generator().manual_seed(6000)
    x = torch.randn(rows, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.03).to(torch.bfloat16)
    b = (torch.randn(N, generator=g) * 0.1).to(torch.bfloat16)
    up = torch.randn(rows, N, generator=g).to(torch.bfloat16)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s:
        if name == "deberta_ffn_gemm":
            oracle.linear_gelu_ref(x, w, b)
        else:
            oracle.gated_act_ref(x.double() @ w.double().t(), up, 0)   # 0: GELU_tanh (oracle/ffn.py)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": n * 2.0 * rows * N * K / dt / 1e12, "unit": "TFLOP/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"{n} x {rows} rows of the {M} x {N} x {K} workload, float64 torch on CPU (oracle)"}


def ffn_gemm_config(name: str) -> dict:
    M, K, N = FFN_GEMM_SHAPES[name]
    what = ("DeBERTa-v3-large FFN dense + exact GELU (kernels/linear_act.py linear_gelu)" if name == "deberta_ffn_gemm"
            else "mT5-large gate projection x GELU_tanh x up (kernels/linear_act.py gated_gelu_tanh)")
    return {"workload": f"{what}, {M} x {K} -> {N}, bf16",
            "l2": "2 rotating input sets (x 128 MB, outputs 368-512 MB) > L2; no flush",
            "launch": "K steps in one CUDA graph"}


def run_ffn_gemm(args, world: int, rank: int, dev, warmup: int):
    """deberta_ffn_gemm: GELU(x W^T + b), the DeBERTa-v3-large feed-forward's first half
    (kernels.linear_act.linear_gelu, DebertaV2Intermediate), 65536 tokens x 1024 -> 4096.
    mt5_ffn_gemm: GELU_tanh(x wi_0^T) * up, the mT5-large gate projection with the gated
    activation in its epilogue (kernels.linear_act.gated_gelu_tanh), 65536 x 1024 -> 2816.
    Tensor-bound: value = 2 M N K / time, TFLOP/s."""
    from kernels.linear_act import gated_gelu_tanh, linear_gelu
    name = args.workload
    M, K, N = FFN_GEMM_SHAPES[name]
    g = torch.Generator(device=dev).manual_seed(6000 + rank)
    w = (torch.randn(N, K, generator=g, device=dev) * 0.03).to(torch.bfloat16)
    if name == "deberta_ffn_gemm":
        b = (torch.randn(N, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        sets = [(torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16),) for _ in range(2)]
        call = lambda x: linear_gelu(x, w, b)
    else:
        sets = [(torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16),
                 torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)) for _ in range(2)]
        call = lambda x, up: gated_gelu_tanh(x, w, up)
    return _run_hbm_op(args, world, rank, dev, warmup, sets, call, 2 * M * N * K, ffn_gemm_config(name),
                       lambda: ffn_gemm_cpu_baseline(name), bound="tensor")


# ----------------------------------------------------------------------------- GLiNER span head
def _span_weights(m) -> dict:
    w = {}
    for pre, seq in (("start", m.project_start), ("end", m.project_end), ("out", m.out_project)):
        w[f"{pre}_w1"], w[f"{pre}_b1"] = seq[0].weight.detach(), seq[0].bias.detach()
        w[f"{pre}_w2"], w[f"{pre}_b2"] = seq[3].weight.detach(), seq[3].bias.detach()
    return w


GLINER_SPAN_CONFIG = {
    "workload": "GLiNER span head (poolers/gliner.py SpanMarkerV0 + class einsum), hidden 1024, max_width 12",
    "requests": 64, "words": "U[32,384] per request", "classes": "U[3,25] per request",
    "weights": "N(0, 0.02), bf16", "scores": "fp32"}


def gliner_span_cpu_baseline(budget_s: float = 12.0):
    """The reference's span head in its own order of operations (oracle.span_scores_ref:
    SpanMarkerV0 MLPs over words and spans, then the class einsum; fp32 torch) on the host
    cores, one request at a time as the reference's pooler loops, for ~12 s: spans/s."""
    import oracle
    from vf_b200 import workloads as W
    torch.set_num_threads(os.cpu_count() or 1)
    b = W.gliner_span_batch(device="cpu")
    w = {k: v.float() for k, v in _span_weights(W.gliner_span_marker(device="cpu")).items()}
    wo, so, co = b["word_offsets"], b["span_offsets"], b["class_offsets"]
    n_spans, g, t0 = 0, 0, time.perf_counter()
    while time.perf_counter() - t0 < budget_s and g < len(wo) - 1:
        oracle.span_scores_ref(b["words"][wo[g]:wo[g + 1]].float()[None], b["span_idx"][so[g]:so[g + 1]][None], w,
                               b["classes"][co[g]:co[g + 1]].float()[None], W.SPAN_MAX_WIDTH, dtype=torch.float32)
        n_spans += so[g + 1] - so[g]
        g += 1
    dt = time.perf_counter() - t0
    return {"value": n_spans / dt, "unit": "spans/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{g} of the 64 requests, one at a time, fp32 torch on CPU (oracle of the reference's "
                      f"SpanMarkerV0 + einsum)"}


def run_gliner_span(args, world: int, rank: int, dev, warmup: int):
    """gliner_span: the span-scoring head of a GLiNER-large pooler over one vLLM batch of 64
    requests (kernels.span_scores.span_scores_packed: the per-word / per-class GEMMs in torch
    and one span-score launch).  value = spans scored per second (whole job); every rank scores
    the same batches (weak scaling).  The roofline line is the span-score kernel alone, timed
    on the same batches' precomputed factors."""
    from kernels.span_scores import span_factors, span_scores_packed
    from vf_b200 import workloads as W
    marker = W.gliner_span_marker(device=dev)
    sets = [W.gliner_span_batch(seed=6100 + i, device=dev) for i in range(4)]
    offs = ("word_offsets", "span_offsets", "class_offsets")

    def call(b):
        return span_scores_packed(marker, b["words"], b["span_idx"], b["classes"], *(b[k] for k in offs),
                                  torch.float32)

    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for i in range(warmup):
            call(sets[i % len(sets)])
        torch.cuda.synchronize()
        sampler = ClockSampler(dev.index or 0)
        sampler.start()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.steps):
            call(sets[i % len(sets)])
        ev1.record(stream)
        torch.cuda.synchronize()
        clocks = sampler.stop()
        ms = ev0.elapsed_time(ev1)
        spans = float(sum(sets[i % len(sets)]["span_offsets"][-1] for i in range(args.steps)))
        # the kernel alone, on the same batches' factors
        fac = [span_factors(marker, b["words"], b["classes"]) for b in sets]
        kcalls = [lambda b=b, f=f: torch.ops.vf_b200.span_scores(f[0], f[1], b["span_idx"], f[2], f[3],
                                                                  *(b[k] for k in offs), torch.float32)
                  for b, f in zip(sets, fac)]
        for i in range(warmup):
            kcalls[i % len(kcalls)]()
        torch.cuda.synchronize()
        ek0, ek1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ek0.record(stream)
        for i in range(args.steps):
            kcalls[i % len(kcalls)]()
        ek1.record(stream)
        torch.cuda.synchronize()
        kms = ek0.elapsed_time(ek1) / args.steps
    K4 = 4 * W.SPAN_HIDDEN
    mma_flops = sum(2.0 * K4 * sum((b["span_offsets"][g + 1] - b["span_offsets"][g]) *
                                   (b["class_offsets"][g + 1] - b["class_offsets"][g])
                                   for g in range(len(b["span_offsets"]) - 1)) for b in sets) / len(sets)
    from vf_b200 import dist as VD
    ms_max, spans_all, _ = VD.reduce_timing(ms, spans, 0.0, dev)
    value = spans_all / (ms_max * 1e-3)
    e2e = None
    if not args.no_e2e:
        b0 = sets[0]
        host = {"words": b0["words"].cpu().pin_memory(), "span_idx": b0["span_idx"].cpu().pin_memory(),
                "classes": b0["classes"].cpu().pin_memory(), **{k: b0[k] for k in offs}}
        n_e2e = max(3, min(args.steps, 10))
        with torch.no_grad():
            ems, h2d, d2h = pipelined_e2e(dev, host, call, n_e2e, world)
        e2e = {"value": b0["span_offsets"][-1] * world * n_e2e / (ems * 1e-3), "unit": "spans/s", "pipelined": True,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": n_e2e}
    if rank != 0:
        return None
    peaks = measured_peaks()
    achieved = mma_flops / (kms * 1e-3) / 1e12
    return {"metric": METRIC, "value": value, "unit": "spans/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": GLINER_SPAN_CONFIG,
            "l2": "4 rotating request batches (~30 MB inputs each) and 92 MB of weights; no flush",
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                         "frac": achieved / peaks["bf16"], "traffic": committed_traffic(args.workload),
                         "peak_source": f"{peaks['source']} bf16 dense (burst)",
                         "what": "span-score kernel alone: 2 x spans x 4D x classes per launch",
                         "kernel_ms": kms, "algorithmic_flops_per_launch": mma_flops},
            "gpu_launches": 2 * args.steps, "clocks": clocks, "e2e": e2e,
            **({"cpu_baseline": gliner_span_cpu_baseline()} if world == 1 and not args.no_cpu_baseline else {})}


def run_gliner_span_reference_gpu(args, dev, warmup: int):
    """The reference's own span head on this GPU (--impl reference_triton --workload gliner_span):
    poolers/gliner.py's SpanMarkerV0 from the reference install with this workload's weights,
    then the pooler's einsum (:285-289), one request at a time as GLiNERSpanPooler.forward loops,
    bf16, on the same batches.  A secondary bar beside the CPU reference arm."""
    import importlib.util
    from vf_b200 import workloads as W
    ref = Path(os.environ.get("VF_REFERENCE", str(ROOT / "baseline" / "_ref")))
    path = ref / "poolers" / "gliner.py"
    if not path.exists():
        return {"impl": "reference_triton", "unavailable": f"no reference install at {ref}"}
    if str(ref) not in sys.path:
        sys.path.append(str(ref))                  # vllm_factory.pooling, imported by the pooler
    spec = importlib.util.spec_from_file_location("_vf_reference_gliner_pooler", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    ours = W.gliner_span_marker(device=dev)
    marker = mod.SpanMarkerV0(W.SPAN_HIDDEN, W.SPAN_MAX_WIDTH, dropout=0.0)
    with torch.no_grad():
        for (na, a), (nb, b) in zip(marker.named_parameters(), ours.named_parameters()):
            assert na == nb and a.shape == b.shape, (na, nb)
            a.copy_(b.float())
    marker = marker.to(device=dev, dtype=torch.bfloat16).eval()
    sets = [W.gliner_span_batch(seed=6100 + i, device=dev) for i in range(4)]

    def step(b):
        wo, so, co = b["word_offsets"], b["span_offsets"], b["class_offsets"]
        for g in range(len(wo) - 1):
            rep = marker(b["words"][wo[g]:wo[g + 1]][None], b["span_idx"][so[g]:so[g + 1]][None])
            torch.einsum("BLKD,BCD->BLKC", rep, b["classes"][co[g]:co[g + 1]][None])

    stream = torch.cuda.current_stream(dev)
    steps = max(3, min(args.steps, 10))
    with torch.no_grad():
        for i in range(warmup):
            step(sets[i % len(sets)])
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(steps):
            step(sets[i % len(sets)])
        ev1.record(stream)
        torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    spans = float(sum(sets[i % len(sets)]["span_offsets"][-1] for i in range(steps)))
    return {"metric": METRIC, "value": spans / (ms * 1e-3), "unit": "spans/s", "n_gpus": 1, "steps": steps,
            "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference_triton",
            "config": GLINER_SPAN_CONFIG,
            "what": "the reference's SpanMarkerV0 + einsum (torch, bf16) on this GPU, one request at a time"}


# ----------------------------------------------------------------------------- attention lines
def reference_triton_kernels():
    """The reference's own Triton modules (kernels/flash_attention_rpb.py,
    kernels/flash_deberta_attention.py) from the reference install (VF_REFERENCE, else
    baseline/_ref), loaded under private names so they never shadow this repository's
    `kernels` package.  Returns (modules, None) or (None, why)."""
    import importlib.util
    ref = Path(os.environ.get("VF_REFERENCE", str(ROOT / "baseline" / "_ref")))
    mods = {}
    for m in ("flash_attention_rpb", "flash_deberta_attention"):
        path = ref / "kernels" / f"{m}.py"
        if not path.exists():
            return None, f"no reference install at {ref}"
        spec = importlib.util.spec_from_file_location(f"_vf_reference_triton_{m}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mods[m] = mod
    if not getattr(mods["flash_deberta_attention"], "HAS_TRITON", False):
        return None, "the reference's Triton kernels did not import"
    return mods, None


def reference_triton_call(name: str, mods: dict):
    """The reference's stock GPU path for a workload, on the same input sets as this
    repository's arm: flash_attention_rpb_final as T5SelfAttention.forward calls it
    (models/mt5/mt5_encoder.py:269-280), and flash_deberta_attention with the caller's
    position products as DisentangledSelfAttentionV2._flash_forward forms them
    (models/deberta_v2/deberta_v2_encoder.py:275-322).  For a fused workload every step also
    forms those products (torch matmuls), which is the work the fused kernel absorbs."""
    if "varlen" in name:
        return None
    if name == "mt5_c2":
        fn = mods["flash_attention_rpb"].flash_attention_rpb_final
        return lambda x: fn(x["q"], x["k"], x["v"], rpb_table=x["rpb_table"], num_buckets=32, max_distance=128,
                            is_decoder=False, padding_mask=x["padding_mask"], dropout_p=0.0, softmax_scale=1.0,
                            use_autotune=True)
    fn = mods["flash_deberta_attention"].flash_deberta_attention
    if name.endswith("_fused"):
        def call(x):
            pk = torch.matmul(x["q"], x["rel_key"].transpose(-1, -2))
            pq = torch.matmul(x["k"], x["rel_query"].transpose(-1, -2).to(dtype=x["k"].dtype))
            return fn(q=x["q"], k=x["k"], v=x["v"], seq_lengths=x["seq_lengths"], pos_key=pk, pos_query=pq,
                      causal=False, sm_scale=x["sm_scale"], position_buckets=256, max_relative_distance=512,
                      use_log_bucket=True)
        return call
    return lambda x: fn(q=x["q"], k=x["k"], v=x["v"], seq_lengths=x["seq_lengths"], pos_key=x["pos_key"],
                        pos_query=x["pos_query"], causal=False, sm_scale=x["sm_scale"], position_buckets=256,
                        max_relative_distance=512, use_log_bucket=True)


def run_attention(args, name: str, steps: int, world: int, rank: int, dev, warmup: int, cpu_base: bool,
                  impl: str = "ours"):
    """One attention workload: `steps` calls of the drop-in, each on a different input set,
    timed on the device; value = valid FLOPs of all ranks / max rank time.  Every rank takes
    the same collective steps; rank 0 gets the line, the others None.  impl="reference_triton"
    times the reference's Triton path (reference_triton_call) on the same inputs, without the
    e2e and CPU legs."""
    sets, call, flops, tokens, cfg, keys, lens, launches = build_workload(name, rank, dev)
    if impl == "reference_triton":
        mods, why = reference_triton_kernels()
        call = reference_triton_call(name, mods) if mods else None
        if call is None:
            return {"impl": impl, "unavailable": why or f"the reference has no GPU path for {name}"}
        launches, cpu_base = None, False
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    for i in range(warmup):
        call(sets[i % len(sets)])
    torch.cuda.synchronize()

    sampler = ClockSampler(dev.index or 0)
    sampler.start()
    barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for i in range(steps):
        call(sets[i % len(sets)])
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    ms = ev0.elapsed_time(ev1)

    from vf_b200 import dist as VD
    ms_max, flops_all, tokens_all = VD.reduce_timing(ms, flops, tokens, dev)
    value = flops_all * steps / (ms_max * 1e-3) / 1e12

    # ---- end to end through the public call, host buffers, copies inside the timed region
    e2e = None
    if not args.no_e2e and impl == "ours":
        host = {k: (v.cpu().pin_memory() if isinstance(v, torch.Tensor) and v.is_cuda and k in keys else v)
                for k, v in sets[0].items()}
        n_e2e = max(3, min(steps, 30))
        ems, h2d, d2h = pipelined_e2e(dev, {k: v for k, v in host.items() if k in keys},
                                      lambda x: call({**host, **x}), n_e2e, world)
        barrier()
        e2e = {"value": flops_all * n_e2e / (ems * 1e-3) / 1e12, "unit": "TFLOP/s", "pipelined": True,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": n_e2e}
    barrier()
    if rank != 0:
        return None

    peaks = measured_peaks()
    dtype_label = cfg.pop("_dtype", "bf16")
    l2_note = cfg.pop("_l2")
    achieved = flops / (ms / steps * 1e-3) / 1e12      # this rank's launches
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16"], "unit": "TFLOP/s",
                "frac": achieved / peaks["bf16"], "traffic": committed_traffic(name),
                "peak_source": f"{peaks['source']} bf16 dense (burst)",
                "algorithmic_flops_per_launch": flops}
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms_max / steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype_label, "data": "synthetic", "config": cfg, "l2": l2_note,
            "tokens_per_s": tokens_all * steps / (ms_max * 1e-3),
            "pct_bf16_peak": value / (peaks["bf16"] * world),
            "roofline": roofline, "gpu_launches": steps * launches if launches else None, "clocks": clocks,
            "e2e": e2e}
    if impl != "ours":
        line["impl"] = impl
        line["roofline"]["traffic"] = None
    if world == 1 and cpu_base:
        line["cpu_baseline"] = cpu_baseline(name, lens)
    return line


def deberta_line_workload() -> str:
    """The DeBERTa attention sub-result: the fused mode when this build has it."""
    from kernels import flash_deberta_attention as FD
    return "deberta_c1_fused" if getattr(FD, "HAS_FUSED_POSITIONS", False) else "deberta_c1"


# ----------------------------------------------------------------------------- reference arm
def reference_line(args, name: str) -> dict:
    if name in ENCODER_WORKLOADS:
        cb = encoder_cpu_baseline(name)
        cfg = attention_config(name)
    elif name == "mt5_ffn_act":
        cb, cfg = gated_act_cpu_baseline(), {"workload": name}
    elif name == "deberta_add_ln":
        cb, cfg = add_layer_norm_cpu_baseline(), {"workload": name}
    elif name in FFN_GEMM_SHAPES:
        cb, cfg = ffn_gemm_cpu_baseline(name), ffn_gemm_config(name)
    elif name == "gliner_span":
        cb, cfg = gliner_span_cpu_baseline(), GLINER_SPAN_CONFIG
    else:
        cb = cpu_baseline(name, None, budget_s=max(5.0, min(60.0, 2.0 * args.steps)))
        cfg = attention_config(name)
    return {"metric": METRIC, "value": cb["value"], "unit": cb["unit"], "n_gpus": args.gpus, "steps": args.steps,
            "warmup": max(args.warmup, 3), "higher_is_better": True,
            "scaling": "strong" if name in ENCODER_WORKLOADS else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "impl": "reference", "config": cfg, "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference_triton"],
                    help="reference = the reference's CPU path (the oracle port) on the host cores; "
                         "reference_triton = the reference's own Triton kernels on this GPU (one GPU, "
                         "attention workloads; a secondary bar, not the driver's reference arm)")
    ap.add_argument("--workload", default="default",
                    help="default = mt5_c2 headline with the DeBERTa C1 attention and C3 encoder lines "
                         "as sub-results; or one of the named workloads")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sub-results", action="store_true")
    args = ap.parse_args()
    warmup = max(args.warmup, 3)
    headline = "mt5_c2" if args.workload == "default" else args.workload
    subs = args.workload == "default" and not args.no_sub_results

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        line = reference_line(args, headline)
        if subs:
            line["sub_results"] = {"deberta_c1": reference_line(args, "deberta_c1_fused"),
                                   "deberta_c3": reference_line(args, "deberta_c3")}
        print(json.dumps(line))
        return

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA GPU")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.impl == "reference_triton":
        if rank != 0:
            return
        import vf_b200
        vf_b200.load()                  # the input generators share this repository's workloads
        if headline == "gliner_span":
            print(json.dumps(run_gliner_span_reference_gpu(args, dev, warmup)))
            return
        line = run_attention(args, headline, args.steps, 1, 0, dev, warmup, False, impl="reference_triton")
        if subs:
            line["sub_results"] = {
                w: run_attention(args, w, args.steps, 1, 0, dev, warmup, False, impl="reference_triton")
                for w in ("deberta_c1", "deberta_c1_fused")}
        print(json.dumps(line))
        return
    if world > 1:
        import datetime
        # NCCL's initialisation log (communicator ranks) goes to stderr; rank 0's stdout
        # carries only the JSON line.  A caller's own NCCL_DEBUG settings are kept.
        if "NCCL_DEBUG" not in os.environ:
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    import vf_b200
    vf_b200.load()
    cpu_base = not args.no_cpu_baseline

    if headline in ENCODER_WORKLOADS:
        line = run_encoder(args, headline, args.steps, world, rank, dev, warmup, cpu_base)
    elif headline == "mt5_ffn_act":
        line = run_gated_act(args, world, rank, dev, warmup)
    elif headline == "deberta_add_ln":
        line = run_add_layer_norm(args, world, rank, dev, warmup)
    elif headline in FFN_GEMM_SHAPES:
        line = run_ffn_gemm(args, world, rank, dev, warmup)
    elif headline == "gliner_span":
        line = run_gliner_span(args, world, rank, dev, warmup)
    else:
        line = run_attention(args, headline, args.steps, world, rank, dev, warmup, cpu_base)
    if subs:
        # Same run, same ranks: the DeBERTa attention layer (weak-scaled like the headline)
        # and the 24-layer DeBERTa encoder (strong-scaled by LPT over the ranks).
        sub_steps = max(3, min(args.steps, 20))
        d1 = run_attention(args, deberta_line_workload(), args.steps, world, rank, dev, warmup, cpu_base)
        c3 = run_encoder(args, "deberta_c3", sub_steps, world, rank, dev, warmup, cpu_base)
        if line is not None:
            line["sub_results"] = {"deberta_c1": d1, "deberta_c3": c3}
            line["gpu_launches"] += d1["gpu_launches"] + c3["gpu_launches"]
    if line is not None:
        print(json.dumps(line))
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
