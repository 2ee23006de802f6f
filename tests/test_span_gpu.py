"""GLiNER span scores on the GPU (csrc/vf_span.cu through torch.ops.vf_b200.span_scores and the
C ABI) against the CPU oracle (oracle/span.py, pinned to the reference's SpanMarkerV0 + einsum
by tests/test_oracle_golden.py).

Kernel-level gate (the same 16-bit U, V, P as input): the kernel rounds relu(U + V) to the
16-bit dtype once and accumulates in fp32, so against float64 arithmetic on the same values
it must be within 1e-2 of the largest score magnitude and cosine >= 0.99999 per span row.
Module-level gate (a bf16 SpanMarkerV0 with the reference's order of operations in fp64 as
truth): max-abs within 2e-2 of the score scale and no further from the truth than 1.5x the
reference's own bf16 torch path; per-span cosine >= 0.9999, or, where the reference's own bf16
path is itself below that (D = 1024), no more than 2e-4 below it and never below 0.9995."""
import ctypes

import pytest
import torch

import golden_inputs as gi
import oracle
from kernels.span_scores import fused_span_scores, span_factors, span_scores_segments
from vf_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _rand_case(seed, segs, K, dtype=torch.bfloat16, idx_dtype=torch.int64, scale=0.5):
    """segs: list of (words, spans, classes).  Returns U, V, P, pb, idx, offsets (CPU tensors)."""
    g = torch.Generator().manual_seed(seed)
    W = sum(s[0] for s in segs)
    S = sum(s[1] for s in segs)
    C = sum(s[2] for s in segs)
    U = (torch.randn(W, K, generator=g) * scale).to(dtype)
    V = (torch.randn(W, K, generator=g) * scale).to(dtype)
    P = (torch.randn(C, K, generator=g) * (1.0 / K ** 0.5)).to(dtype)
    pb = torch.randn(C, generator=g)
    idx = []
    for w, s, _ in segs:
        # indices a little outside [0, w - 1] too: the kernel clamps like extract_elements
        idx.append(torch.randint(-2, max(w, 1) + 2, (s, 2), generator=g))
    idx = torch.cat(idx, 0).to(idx_dtype) if idx else torch.zeros(0, 2, dtype=idx_dtype)
    wo, so, co = [0], [0], [0]
    for w, s, c in segs:
        wo.append(wo[-1] + w)
        so.append(so[-1] + s)
        co.append(co[-1] + c)
    return U, V, P, pb, idx, wo, so, co


def _ref_segments(U, V, P, pb, idx, wo, so, co):
    res = []
    for g in range(len(wo) - 1):
        u, v = U[wo[g]:wo[g + 1]], V[wo[g]:wo[g + 1]]
        p, b = P[co[g]:co[g + 1]], (pb[co[g]:co[g + 1]] if pb is not None else None)
        sidx = idx[so[g]:so[g + 1]].long()
        if sidx.shape[0] == 0 or p.shape[0] == 0:
            res.append(torch.zeros(sidx.shape[0], p.shape[0], dtype=torch.float64))
            continue
        res.append(oracle.span_scores_from_factors_ref(u, v, sidx, p, b))
    return res


def _check(out, ref, what, rel=1e-2, min_cos=0.99999):
    o = out.double().cpu()
    if ref.numel() == 0:
        assert o.numel() == 0
        return
    scale = ref.abs().max().item()
    err = (o - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(o, ref, dim=-1, eps=1e-30)
    assert err <= rel * scale, f"{what}: max_abs {err:.3e} > {rel} x {scale:.3e}"
    if ref.shape[-1] >= 4:
        assert cos.min().item() >= min_cos, f"{what}: min row cosine {cos.min().item():.7f}"


@pytest.mark.parametrize("segs,K", [
    ([(37, 185, 7)], 256),                        # one sentence, partial tile, few classes
    ([(384, 4608, 25)], 4096),                    # GLiNER-large sentence: 384 words x 12 widths, D = 1024
    ([(10, 128, 16), (1, 3, 1), (50, 300, 17), (0, 0, 5), (64, 640, 0), (20, 200, 40)], 1024),
    ([(64, 129, 256)], 512),                      # N = 256 exactly
    ([(64, 257, 300)], 512),                      # two class chunks (256 + 44)
])
def test_span_scores_op_matches_oracle(segs, K):
    U, V, P, pb, idx, wo, so, co = _rand_case(3 + K, segs, K)
    out = torch.ops.vf_b200.span_scores(U.to(DEV), V.to(DEV), idx.to(DEV), P.to(DEV), pb.to(DEV), wo, so, co,
                                        torch.float32)
    refs = _ref_segments(U, V, P, pb, idx, wo, so, co)
    at = 0
    for g, r in enumerate(refs):
        n = r.numel()
        _check(out[at:at + n].view(r.shape), r, f"segment {g}")
        at += n
    assert at == out.numel()


@pytest.mark.parametrize("dtype,idx_dtype,out_dtype,bias", [
    (torch.float16, torch.int32, torch.float32, True),
    (torch.bfloat16, torch.int32, torch.bfloat16, False),
    (torch.float16, torch.int64, torch.float16, True),
])
def test_span_scores_dtypes(dtype, idx_dtype, out_dtype, bias):
    segs = [(40, 200, 9), (17, 85, 12)]
    U, V, P, pb, idx, wo, so, co = _rand_case(11, segs, 768, dtype=dtype, idx_dtype=idx_dtype)
    pbd = pb.to(DEV) if bias else None
    out = torch.ops.vf_b200.span_scores(U.to(DEV), V.to(DEV), idx.to(DEV), P.to(DEV), pbd, wo, so, co, out_dtype)
    assert out.dtype == out_dtype
    refs = _ref_segments(U, V, P, pb if bias else None, idx, wo, so, co)
    rel = 1e-2 if out_dtype == torch.float32 else 1.5e-2
    at = 0
    for g, r in enumerate(refs):
        _check(out[at:at + r.numel()].view(r.shape), r, f"{dtype} segment {g}", rel=rel,
               min_cos=0.99999 if out_dtype == torch.float32 else 0.9999)
        at += r.numel()


def test_span_scores_strided_views():
    # U / V as the two halves of one [W, 2K] buffer, span_idx as a column-sliced view.
    segs = [(33, 150, 11)]
    U, V, P, pb, idx, wo, so, co = _rand_case(5, segs, 512)
    both = torch.cat([U, V], 1).to(DEV)
    wide_idx = torch.cat([idx, torch.zeros_like(idx)], 1).to(DEV)[:, :2]
    out = torch.ops.vf_b200.span_scores(both[:, :512], both[:, 512:], wide_idx, P.to(DEV), pb.to(DEV), wo, so, co,
                                        torch.float32)
    _check(out.view(150, 11), _ref_segments(U, V, P, pb, idx, wo, so, co)[0], "strided")


def test_span_scores_through_c_abi_twice():
    """The C entry point called directly (ctypes), two calls in a row on the same buffers."""
    lib = _lib.load()
    segs = [(30, 150, 9), (12, 60, 3)]
    U, V, P, pb, idx, wo, so, co = _rand_case(7, segs, 256)
    Ud, Vd, Pd, pbd, idxd = U.to(DEV), V.to(DEV), P.to(DEV), pb.to(DEV), idx.to(DEV)
    total = sum((so[g + 1] - so[g]) * (co[g + 1] - co[g]) for g in range(len(segs)))
    out = torch.full((total,), float("nan"), device=DEV)
    arr = lambda xs: (ctypes.c_int64 * len(xs))(*xs)  # noqa: E731
    wa, sa, ca = arr(wo), arr(so), arr(co)
    a = _lib.SpanScoresArgs(dtype=_lib.VF_DTYPE_BF16, start_proj=Ud.data_ptr(), end_proj=Vd.data_ptr(),
                            start_row_stride=256, end_row_stride=256, K=256, span_idx=idxd.data_ptr(),
                            span_idx_int64=1, idx_stride_span=2, idx_stride_pair=1, classes=Pd.data_ptr(),
                            class_row_stride=256, class_bias=pbd.data_ptr(), out=out.data_ptr(),
                            out_dtype=_lib.VF_DTYPE_F32, num_segments=len(segs), word_offsets=wa, span_offsets=sa,
                            class_offsets=ca)
    refs = _ref_segments(U, V, P, pb, idx, wo, so, co)
    for _ in range(2):
        rc = lib.vf_span_scores_fwd(ctypes.byref(a), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0, lib.vf_last_error().decode()
        torch.cuda.synchronize()
        at = 0
        for g, r in enumerate(refs):
            _check(out[at:at + r.numel()].view(r.shape), r, f"abi segment {g}")
            at += r.numel()


def _marker_module(weights, D, W, dtype):
    """A SpanMarkerV0-shaped module (project_start / project_end / out_project Sequentials)
    with the golden weights."""
    from torch import nn

    def proj(din, dout, pre):
        m = nn.Sequential(nn.Linear(din, 4 * dout), nn.ReLU(), nn.Dropout(0.0), nn.Linear(4 * dout, dout))
        with torch.no_grad():
            m[0].weight.copy_(weights[f"{pre}_w1"])
            m[0].bias.copy_(weights[f"{pre}_b1"])
            m[3].weight.copy_(weights[f"{pre}_w2"])
            m[3].bias.copy_(weights[f"{pre}_b2"])
        return m

    mk = nn.Module()
    mk.max_width = W
    mk.project_start = proj(D, D, "start")
    mk.project_end = proj(D, D, "end")
    mk.out_project = proj(2 * D, D, "out")
    return mk.to(DEV, dtype).eval()


def test_fused_span_scores_on_the_golden_case():
    c = gi.span_case()
    D = c["h"].shape[-1]
    mk = _marker_module(c["weights"], D, c["max_width"], torch.bfloat16)
    with torch.no_grad():
        out = fused_span_scores(mk, c["h"].to(DEV, torch.bfloat16), c["span_idx"].to(DEV), c["pe"].to(DEV, torch.bfloat16))
    truth = oracle.span_scores_ref(c["h"], c["span_idx"], c["weights"], c["pe"], c["max_width"])
    assert out.shape == (1,) + truth.shape
    # the reference's own order of operations in bf16 on the same device
    with torch.no_grad():
        theirs = oracle.span_scores_ref(c["h"].to(DEV), c["span_idx"].to(DEV),
                                        {k: v.to(DEV) for k, v in c["weights"].items()}, c["pe"].to(DEV),
                                        c["max_width"], dtype=torch.bfloat16).double().cpu()
    o = out[0].double().cpu()
    scale = truth.abs().max().item()
    ours_err = (o - truth).abs().max().item()
    theirs_err = (theirs - truth).abs().max().item()
    assert ours_err <= 2e-2 * scale, (ours_err, scale)
    assert ours_err <= 1.5 * theirs_err + 1e-3 * scale, (ours_err, theirs_err)
    cos = torch.nn.functional.cosine_similarity(o.reshape(-1, o.shape[-1]), truth.reshape(-1, truth.shape[-1]), dim=-1)
    assert cos.min().item() >= 0.9999


def test_span_scores_segments_match_per_sentence_modules():
    """Three sentences of a GLiNER-large-sized marker (D = 1024, 12 widths) in one launch,
    against the reference-order oracle per sentence."""
    g = torch.Generator().manual_seed(41)
    D, W = 1024, 12
    weights = {}
    for pre, din, dout in (("start", D, D), ("end", D, D), ("out", 2 * D, D)):
        weights[f"{pre}_w1"] = torch.randn(4 * dout, din, generator=g) * 0.02
        weights[f"{pre}_b1"] = torch.randn(4 * dout, generator=g) * 0.02
        weights[f"{pre}_w2"] = torch.randn(dout, 4 * dout, generator=g) * 0.02
        weights[f"{pre}_b2"] = torch.randn(dout, generator=g) * 0.02
    weights = {k: v.to(torch.bfloat16).float() for k, v in weights.items()}
    mk = _marker_module(weights, D, W, torch.bfloat16)
    words, spans, classes = [], [], []
    for n, C in ((96, 5), (17, 12), (150, 30)):
        words.append(torch.randn(n, D, generator=g).to(torch.bfloat16))
        first = torch.arange(n).repeat_interleave(W)
        last = first + torch.arange(W).repeat(n)
        keep = (last < n).unsqueeze(-1)
        spans.append(torch.stack([first, last], -1) * keep)
        classes.append(torch.randn(C, D, generator=g).to(torch.bfloat16))
    with torch.no_grad():
        outs = span_scores_segments(mk, [w.to(DEV) for w in words], [s.to(DEV) for s in spans],
                                    [c.to(DEV) for c in classes], out_dtype=torch.float32)
    wd = {k: v.to(DEV) for k, v in weights.items()}
    for w, s, c, o in zip(words, spans, classes, outs):
        truth = oracle.span_scores_ref(w[None].float(), s[None], weights, c[None].float(), W).reshape(-1, c.shape[0])
        with torch.no_grad():   # the reference's order of operations in bf16 on the GPU
            theirs = oracle.span_scores_ref(w[None].to(DEV), s[None].to(DEV), wd, c[None].to(DEV), W,
                                            dtype=torch.bfloat16).reshape(-1, c.shape[0]).double().cpu()
        o = o.double().cpu()
        scale = truth.abs().max().item()
        ours_err, theirs_err = (o - truth).abs().max().item(), (theirs - truth).abs().max().item()
        cos = torch.nn.functional.cosine_similarity(o, truth, dim=-1).min().item()
        cos_theirs = torch.nn.functional.cosine_similarity(theirs, truth, dim=-1).min().item()
        assert ours_err <= 2e-2 * scale, (ours_err, scale)
        assert ours_err <= 1.5 * theirs_err + 1e-3 * scale, (ours_err, theirs_err)
        assert cos >= min(0.9999, cos_theirs - 2e-4) and cos >= 0.9995, (cos, cos_theirs)


def test_span_factors_equal_oracle_factors():
    c = gi.span_case()
    D = c["h"].shape[-1]
    mk = _marker_module(c["weights"], D, c["max_width"], torch.float32)
    with torch.no_grad():
        U, V, P, pb = span_factors(mk, c["h"][0].to(DEV), c["pe"][0].to(DEV))
    Ur, Vr, Pr, pbr = oracle.span_factors_ref(c["h"], c["weights"], c["pe"])
    for a, b in ((U, Ur), (V, Vr), (P, Pr)):
        assert (a.double().cpu() - b).abs().max().item() <= 2e-3 * b.abs().max().item()
    assert (pb.double().cpu() - pbr).abs().max().item() <= 1e-4


def _reference_root():
    import os
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    env = os.environ.get("VF_REFERENCE")
    for cand in ([Path(env)] if env else []) + [root / "baseline" / "_ref"]:
        if (cand / "poolers" / "gliner.py").exists():
            return cand
    return None


def test_reference_gliner_pooler_with_the_kernel_installed():
    """The reference's GLiNERSpanPooler, bf16, with its forward replaced by the batched
    span-score forward, against the fp32 copy of its own forward; no further from it than 1.5x
    the reference's own bf16 forward (tests/reference_pooler_run.py)."""
    import json
    import subprocess
    import sys
    from pathlib import Path
    ref = _reference_root()
    if ref is None:
        pytest.skip("no reference install (VF_REFERENCE or baseline/_ref)")
    root = Path(__file__).resolve().parents[1]
    proc = subprocess.run([sys.executable, str(root / "tests" / "reference_pooler_run.py"), "--reference", str(ref)],
                          capture_output=True, text=True, timeout=600, cwd=str(root))
    line = [ln for ln in proc.stdout.splitlines() if ln.startswith("RESULT ")]
    assert proc.returncode == 0 and line, proc.stdout[-3000:] + proc.stderr[-3000:]
    r = json.loads(line[-1][len("RESULT "):])
    assert r["fused_forward"] == "kernels.span_scores"
    assert len(r["requests"]) == 4
    for req in r["requests"]:
        ours, theirs = req["fused"], req["torch_bf16"]
        assert ours["shape_ok"] and theirs["shape_ok"], req
        assert ours["max_abs"] <= 2e-2 * max(ours["scale"], 1.0), req
        assert ours["max_abs"] <= 1.5 * theirs["max_abs"] + 1e-3 * max(ours["scale"], 1.0), req
        # bf16 LSTM and projections before the scores bound both paths' cosine alike
        assert ours["min_cos"] >= min(0.9999, theirs["min_cos"] - 2e-4) and ours["min_cos"] >= 0.9995, req
