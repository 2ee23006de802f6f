"""GLiNER span scores, CPU side: the C entry point's argument checks (no compute call is made:
every case is rejected, or has no work, before any CUDA call), the torch op's fake / CPU
registrations, the drop-in's installer, and the oracle's factored form against the reference
order of operations on edge cases (clamped indices, masked spans, C = 1, one word)."""
import ctypes

import pytest
import torch

import oracle
from vf_b200 import _lib


def _arr(xs):
    return (ctypes.c_int64 * len(xs))(*xs)


def _args(**kw):
    a = _lib.SpanScoresArgs(dtype=_lib.VF_DTYPE_BF16, start_proj=0x10000, end_proj=0x20000, start_row_stride=256,
                            end_row_stride=256, K=256, span_idx=0x30000, span_idx_int64=1, idx_stride_span=2,
                            idx_stride_pair=1, classes=0x40000, class_row_stride=256, class_bias=None, out=0x50000,
                            out_dtype=_lib.VF_DTYPE_F32, num_segments=1)
    offs = {"word_offsets": [0, 10], "span_offsets": [0, 50], "class_offsets": [0, 4]}
    for k, v in kw.items():
        if k in offs:
            offs[k] = v
        else:
            setattr(a, k, v)
    keep = [_arr(offs["word_offsets"]), _arr(offs["span_offsets"]), _arr(offs["class_offsets"])]
    a.word_offsets, a.span_offsets, a.class_offsets = keep
    return a, keep


@pytest.mark.parametrize("kw,code,msg", [
    (dict(dtype=_lib.VF_DTYPE_F32), _lib.VF_EUNSUPPORTED, "dtype"),
    (dict(out_dtype=7), _lib.VF_EINVAL, "out dtype"),
    (dict(num_segments=-1), _lib.VF_EINVAL, "num_segments"),
    (dict(K=100), _lib.VF_EINVAL, "multiple of 64"),
    (dict(K=0), _lib.VF_EINVAL, "multiple of 64"),
    (dict(span_offsets=[5, 2]), _lib.VF_EINVAL, "decrease"),
    (dict(word_offsets=[0, 0]), _lib.VF_EINVAL, "no words"),
    (dict(word_offsets=[-1, 3]), _lib.VF_EINVAL, ">= 0"),
    (dict(start_proj=None), _lib.VF_EINVAL, "non-null"),
    (dict(out=None), _lib.VF_EINVAL, "non-null"),
    (dict(class_row_stride=128), _lib.VF_EINVAL, "at least K"),
    (dict(start_proj=0x10008), _lib.VF_EINVAL, "16-byte"),
    (dict(end_row_stride=260), _lib.VF_EINVAL, "16-byte"),
    (dict(idx_stride_span=-2), _lib.VF_EINVAL, "negative"),
])
def test_span_scores_rejects_before_launch(kw, code, msg):
    lib = _lib.load()
    a, _keep = _args(**kw)
    rc = lib.vf_span_scores_fwd(ctypes.byref(a), None)
    assert rc == code
    assert msg in lib.vf_last_error().decode()


def test_span_scores_null_args_and_offsets():
    lib = _lib.load()
    assert lib.vf_span_scores_fwd(None, None) == _lib.VF_EINVAL
    a, _keep = _args()
    a.word_offsets = None
    assert lib.vf_span_scores_fwd(ctypes.byref(a), None) == _lib.VF_EINVAL


@pytest.mark.parametrize("kw", [
    dict(num_segments=0),
    dict(span_offsets=[0, 0]),                     # no spans
    dict(class_offsets=[3, 3]),                    # no classes
    dict(start_proj=None, span_offsets=[4, 4]),    # nothing to do: pointers are not read
])
def test_span_scores_without_work_returns_ok_without_cuda(kw):
    lib = _lib.load()
    a, _keep = _args(**kw)
    assert lib.vf_span_scores_fwd(ctypes.byref(a), None) == _lib.VF_OK


def test_span_args_struct_layout():
    assert ctypes.sizeof(_lib.SpanScoresArgs) % 8 == 0
    assert _lib.SpanScoresArgs.word_offsets.offset > _lib.SpanScoresArgs.num_segments.offset


def test_span_scores_op_fake_and_cpu():
    import vf_b200.ops  # noqa: F401
    u = torch.empty(10, 256, dtype=torch.bfloat16, device="meta")
    idx = torch.empty(50, 2, dtype=torch.long, device="meta")
    c = torch.empty(7, 256, dtype=torch.bfloat16, device="meta")
    out = torch.ops.vf_b200.span_scores(u, u, idx, c, None, [0, 4, 10], [0, 20, 50], [0, 3, 7], torch.float32)
    assert out.shape == (20 * 3 + 30 * 4,) and out.dtype == torch.float32
    with pytest.raises(RuntimeError, match="no CPU implementation"):
        torch.ops.vf_b200.span_scores(torch.zeros(10, 256, dtype=torch.bfloat16), torch.zeros(10, 256, dtype=torch.bfloat16),
                                      torch.zeros(5, 2, dtype=torch.long), torch.zeros(3, 256, dtype=torch.bfloat16),
                                      None, [0, 10], [0, 5], [0, 3], torch.float32)


def test_dropin_raises_on_cpu_and_installs_idempotently():
    from kernels import span_scores

    class Marker(torch.nn.Module):
        def __init__(self, D):
            super().__init__()
            mk = lambda i, o: torch.nn.Sequential(torch.nn.Linear(i, 4 * o), torch.nn.ReLU(),  # noqa: E731
                                                  torch.nn.Dropout(0.0), torch.nn.Linear(4 * o, o))
            self.project_start, self.project_end, self.out_project = mk(D, D), mk(D, D), mk(2 * D, D)

    m = Marker(16).eval()
    with pytest.raises(RuntimeError, match="CUDA"):
        span_scores.span_scores_segments(m, [torch.zeros(4, 16)], [torch.zeros(8, 2, dtype=torch.long)],
                                         [torch.zeros(3, 16)])

    class Pooler:
        def forward(self, hidden_states, ctx):
            return "reference"

    span_scores.install_fused_span_scoring(Pooler)
    span_scores.install_fused_span_scoring(Pooler)
    assert Pooler.forward is span_scores.gliner_span_pooler_forward
    assert Pooler._vf_reference_forward(None, None, None) == "reference"


def _weights(D, seed):
    g = torch.Generator().manual_seed(seed)
    w = {}
    for pre, din, dout in (("start", D, D), ("end", D, D), ("out", 2 * D, D)):
        w[f"{pre}_w1"] = torch.randn(4 * dout, din, generator=g) * 0.1
        w[f"{pre}_b1"] = torch.randn(4 * dout, generator=g) * 0.1
        w[f"{pre}_w2"] = torch.randn(dout, 4 * dout, generator=g) * 0.1
        w[f"{pre}_b2"] = torch.randn(dout, generator=g) * 0.1
    return w, g


@pytest.mark.parametrize("L,W,C", [(1, 3, 1), (9, 4, 2), (20, 12, 5)])
def test_factored_form_equals_reference_order_on_edge_cases(L, W, C):
    D = 16
    w, g = _weights(D, L * 100 + C)
    h = torch.randn(1, L, D, generator=g)
    pe = torch.randn(1, C, D, generator=g)
    # indices past the sentence (clamped), negative ones, and masked spans (0, 0)
    idx = torch.randint(-3, L + 3, (1, L * W, 2), generator=g)
    idx[0, ::5] = 0
    ref = oracle.span_scores_ref(h, idx, w, pe, W)
    fac = oracle.span_scores_factored_ref(h, idx, w, pe, W)
    assert (ref - fac).abs().max().item() < 1e-10
