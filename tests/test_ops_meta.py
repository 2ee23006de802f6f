"""The torch.ops layer on the CPU: every op has a Meta implementation (shape and dtype of
the output, for tracing) and raises on CPU tensors (there is no CPU implementation)."""
import pytest
import torch

import vf_b200.ops  # noqa: F401

OPS = torch.ops.vf_b200


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_meta_shapes_and_dtypes(dtype):
    m = dict(device="meta", dtype=dtype)
    q = torch.empty(2, 3, 100, 64, **m)
    assert OPS.rpb_attention(q, q, q, None, 32, 128, False, None, 0.0, 1.0).shape == q.shape
    o = OPS.deberta_attention(q, q, q, None, None, None, False, None, 256, 512, True)
    assert o.shape == q.shape and o.dtype == dtype
    qp = torch.empty(100, 3, 64, **m)
    cu = torch.empty(3, dtype=torch.int32, device="meta")
    o = OPS.rpb_attention_varlen(qp, qp, qp, cu, 60, None, 32, 128, False, 1.0)
    assert o.shape == qp.shape and o.dtype == dtype
    o = OPS.deberta_attention_varlen(qp, qp, qp, cu, 60, None, None, False, None, 256, 512, True)
    assert o.shape == qp.shape and o.dtype == dtype
    g = torch.empty(5, 7, 2816, **m)
    o = OPS.gated_act(g, g, 0)
    assert o.shape == g.shape and o.dtype == dtype
    o = OPS.gated_act(g, None, 1)
    assert o.shape == g.shape and o.dtype == dtype
    h = torch.empty(5, 7, 1024, **m)
    w = torch.empty(1024, **m)
    o = OPS.add_layer_norm(h, h, w, w, 1e-7)
    assert o.shape == h.shape and o.dtype == dtype


def test_cpu_tensors_raise():
    q = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16)
    qp = torch.zeros(8, 1, 64, dtype=torch.bfloat16)
    cu = torch.tensor([0, 8], dtype=torch.int32)
    for call in (lambda: OPS.rpb_attention(q, q, q, None, 32, 128, False, None, 0.0, 1.0),
                 lambda: OPS.deberta_attention(q, q, q, None, None, None, False, None, 256, 512, True),
                 lambda: OPS.rpb_attention_varlen(qp, qp, qp, cu, 8, None, 32, 128, False, 1.0),
                 lambda: OPS.deberta_attention_varlen(qp, qp, qp, cu, 8, None, None, False, None, 256, 512, True),
                 lambda: OPS.gated_act(q, q, 0),
                 lambda: OPS.add_layer_norm(qp, qp, qp[0, 0], None, 1e-7)):
        with pytest.raises(RuntimeError, match="CUDA"):
            call()


def test_op_layer_uses_the_shared_cxx_runtime():
    """The torch op layer must not carry its own libstdc++: with a private copy (a toolchain
    that links libstdc++.a), formatting a number into a TORCH_CHECK message crashed the
    process on the duplicated locale facets instead of raising RuntimeError."""
    from vf_b200 import build
    assert build.embedded_cxx_runtime(build.TORCH_LIB_PATH) == []
    assert build.embedded_cxx_runtime(build.LIB_PATH) == []
