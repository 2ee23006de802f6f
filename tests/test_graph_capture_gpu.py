"""The ops inside CUDA graphs: each is captured once (after an eager warm-up call, which
does the one-time kernel set-up) and replayed with new input values written into the
captured buffers; the replay must equal an eager call on the same values bit for bit."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _capture_and_check(make_inputs, call):
    static = make_inputs(0)
    call(*static)                                # eager warm-up (kernel attributes set once)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = call(*static)
    for seed in (1, 2):
        fresh = make_inputs(seed)
        for s, f in zip(static, fresh):
            if isinstance(s, torch.Tensor):
                s.copy_(f)
        g.replay()
        torch.cuda.synchronize()
        eager = call(*fresh)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


def _rand(seed, *shape, dtype=torch.bfloat16, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(dtype)


def test_rpb_padded_and_packed_in_graphs():
    from kernels.flash_attention_rpb import flash_attention_rpb_final, flash_attention_rpb_varlen
    mask = torch.zeros(2, 1, 1, 300, dtype=torch.bfloat16, device="cuda")
    mask[1, ..., 200:] = torch.finfo(torch.bfloat16).min
    _capture_and_check(lambda s: (_rand(s, 2, 4, 300, 64), _rand(s + 10, 2, 4, 300, 64), _rand(s + 20, 2, 4, 300, 64),
                                  _rand(s + 30, 32, 4), mask),
                       lambda q, k, v, t, m: flash_attention_rpb_final(q, k, v, t, 32, 128, False, m))
    cu = torch.tensor([0, 130, 131, 400], dtype=torch.int32, device="cuda")
    _capture_and_check(lambda s: (_rand(s, 400, 4, 64), _rand(s + 10, 400, 4, 64), _rand(s + 20, 400, 4, 64),
                                  _rand(s + 30, 32, 4)),
                       lambda q, k, v, t: flash_attention_rpb_varlen(q, k, v, cu, 269, t, 32, 128))


def test_deberta_padded_and_packed_in_graphs():
    from kernels.flash_deberta_attention import flash_deberta_attention, flash_deberta_attention_varlen
    sm = 1 / math.sqrt(64 * 3)
    sl = torch.tensor([300, 170], dtype=torch.int32, device="cuda")
    _capture_and_check(lambda s: tuple(_rand(s + i, 2, 4, 300, d, scale=3.0 if d == 512 else 1.0)
                                       for i, d in enumerate((64, 64, 64, 512, 512))),
                       lambda q, k, v, pk, pq: flash_deberta_attention(q, k, v, sl, pk, pq, False, sm, 256, 512, True))
    cu = torch.tensor([0, 130, 131, 400], dtype=torch.int32, device="cuda")
    _capture_and_check(lambda s: tuple(_rand(s + i, 400, 4, d, scale=3.0 if d == 512 else 1.0)
                                       for i, d in enumerate((64, 64, 64, 512, 512))),
                       lambda q, k, v, pk, pq: flash_deberta_attention_varlen(q, k, v, cu, 269, pk, pq, False, sm,
                                                                              256, 512, True))


def test_gated_act_and_add_layer_norm_in_graphs():
    """The two HBM-bound ops beside the path (bench.py times them as a captured graph)."""
    from kernels.ff_fused import fused_gelu_mul_dropout
    from kernels.fused_add_layernorm import fused_add_layer_norm
    _capture_and_check(lambda s: (_rand(s, 300, 2 * 704, scale=2.0),),
                       lambda gu: fused_gelu_mul_dropout(gu[:, :704], gu[:, 704:], "gelu_new"))
    w, b = _rand(7, 1024) + 1.0, _rand(8, 1024, scale=0.1)
    _capture_and_check(lambda s: (_rand(s, 513, 1024), _rand(s + 10, 513, 1024)),
                       lambda x, r: fused_add_layer_norm(x, r, w, b, 1e-7))


def test_deberta_fused_mode_in_graphs():
    """The fused position mode (set-up kernel writing the workspace, then the attention
    kernel) captured in a graph, workspace from the graph's memory pool: replays equal eager
    calls bit for bit."""
    from kernels.flash_deberta_attention import flash_deberta_attention, flash_deberta_attention_varlen
    sl = torch.tensor([300, 170], dtype=torch.int32, device="cuda")
    _capture_and_check(lambda s: tuple(_rand(s + i, *shape, scale=0.4 if i >= 3 else 1.0)
                                       for i, shape in enumerate([(2, 4, 300, 64)] * 3 + [(1, 4, 512, 64)] * 2)),
                       lambda q, k, v, rk, rq: flash_deberta_attention(q, k, v, sl, None, None, False, 0.07, 256, 512,
                                                                       True, rel_key=rk, rel_query=rq))
    cu = torch.tensor([0, 130, 131, 400], dtype=torch.int32, device="cuda")
    _capture_and_check(lambda s: tuple(_rand(s + i, *shape, scale=0.4 if i >= 3 else 1.0)
                                       for i, shape in enumerate([(400, 4, 64)] * 3 + [(1, 4, 512, 64)] * 2)),
                       lambda q, k, v, rk, rq: flash_deberta_attention_varlen(q, k, v, cu, 269, None, None, False, 0.07,
                                                                              256, 512, True, rel_key=rk, rel_query=rq))
