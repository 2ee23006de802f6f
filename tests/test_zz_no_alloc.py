"""The fused DeBERTa entry point for callers that cannot allocate device memory per call
(vf_deberta_attention_fused_noalloc_fwd: an FFI host without a CUDA allocator of its own,
or a process whose device memory is reserved up front by its own pool).  It uses a fixed
scratch array compiled into the library instead of a caller-provided workspace.

Checked through the C ABI against vf_deberta_attention_fused_fwd (the same operator with a
workspace) on two calls in a row with different inputs, since every call reuses the same
scratch, within the parity gates of the other GPU tests.  A call whose scratch would exceed
the 8 MiB array is refused before any launch.  This file is collected last, so a run that
stops at the first failure has already run every other test."""
import ctypes

import pytest
import torch

from _util import assert_close, lens_mask
from vf_b200 import _lib

pytestmark = pytest.mark.gpu

H, S = 4, 256


def _view(t):
    d = _lib.Tensor4d()
    d.data = t.data_ptr()
    for i in range(4):
        d.size[i] = t.size(i)
        d.stride[i] = t.stride(i)
    return d


def _inputs(seed, B=3, L=384, lens=(384, 200, 77)):
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(seed)
    bf = torch.bfloat16
    q, k, v = (torch.randn(B, H, L, 64, generator=g).to(bf).to(dev) for _ in range(3))
    rk, rq = ((torch.randn(1, H, 2 * S, 64, generator=g) * 0.4).to(bf).to(dev) for _ in range(2))
    sl = torch.tensor(lens, dtype=torch.int32, device=dev)
    return q, k, v, rk, rq, sl


def _args(q, k, v, out, rk, rq, sl):
    a = _lib.DebertaFusedArgs()
    a.dtype = _lib.VF_DTYPE_BF16
    a.q, a.k, a.v, a.out = _view(q), _view(k), _view(v), _view(out)
    a.seq_lengths = sl.data_ptr()
    a.rel_key, a.rel_query = _view(rk), _view(rq)
    a.has_sm_scale, a.sm_scale = 1, 0.07
    a.position_buckets, a.max_relative_distance, a.use_log_bucket = S, 512, 1
    return a


def _with_workspace(lib, x, stream):
    q, k, v, rk, rq, sl = x
    out = torch.empty_like(q)
    n = lib.vf_deberta_fused_workspace_bytes(q.size(0), H, q.size(2), k.size(2))
    ws = torch.empty(n + 256, dtype=torch.uint8, device=q.device)
    wsp = (ws.data_ptr() + 255) // 256 * 256
    rc = lib.vf_deberta_attention_fused_fwd(ctypes.byref(_args(q, k, v, out, rk, rq, sl)), ctypes.c_void_p(wsp), n,
                                            ctypes.c_void_p(stream))
    assert rc == _lib.VF_OK, lib.vf_last_error()
    torch.cuda.synchronize()
    return out


def test_noalloc_entry_matches_workspace_entry_on_two_calls():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    for seed, lens in ((0, (384, 200, 77)), (1, (129, 384, 1))):
        x = _inputs(seed, lens=lens)
        q, k, v, rk, rq, sl = x
        ref = _with_workspace(lib, x, stream)
        out = torch.full_like(q, float("nan"))
        rc = lib.vf_deberta_attention_fused_noalloc_fwd(ctypes.byref(_args(q, k, v, out, rk, rq, sl)),
                                                        ctypes.c_void_p(stream))
        assert rc == _lib.VF_OK, lib.vf_last_error()
        torch.cuda.synchronize()
        assert_close(out, ref.float(), lens_mask(sl.cpu(), q.size(2)), what=f"noalloc call seed {seed}")
        pad = ~lens_mask(sl.cpu(), q.size(2))
        assert (out.float().cpu()[pad[:, None, :].expand(out.shape[:3])] == 0).all()


def test_noalloc_entry_refuses_calls_beyond_its_scratch():
    lib = _lib.load()
    big = 4096   # 4 heads x (4096 + 4096) rows x 64 x 2 tables x 2 bytes = 8 MiB plus the unit order
    q = torch.zeros(1, H, big, 64, dtype=torch.bfloat16, device="cuda")
    rk = torch.zeros(1, H, 2 * S, 64, dtype=torch.bfloat16, device="cuda")
    sl = torch.tensor([big], dtype=torch.int32, device="cuda")
    rc = lib.vf_deberta_attention_fused_noalloc_fwd(ctypes.byref(_args(q, q, q, q, rk, rk, sl)), None)
    assert rc == _lib.VF_EUNSUPPORTED
    assert "static scratch" in lib.vf_last_error().decode()
