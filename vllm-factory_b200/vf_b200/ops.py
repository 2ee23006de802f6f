"""torch.ops.vf_b200.* — custom ops over the libvf_b200 C ABI.

Both ops take borrowed tensors (any strides the kernels accept; others are made
contiguous), allocate only their output, and launch on the caller's current CUDA stream.
CPU tensors raise: there is no CPU path behind these ops.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib

_DTYPE_CODE = {
    torch.float32: _lib.VF_DTYPE_F32,
    torch.float16: _lib.VF_DTYPE_F16,
    torch.bfloat16: _lib.VF_DTYPE_BF16,
}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _t4(t: Optional[torch.Tensor]) -> _lib.Tensor4d:
    d = _lib.Tensor4d()
    if t is None:
        return d
    if t.dim() != 4:
        raise ValueError(f"expected a 4-D tensor, got shape {tuple(t.shape)}")
    d.data = t.data_ptr()
    for i in range(4):
        d.size[i] = t.shape[i]
        d.stride[i] = t.stride(i)
    return d


def _tma_ready(t: torch.Tensor) -> torch.Tensor:
    """Returns `t` if its layout can be described by a TMA tensor map, else a contiguous copy.

    TMA needs a unit innermost stride, 16-byte aligned base and 16-byte multiple strides.
    """
    es = t.element_size()
    ok = (t.stride(-1) == 1 and t.data_ptr() % 16 == 0
          and all(t.stride(i) > 0 and (t.stride(i) * es) % 16 == 0 for i in range(3)))
    return t if ok else t.contiguous()


def _require_cuda(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"vf_b200: {name} must be a CUDA tensor (no CPU implementation)")


def _stream_ptr(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


@torch.library.custom_op("vf_b200::rpb_attention", mutates_args=())
def rpb_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  rpb_table: Optional[torch.Tensor], num_buckets: int, max_distance: int,
                  is_decoder: bool, padding_mask: Optional[torch.Tensor],
                  dropout_p: float, softmax_scale: float) -> torch.Tensor:
    """T5 relative-position-bias attention; semantics of kernels/flash_attention_rpb.py:296."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share a dtype")
    q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    out = torch.empty_like(q)
    if out.stride(-1) != 1 or (out.stride(2) * out.element_size()) % 16 != 0:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    args = _lib.RpbArgs()
    args.dtype = _dtype_code(q)
    args.q, args.k, args.v, args.out = _t4(q), _t4(k), _t4(v), _t4(out)
    if rpb_table is not None:
        _require_cuda("rpb_table", rpb_table)
        if rpb_table.dim() != 2:
            raise ValueError("rpb_table must be [num_buckets, heads]")
        args.rpb_table = rpb_table.data_ptr()
        args.table_rows, args.table_cols = rpb_table.shape
        args.table_stride_row, args.table_stride_col = rpb_table.stride()
        args.table_dtype = _dtype_code(rpb_table)
    args.num_buckets = int(num_buckets)
    args.max_distance = int(max_distance)
    args.is_decoder = int(bool(is_decoder))
    if padding_mask is not None:
        _require_cuda("padding_mask", padding_mask)
        args.padding_mask = _t4(padding_mask)
        args.mask_dtype = _dtype_code(padding_mask)
    args.dropout_p = float(dropout_p)
    args.softmax_scale = float(softmax_scale)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().vf_rpb_attention_fwd(ctypes.byref(args), _stream_ptr(q.device)))
    return out


@rpb_attention.register_fake
def _rpb_attention_fake(q, k, v, rpb_table, num_buckets, max_distance, is_decoder,
                        padding_mask, dropout_p, softmax_scale):
    return torch.empty_like(q)


@torch.library.custom_op("vf_b200::deberta_attention", mutates_args=())
def deberta_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      seq_lengths: Optional[torch.Tensor], pos_key: Optional[torch.Tensor],
                      pos_query: Optional[torch.Tensor], causal: bool,
                      sm_scale: Optional[float], position_buckets: int,
                      max_relative_distance: int, use_log_bucket: bool) -> torch.Tensor:
    """DeBERTa disentangled attention; semantics of kernels/flash_deberta_attention.py:455."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(name, t)
    if not (q.dtype == k.dtype == v.dtype):
        raise TypeError("q, k, v must share a dtype")
    q, k, v = _tma_ready(q), _tma_ready(k), _tma_ready(v)
    out = torch.empty_like(q)
    if out.stride(-1) != 1 or (out.stride(2) * out.element_size()) % 16 != 0:
        out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    args = _lib.DebertaArgs()
    args.dtype = _dtype_code(q)
    args.q, args.k, args.v, args.out = _t4(q), _t4(k), _t4(v), _t4(out)
    if seq_lengths is not None:
        _require_cuda("seq_lengths", seq_lengths)
        if seq_lengths.dtype != torch.int32 or not seq_lengths.is_contiguous():
            seq_lengths = seq_lengths.to(torch.int32).contiguous()
        if seq_lengths.numel() != q.shape[0]:
            raise ValueError("seq_lengths must have one entry per batch row")
        args.seq_lengths = seq_lengths.data_ptr()
    for name, t in (("pos_key", pos_key), ("pos_query", pos_query)):
        if t is not None:
            _require_cuda(name, t)
            if t.dtype != q.dtype:
                raise TypeError(f"{name} must have the dtype of q")
    args.pos_key = _t4(pos_key)
    args.pos_query = _t4(pos_query)
    args.causal = int(bool(causal))
    args.has_sm_scale = int(sm_scale is not None)
    args.sm_scale = float(sm_scale) if sm_scale is not None else 0.0
    args.position_buckets = int(position_buckets)
    args.max_relative_distance = int(max_relative_distance)
    args.use_log_bucket = int(bool(use_log_bucket))
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().vf_deberta_attention_fwd(ctypes.byref(args), _stream_ptr(q.device)))
    return out


@deberta_attention.register_fake
def _deberta_attention_fake(q, k, v, seq_lengths, pos_key, pos_query, causal, sm_scale,
                            position_buckets, max_relative_distance, use_log_bucket):
    return torch.empty_like(q)
