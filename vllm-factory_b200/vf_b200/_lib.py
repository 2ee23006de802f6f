"""ctypes binding of libvf_b200.so (include/vf_b200.h).

This is the binding a maintainer of the reference would add: the reference's Python
launchers (kernels/flash_attention_rpb.py:296, kernels/flash_deberta_attention.py:455)
called Triton; here they call the C entry points below.  Loading fails loudly: there is
no CPU or Triton fallback behind this module.
"""
from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = Path(os.environ.get("VF_B200_LIB", str(_PKG / "libvf_b200.so")))

VF_OK = 0
VF_EINVAL = -1
VF_EUNSUPPORTED = -2
VF_ECUDA = -3

VF_DTYPE_F32 = 0
VF_DTYPE_F16 = 1
VF_DTYPE_BF16 = 2

ABI_VERSION = 1

EXPORTED_SYMBOLS = (
    "vf_rpb_attention_fwd",
    "vf_rpb_attention_varlen_fwd",
    "vf_deberta_attention_fwd",
    "vf_deberta_attention_varlen_fwd",
    "vf_deberta_attention_fused_fwd",
    "vf_deberta_attention_fused_varlen_fwd",
    "vf_deberta_fused_workspace_bytes",
    "vf_deberta_attention_fused_noalloc_fwd",
    "vf_gated_act_fwd",
    "vf_add_layer_norm_fwd",
    "vf_span_scores_fwd",
    "vf_linear_act_fwd",
    "vf_t5_relative_bucket",
    "vf_deberta_log_bucket",
    "vf_last_error",
    "vf_device_error",
    "vf_abi_version",
    "vf_selftest_wait_timeout",
)


class Tensor4d(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("size", ctypes.c_int64 * 4),
        ("stride", ctypes.c_int64 * 4),
    ]


class RpbArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("q", Tensor4d),
        ("k", Tensor4d),
        ("v", Tensor4d),
        ("out", Tensor4d),
        ("rpb_table", ctypes.c_void_p),
        ("table_rows", ctypes.c_int64),
        ("table_cols", ctypes.c_int64),
        ("table_stride_row", ctypes.c_int64),
        ("table_stride_col", ctypes.c_int64),
        ("table_dtype", ctypes.c_int),
        ("num_buckets", ctypes.c_int32),
        ("max_distance", ctypes.c_int32),
        ("is_decoder", ctypes.c_int32),
        ("padding_mask", Tensor4d),
        ("mask_dtype", ctypes.c_int),
        ("dropout_p", ctypes.c_float),
        ("softmax_scale", ctypes.c_float),
    ]


VF_ACT_GELU_TANH, VF_ACT_GELU_ERF, VF_ACT_RELU, VF_ACT_SILU = 0, 1, 2, 3


class GatedActArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("gate", ctypes.c_void_p),
        ("up", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("gate_row_stride", ctypes.c_int64),
        ("up_row_stride", ctypes.c_int64),
        ("out_row_stride", ctypes.c_int64),
        ("act", ctypes.c_int32),
    ]


class AddLayerNormArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("x", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64),
        ("residual_row_stride", ctypes.c_int64),
        ("out_row_stride", ctypes.c_int64),
        ("eps", ctypes.c_float),
    ]


class LinearActArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("x", ctypes.c_void_p),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("mul", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("x_row_stride", ctypes.c_int64),
        ("weight_row_stride", ctypes.c_int64),
        ("mul_row_stride", ctypes.c_int64),
        ("out_row_stride", ctypes.c_int64),
        ("act", ctypes.c_int32),
    ]


class SpanScoresArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("start_proj", ctypes.c_void_p),
        ("end_proj", ctypes.c_void_p),
        ("start_row_stride", ctypes.c_int64),
        ("end_row_stride", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("span_idx", ctypes.c_void_p),
        ("span_idx_int64", ctypes.c_int32),
        ("idx_stride_span", ctypes.c_int64),
        ("idx_stride_pair", ctypes.c_int64),
        ("classes", ctypes.c_void_p),
        ("class_row_stride", ctypes.c_int64),
        ("class_bias", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("out_dtype", ctypes.c_int),
        ("num_segments", ctypes.c_int32),
        ("word_offsets", ctypes.POINTER(ctypes.c_int64)),
        ("span_offsets", ctypes.POINTER(ctypes.c_int64)),
        ("class_offsets", ctypes.POINTER(ctypes.c_int64)),
    ]


class DebertaArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("q", Tensor4d),
        ("k", Tensor4d),
        ("v", Tensor4d),
        ("out", Tensor4d),
        ("seq_lengths", ctypes.c_void_p),
        ("pos_key", Tensor4d),
        ("pos_query", Tensor4d),
        ("causal", ctypes.c_int32),
        ("has_sm_scale", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("position_buckets", ctypes.c_int32),
        ("max_relative_distance", ctypes.c_int32),
        ("use_log_bucket", ctypes.c_int32),
    ]


class DebertaFusedArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("q", Tensor4d),
        ("k", Tensor4d),
        ("v", Tensor4d),
        ("out", Tensor4d),
        ("seq_lengths", ctypes.c_void_p),
        ("rel_key", Tensor4d),
        ("rel_query", Tensor4d),
        ("causal", ctypes.c_int32),
        ("has_sm_scale", ctypes.c_int32),
        ("sm_scale", ctypes.c_float),
        ("position_buckets", ctypes.c_int32),
        ("max_relative_distance", ctypes.c_int32),
        ("use_log_bucket", ctypes.c_int32),
    ]


class VfError(RuntimeError):
    """A libvf_b200 entry point returned an error code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"vf_b200 error {code}: {msg}")
        self.code = code


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Loads the in-tree library once; raises if it is missing or has the wrong ABI."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} not found: build it with `python -m vf_b200.build` "
                "(or __graft_entry__.build()); there is no fallback implementation")
        lib = ctypes.CDLL(str(LIB_PATH))
        lib.vf_rpb_attention_fwd.argtypes = [ctypes.POINTER(RpbArgs), ctypes.c_void_p]
        lib.vf_rpb_attention_fwd.restype = ctypes.c_int
        lib.vf_rpb_attention_varlen_fwd.argtypes = [ctypes.POINTER(RpbArgs), ctypes.c_void_p, ctypes.c_int32,
                                                    ctypes.c_int32, ctypes.c_void_p]
        lib.vf_rpb_attention_varlen_fwd.restype = ctypes.c_int
        lib.vf_deberta_attention_fwd.argtypes = [ctypes.POINTER(DebertaArgs), ctypes.c_void_p]
        lib.vf_deberta_attention_fwd.restype = ctypes.c_int
        lib.vf_deberta_attention_varlen_fwd.argtypes = [ctypes.POINTER(DebertaArgs), ctypes.c_void_p,
                                                        ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p]
        lib.vf_deberta_attention_varlen_fwd.restype = ctypes.c_int
        lib.vf_deberta_fused_workspace_bytes.argtypes = [ctypes.c_int64] * 4
        lib.vf_deberta_fused_workspace_bytes.restype = ctypes.c_int64
        lib.vf_deberta_attention_fused_fwd.argtypes = [ctypes.POINTER(DebertaFusedArgs), ctypes.c_void_p,
                                                       ctypes.c_int64, ctypes.c_void_p]
        lib.vf_deberta_attention_fused_fwd.restype = ctypes.c_int
        lib.vf_deberta_attention_fused_varlen_fwd.argtypes = [ctypes.POINTER(DebertaFusedArgs), ctypes.c_void_p,
                                                              ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p,
                                                              ctypes.c_int64, ctypes.c_void_p]
        lib.vf_deberta_attention_fused_varlen_fwd.restype = ctypes.c_int
        lib.vf_deberta_attention_fused_noalloc_fwd.argtypes = [ctypes.POINTER(DebertaFusedArgs), ctypes.c_void_p]
        lib.vf_deberta_attention_fused_noalloc_fwd.restype = ctypes.c_int
        lib.vf_gated_act_fwd.argtypes = [ctypes.POINTER(GatedActArgs), ctypes.c_void_p]
        lib.vf_gated_act_fwd.restype = ctypes.c_int
        lib.vf_add_layer_norm_fwd.argtypes = [ctypes.POINTER(AddLayerNormArgs), ctypes.c_void_p]
        lib.vf_add_layer_norm_fwd.restype = ctypes.c_int
        lib.vf_span_scores_fwd.argtypes = [ctypes.POINTER(SpanScoresArgs), ctypes.c_void_p]
        lib.vf_span_scores_fwd.restype = ctypes.c_int
        lib.vf_linear_act_fwd.argtypes = [ctypes.POINTER(LinearActArgs), ctypes.c_void_p]
        lib.vf_linear_act_fwd.restype = ctypes.c_int
        lib.vf_t5_relative_bucket.argtypes = [ctypes.c_int32] * 5 + [ctypes.POINTER(ctypes.c_int32)]
        lib.vf_t5_relative_bucket.restype = ctypes.c_int
        lib.vf_deberta_log_bucket.argtypes = [ctypes.c_int32] * 4 + [ctypes.POINTER(ctypes.c_int32)]
        lib.vf_deberta_log_bucket.restype = ctypes.c_int
        lib.vf_last_error.argtypes = []
        lib.vf_last_error.restype = ctypes.c_char_p
        lib.vf_device_error.argtypes = [ctypes.c_int32]
        lib.vf_device_error.restype = ctypes.c_int
        lib.vf_abi_version.argtypes = []
        lib.vf_abi_version.restype = ctypes.c_int
        lib.vf_selftest_wait_timeout.argtypes = [ctypes.c_int64, ctypes.c_void_p]
        lib.vf_selftest_wait_timeout.restype = ctypes.c_int
        if lib.vf_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{LIB_PATH}: ABI version {lib.vf_abi_version()} != {ABI_VERSION}")
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != VF_OK:
        msg = load().vf_last_error().decode(errors="replace")
        raise VfError(rc, msg)


def t5_relative_bucket(num_buckets: int, max_distance: int, bidirectional: bool, rmin: int, rmax: int):
    """Bucket of every relative position r in [rmin, rmax] (list of ints)."""
    n = rmax - rmin + 1
    buf = (ctypes.c_int32 * n)()
    check(load().vf_t5_relative_bucket(num_buckets, max_distance, int(bidirectional), rmin, rmax, buf))
    return list(buf)


def deberta_log_bucket(bucket_size: int, max_position: int, rmin: int, rmax: int):
    """DeBERTa log-bucket position of every relative position r in [rmin, rmax]."""
    n = rmax - rmin + 1
    buf = (ctypes.c_int32 * n)()
    check(load().vf_deberta_log_bucket(bucket_size, max_position, rmin, rmax, buf))
    return list(buf)


def selftest_wait_timeout(limit_cycles: int = 2_000_000, stream: int = 0) -> None:
    """Runs the bounded-wait self-test kernel (see include/vf_b200.h)."""
    check(load().vf_selftest_wait_timeout(int(limit_cycles), ctypes.c_void_p(stream)))


def device_error(clear: bool = True) -> int:
    rc = load().vf_device_error(int(clear))
    if rc < 0:
        check(rc)
    return rc
