"""ctypes binding of the C ABI in include/need_scan.h (libneed_scan.so).

The structures mirror the header field for field; ``load()`` opens the in-tree
library and declares every entry point.  Nothing here touches the GPU: the
first CUDA call happens inside an entry point.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_char_p, c_double, c_int32, c_int64, c_size_t, c_uint32,
                    c_void_p, c_uint64)

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_lib", "libneed_scan.so")
ABI_VERSION = 2

# need_status
OK, ERR_INVALID, ERR_UNSUPPORTED, ERR_CUDA, ERR_WORKSPACE = 0, 1, 2, 3, 4
# need_dtype
F32, BF16, F16 = 0, 1, 2
# need_form
FORM_AFFINE, FORM_GATED, FORM_SSD, FORM_RETENTION = 0, 1, 2, 3


class NeedView(Structure):
    _fields_ = [("ptr", c_void_p), ("stride_b", c_int64), ("stride_h", c_int64), ("stride_t", c_int64)]


class NeedScanArgs(Structure):
    _fields_ = [
        ("form", c_int32), ("dtype", c_int32), ("decay_dtype", c_int32), ("decay_per_row", c_int32),
        ("nb", c_int64), ("nh", c_int64), ("T", c_int64), ("C", c_int64),
        ("in_", NeedView * 5),
        ("out", c_void_p), ("out_stride_b", c_int64), ("out_stride_h", c_int64), ("out_stride_t", c_int64),
        ("d_skip", c_void_p), ("dt_min", c_double), ("dt_max", c_double),
        ("h0", c_void_p), ("h_final", c_void_p),
        ("seg_start", c_void_p), ("seg_stride_b", c_int64), ("seg_stride_t", c_int64),
        ("summary", c_void_p), ("tile_prod", c_void_p), ("tile_carry", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", c_size_t),
        ("sp_list", c_void_p), ("sp_list_words", c_uint64),
    ]


class NeedVerifyArgs(Structure):
    _fields_ = [
        ("form", c_int32), ("dtype", c_int32), ("nseq", c_int64), ("C", c_int64),
        ("states", c_void_p), ("slot", c_void_p), ("cu_k", c_void_p), ("total_k", c_int64),
        ("in_", c_void_p * 5), ("d_skip", c_void_p), ("dt_min", c_double), ("dt_max", c_double),
        ("y", c_void_p), ("states_k", c_void_p), ("head_dim", c_int64),
        ("conv_k", c_int32), ("conv_weight", c_void_p), ("conv_bias", c_void_p),
        ("conv_hist", c_void_p), ("conv_hist_k", c_void_p),
    ]


TOK_U16, TOK_U32, TOK_I32, TOK_I64 = 0, 1, 2, 3


class NeedSegmentArgs(Structure):
    _fields_ = [
        ("tokens", c_void_p), ("token_dtype", c_int32), ("nb", c_int64), ("T", c_int64),
        ("tok_stride_b", c_int64), ("tok_stride_t", c_int64), ("eos_id", c_int64), ("bos_id", c_int64),
        ("seg_start", c_void_p), ("seg_stride_b", c_int64), ("seg_stride_t", c_int64),
    ]


class NeedConvArgs(Structure):
    _fields_ = [
        ("dtype", c_int32), ("K", c_int32), ("nb", c_int64), ("T", c_int64), ("C", c_int64),
        ("u", c_void_p), ("u_stride_b", c_int64), ("u_stride_t", c_int64),
        ("out", c_void_p), ("out_stride_b", c_int64), ("out_stride_t", c_int64),
        ("weight", c_void_p), ("w_stride_c", c_int64), ("w_stride_k", c_int64), ("bias", c_void_p),
        ("seg_start", c_void_p), ("seg_stride_b", c_int64), ("seg_stride_t", c_int64),
    ]


class NeedSsdConv(Structure):
    _fields_ = [
        ("K", c_int32), ("weight", c_void_p), ("w_stride_c", c_int64), ("w_stride_k", c_int64), ("bias", c_void_p),
    ]


class NeedNormArgs(Structure):
    _fields_ = [
        ("dtype", c_int32), ("weight_dtype", c_int32), ("nb", c_int64), ("T", c_int64), ("C", c_int64),
        ("x", c_void_p), ("x_stride_b", c_int64), ("x_stride_t", c_int64),
        ("out", c_void_p), ("out_stride_b", c_int64), ("out_stride_t", c_int64),
        ("weight", c_void_p), ("eps", c_double),
    ]


class NeedAssocArgs(Structure):
    _fields_ = [
        ("dtype", c_int32), ("qk_dtype", c_int32),
        ("nb", c_int64), ("T", c_int64), ("r", c_int64), ("d", c_int64),
        ("q_raw", c_void_p), ("q_stride_b", c_int64), ("q_stride_t", c_int64),
        ("k_raw", c_void_p), ("k_stride_b", c_int64), ("k_stride_t", c_int64),
        ("v", c_void_p), ("v_stride_b", c_int64), ("v_stride_t", c_int64),
        ("write_mask", c_void_p), ("mask_dtype", c_int32), ("mask_stride_b", c_int64), ("mask_stride_t", c_int64),
        ("out", c_void_p), ("out_stride_b", c_int64), ("out_stride_t", c_int64),
        ("eps", c_double), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
    ]


class NeedAssocStepArgs(Structure):
    _fields_ = [
        ("dtype", c_int32), ("qk_dtype", c_int32), ("nseq", c_int64), ("r", c_int64), ("d", c_int64),
        ("q_raw", c_void_p), ("q_stride", c_int64), ("k_raw", c_void_p), ("k_stride", c_int64),
        ("v", c_void_p), ("v_stride", c_int64), ("write_mask", c_void_p), ("mask_dtype", c_int32),
        ("state", c_void_p), ("state_stride_n", c_int64), ("state_stride_r", c_int64),
        ("denom", c_void_p), ("denom_stride_n", c_int64), ("slot", c_void_p),
        ("out", c_void_p), ("out_stride", c_int64), ("eps", c_double),
    ]


# every symbol the header declares, with (restype, argtypes)
SIGNATURES = {
    "need_abi_version": (c_int32, []),
    "need_last_error": (c_char_p, []),
    "need_scan_chunk_len": (c_int64, [c_int32, c_int32, c_int32, c_int32]),
    "need_scan_workspace_size": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int64, c_int64, c_int64, c_int64]),
    "need_workspace_error": (c_int32, [c_void_p, POINTER(c_uint32), c_void_p]),
    "need_test_set_lookback_polls": (None, [c_uint32]),
    "need_affine_recurrence_scan": (c_int32, [POINTER(NeedScanArgs), c_void_p]),
    "need_affine_recurrence_scan_backward": (c_int32, [POINTER(NeedScanArgs), c_void_p]),
    "need_ssd_scan": (c_int32, [POINTER(NeedScanArgs), c_void_p]),
    "need_ssd_scan_rms_norm": (c_int32, [POINTER(NeedScanArgs), c_void_p, c_int32, c_double, c_void_p]),
    "need_ssd_conv_scan": (c_int32, [POINTER(NeedScanArgs), POINTER(NeedSsdConv), c_void_p, c_int32, c_double,
                                     c_void_p]),
    "need_rms_norm": (c_int32, [POINTER(NeedNormArgs), c_void_p]),
    "need_assoc_memory_workspace_size": (c_size_t, [c_int64, c_int64, c_int64, c_int32]),
    "need_assoc_memory": (c_int32, [POINTER(NeedAssocArgs), c_void_p]),
    "need_assoc_memory_step": (c_int32, [POINTER(NeedAssocStepArgs), c_void_p]),
    "need_recurrent_retention_scan": (c_int32, [POINTER(NeedScanArgs), c_void_p]),
    "need_gated_scan": (c_int32, [POINTER(NeedScanArgs), c_void_p]),
    "need_gated_scan_noalloc": (c_int32, [POINTER(NeedScanArgs), c_void_p]),
    "need_gated_scan_noalloc_error": (c_int32, [POINTER(c_uint32), c_void_p]),
    "need_ragged_verify": (c_int32, [POINTER(NeedVerifyArgs), c_void_p]),
    "need_segment_starts": (c_int32, [POINTER(NeedSegmentArgs), c_void_p]),
    "need_ssd_conv_silu": (c_int32, [POINTER(NeedConvArgs), c_void_p]),
    "need_commit_states": (c_int32, [c_int32, c_int64, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                                     c_void_p, c_void_p]),
    "need_sp_local_scan": (c_int32, [POINTER(NeedScanArgs), c_int32, c_void_p]),
    "need_sp_list_size": (c_size_t, [c_int32, c_int64, c_int64, c_int64, c_int64]),
    "need_sp_fixup": (c_int32, [POINTER(NeedScanArgs), c_void_p, c_int32, c_int32, c_void_p]),
}

_LIB = None


class NeedError(RuntimeError):
    """A C-ABI call returned a non-zero need_status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed (status {code}): {msg}")
        self.code = code


def load(path: str = LIB_PATH):
    """Opens libneed_scan.so (raises if it has not been built) and declares its entry points."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m need_b200.build` "
                           "(there is no CPU fallback for the scan kernels)")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    ver = lib.need_abi_version()
    if ver != ABI_VERSION:
        raise RuntimeError(f"libneed_scan ABI version {ver}, expected {ABI_VERSION}")
    _LIB = lib
    return lib


def check(fn: str, code: int) -> None:
    if code != OK:
        msg = _LIB.need_last_error().decode(errors="replace") if _LIB is not None else ""
        raise NeedError(fn, code, msg)
