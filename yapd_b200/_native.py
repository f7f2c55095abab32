"""ctypes binding of ``include/yapd_select.h`` (the library's C ABI).

The structures below mirror the header field by field.  Loading fails loudly
when the in-tree library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

from .build import LIB

YAPD_OK = 0
YAPD_DTYPE_F32 = 0
YAPD_DTYPE_BF16 = 1
YAPD_HISTORY_NONE = 0
YAPD_HISTORY_BITMAP = 1
YAPD_HISTORY_BYTES = 2
YAPD_NOISE_PHILOX = 0
YAPD_NOISE_EXPLICIT = 1
YAPD_MAX_V = 8208
YAPD_MAX_L = 32
YAPD_ABI_VERSION = 4
YAPD_STATUS_WAIT_TIMEOUT = 1
YAPD_STATUS_INTERNAL = 2
YAPD_STATUS_ROWS_SKIPPED = 4
YAPD_STATUS_CANDIDATE_OVERFLOW = 8

EXPORTED = [
    "yapd_abi_version", "yapd_status_string", "yapd_select_workspace_size",
    "yapd_sample_workspace_size", "yapd_clear_status", "yapd_read_status",
    "yapd_select_step", "yapd_sample_rows", "yapd_select_step_noalloc",
    "yapd_lmhead_workspace_size", "yapd_lmhead_select_step",
]
YAPD_NOALLOC_MAX_POSITIONS = 16384


class Sampling(C.Structure):
    _fields_ = [
        ("temperature", C.c_void_p), ("top_k", C.c_void_p), ("top_p", C.c_void_p),
        ("min_p", C.c_void_p), ("rep_penalty", C.c_void_p),
        ("temperature_s", C.c_float), ("top_k_s", C.c_int32), ("top_p_s", C.c_float),
        ("min_p_s", C.c_float), ("rep_penalty_s", C.c_float),
        ("zero_temp_greedy", C.c_int32), ("history_kind", C.c_int32),
        ("history", C.c_void_p), ("history_stride", C.c_int64),
    ]


class Noise(C.Structure):
    _fields_ = [
        ("kind", C.c_int32), ("seed", C.c_uint64), ("offset", C.c_uint64),
        ("gumbel_tok", C.c_void_p), ("gt_stride_req", C.c_int64), ("gt_stride_pos", C.c_int64),
        ("gumbel_pos", C.c_void_p),
    ]


class EngineState(C.Structure):
    _fields_ = [
        ("xt_full", C.c_void_p), ("xt_stride", C.c_int64), ("blk_start", C.c_void_p),
        ("cache_len", C.c_void_p), ("n_speech", C.c_void_p), ("blk_limit", C.c_int64),
        ("cache_limit", C.c_int64), ("flags", C.c_void_p),
    ]


class SelectArgs(C.Structure):
    _fields_ = [
        ("B", C.c_int32), ("nb", C.c_int32), ("L", C.c_int32), ("V", C.c_int32), ("K", C.c_int32),
        ("mask_id", C.c_int64), ("stop_id", C.c_int64),
        ("logits_dtype", C.c_int32), ("logits", C.c_void_p),
        ("stride_req", C.c_int64), ("stride_branch", C.c_int64), ("stride_pos", C.c_int64),
        ("logits_numel", C.c_int64),
        ("xt", C.c_void_p), ("k_step", C.c_void_p), ("is_commit", C.c_void_p),
        ("log_prior", C.c_void_p), ("sched_t", C.c_void_p), ("q_t", C.c_void_p),
        ("cfg_scale", C.c_float), ("cfg_one_plus", C.c_float), ("pmi_lambda", C.c_float),
        ("pos_noise", C.c_int32), ("use_quantile", C.c_int32), ("dense", C.c_int32),
        ("sampling", Sampling), ("noise", Noise),
        ("xt_out", C.c_void_p), ("sampled", C.c_void_p), ("pmi", C.c_void_p),
        ("n_unmask", C.c_void_p), ("n_mask_after", C.c_void_p), ("hit_eos", C.c_void_p),
        ("k_step_out", C.c_void_p), ("is_commit_out", C.c_void_p),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("prof_event_begin", C.c_void_p), ("prof_event_end", C.c_void_p),
        ("engine", C.c_void_p), ("positions_sampled", C.c_void_p), ("wait_limit_ns", C.c_int64),
        ("quantile_lerp", C.c_int32),
    ]


class SampleArgs(C.Structure):
    _fields_ = [
        ("R", C.c_int32), ("V", C.c_int32), ("logits_dtype", C.c_int32), ("logits", C.c_void_p),
        ("stride_row", C.c_int64), ("logits_numel", C.c_int64),
        ("sampling", Sampling), ("noise", Noise),
        ("sampled", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("wait_limit_ns", C.c_int64),
    ]


class LmheadArgs(C.Structure):
    _fields_ = [
        ("hidden", C.c_void_p),
        ("h_stride_req", C.c_int64), ("h_stride_branch", C.c_int64), ("h_stride_pos", C.c_int64),
        ("hidden_numel", C.c_int64),
        ("weight", C.c_void_p), ("w_stride", C.c_int64), ("weight_numel", C.c_int64),
        ("D", C.c_int32), ("logits_out", C.c_void_p),
        ("select", SelectArgs),
    ]


_lib = None


def lib():
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB):
        raise RuntimeError(
            f"yapd_b200 CUDA library not found at {LIB}; run `python -m yapd_b200.build` "
            "(there is no CPU fallback)")
    h = C.CDLL(LIB)
    h.yapd_abi_version.restype = C.c_int
    h.yapd_status_string.restype = C.c_char_p
    h.yapd_status_string.argtypes = [C.c_int]
    h.yapd_select_workspace_size.restype = C.c_size_t
    h.yapd_select_workspace_size.argtypes = [C.c_int32, C.c_int32]
    h.yapd_sample_workspace_size.restype = C.c_size_t
    h.yapd_sample_workspace_size.argtypes = [C.c_int32]
    h.yapd_clear_status.restype = C.c_int
    h.yapd_clear_status.argtypes = [C.c_void_p, C.c_void_p]
    h.yapd_read_status.restype = C.c_int
    h.yapd_read_status.argtypes = [C.c_void_p, C.c_void_p, C.POINTER(C.c_uint32)]
    h.yapd_select_step.restype = C.c_int
    h.yapd_select_step.argtypes = [C.POINTER(SelectArgs), C.c_void_p]
    h.yapd_sample_rows.restype = C.c_int
    h.yapd_sample_rows.argtypes = [C.POINTER(SampleArgs), C.c_void_p]
    h.yapd_select_step_noalloc.restype = C.c_int
    h.yapd_select_step_noalloc.argtypes = [C.POINTER(SelectArgs), C.c_void_p]
    h.yapd_lmhead_workspace_size.restype = C.c_size_t
    h.yapd_lmhead_workspace_size.argtypes = [C.c_int32, C.c_int32]
    h.yapd_lmhead_select_step.restype = C.c_int
    h.yapd_lmhead_select_step.argtypes = [C.POINTER(LmheadArgs), C.c_void_p]
    if h.yapd_abi_version() != YAPD_ABI_VERSION:
        raise RuntimeError("yapd_select ABI version mismatch")
    _lib = h
    return h


def check(rc: int) -> None:
    if rc != YAPD_OK:
        msg = lib().yapd_status_string(rc).decode()
        raise RuntimeError(f"yapd_select error {rc}: {msg}")
