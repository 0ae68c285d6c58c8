"""ctypes binding of libneedle_cuda.so (include/needle_cuda.h).

The library must exist (built by needle_b200.build) -- there is no CPU fallback: every call
either runs on the GPU or raises NeedleError.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libneedle_cuda.so")

# packages/needle.js/src/errors.ts:1-11, in order: status k (1..10) is CODES[k - 1].
CODES = ["INVALID_CACT", "UNSUPPORTED_CACT", "WEIGHTS_NOT_FOUND", "WEIGHTS_INTEGRITY",
         "WEBGPU_UNAVAILABLE", "BACKEND_UNAVAILABLE", "CONTEXT_OVERFLOW", "INVALID_TOOL_SCHEMA",
         "GRAMMAR_DEAD_END", "GENERATION_ABORTED"]
TOKEN_PENDING = -1
ALLOWED_MASK = -2  # NEEDLE_ALLOWED_MASK: allowed_offset names a slot of the device mask pool
KV_INT8 = 0
KV_FLOAT32 = 1
NUMERICS_EXACT = 0
NUMERICS_FAST = 1
NUMERICS_FAST_ATTENTION = 2
NOALLOC_MAX_FLOATS = 1 << 20  # NEEDLE_NOALLOC_MAX_FLOATS
WAIT_ATTENTION, WAIT_TABLE_GEMV, WAIT_TENSOR_GEMM, WAIT_SELFTEST = 1, 2, 4, 8  # NEEDLE_WAIT_*


class NeedleError(RuntimeError):
    """NeedleError (packages/needle.js/src/errors.ts:14-24): a message with a stable code."""

    def __init__(self, code: str, message: str):
        super().__init__(message)
        self.code = code


class Opts(C.Structure):
    _fields_ = [("struct_size", C.c_uint32), ("device", C.c_int32), ("max_seqs", C.c_int32),
                ("max_len", C.c_int32), ("max_sink", C.c_int32), ("kv_mode", C.c_int32),
                ("numerics", C.c_int32), ("micro_batches", C.c_int32), ("sched_chunk", C.c_int32),
                ("sched_items", C.c_int32), ("reserved", C.c_int32 * 6)]


class Geometry(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "vocabulary_size", "model_dimension", "heads", "kv_heads", "layers", "head_dimension",
        "maximum_sequence_length", "hadamard_dimension", "mhc_lanes", "engram_slots",
        "engram_sub_dimension", "engram_tables", "engram_taps", "engram_dilation", "kv_window",
        "kv_bits", "engram_order_count")] + [
        ("engram_orders", C.c_int32 * 4), ("engram_site_count", C.c_int32),
        ("engram_sites", C.c_int32 * 4), ("rope_theta", C.c_float), ("num_tensors", C.c_int32),
        ("kv_capacity", C.c_int32)]


class StepItem(C.Structure):
    _fields_ = [("seq", C.c_int32), ("token", C.c_int32), ("select", C.c_int32),
                ("allowed_count", C.c_int32), ("allowed_offset", C.c_uint32)]


class Selected(C.Structure):
    _fields_ = [("id", C.c_int32), ("reserved", C.c_int32), ("log_probability", C.c_double)]


class CqMatrixDesc(C.Structure):
    _fields_ = [("packed", C.c_void_p), ("norms", C.c_void_p), ("rows", C.c_int32),
                ("input_size", C.c_int32), ("group_size", C.c_int32), ("bits", C.c_int32)]


EXPORTS = {
    "needle_cuda_last_error": (C.c_char_p, []),
    "needle_cuda_default_opts": (C.c_int, [C.POINTER(Opts)]),
    "needle_cuda_open": (C.c_int, [C.c_void_p, C.c_size_t, C.POINTER(Opts), C.POINTER(C.c_void_p)]),
    "needle_cuda_close": (C.c_int, [C.c_void_p]),
    "needle_cuda_geometry": (C.c_int, [C.c_void_p, C.POINTER(Geometry)]),
    "needle_cuda_seq_reset": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32]),
    "needle_cuda_seq_reset_ex": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "needle_cuda_confidence": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_double)]),
    "needle_cuda_seq_position": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int32)]),
    "needle_cuda_step": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t,
                                   C.c_void_p, C.c_void_p]),
    "needle_cuda_step_begin": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32]),
    "needle_cuda_step_end": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_size_t, C.c_void_p]),
    "needle_cuda_resident_forward": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                               C.c_void_p, C.c_int32, C.c_int32]),
    "needle_cuda_resident_finish": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p]),
    "needle_cuda_resident_select": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p]),
    "needle_cuda_prefill": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32, C.c_void_p]),
    "needle_cuda_read_kv": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.c_void_p, C.POINTER(C.c_int32)]),
    "needle_cuda_read_kv_f32": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                          C.POINTER(C.c_int32)]),
    "needle_cuda_read_lanes": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p]),
    "needle_cuda_matvec": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                     C.c_int32, C.c_void_p]),
    "needle_cuda_row": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "needle_cuda_cq_matvec_dev": (C.c_int, [C.POINTER(CqMatrixDesc), C.c_void_p, C.c_void_p,
                                            C.c_int32, C.c_void_p, C.c_void_p]),
    "needle_cuda_cq_matvec_dev_fast": (C.c_int, [C.POINTER(CqMatrixDesc), C.c_void_p, C.c_void_p,
                                                 C.c_int32, C.c_void_p, C.c_void_p]),
    "needle_cuda_cq_matvec_dev_noalloc": (C.c_int, [C.POINTER(CqMatrixDesc), C.c_void_p, C.c_void_p,
                                                    C.c_int32, C.c_void_p, C.c_void_p]),
    "needle_cuda_attention_dev": (C.c_int, [C.c_void_p] * 6 + [C.c_int32, C.c_int32, C.c_void_p,
                                                                C.c_void_p]),
    "needle_cuda_attention_dev_fast": (C.c_int, [C.c_void_p] * 6 + [C.c_int32, C.c_int32, C.c_void_p,
                                                                     C.c_void_p]),
    "needle_cuda_wait_status": (C.c_int, [C.c_int32, C.POINTER(C.c_uint32), C.c_int32]),
    "needle_cuda_wait_selftest": (C.c_int, [C.c_uint64, C.c_void_p]),
    "needle_cuda_stream": (C.c_void_p, [C.c_void_p]),
    "needle_cuda_sched_load": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                         C.c_int32]),
    "needle_cuda_sched_step": (C.c_int, [C.c_void_p, C.c_int32]),
    "needle_cuda_sched_status": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64), C.POINTER(C.c_int64),
                                           C.POINTER(C.c_int32), C.c_void_p]),
    "needle_cuda_sched_ids": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "needle_cuda_sched_slot": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                         C.POINTER(C.c_int32)]),
    "needle_cuda_mask_pool": (C.c_int, [C.c_void_p, C.c_int32]),
    "needle_cuda_masks_put": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p]),
    "needle_cuda_kernel_launches": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    "needle_cuda_check_guards": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "needle_cuda_profile": (C.c_int, [C.c_void_p, C.c_int32]),
    "needle_cuda_profile_read": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_char_p),
                                           C.POINTER(C.c_double), C.POINTER(C.c_int64),
                                           C.POINTER(C.c_int32)]),
    # include/needle_grammar.h
    "needle_grammar_tools": (C.c_int, [C.c_char_p, C.c_int32, C.POINTER(C.c_void_p)]),
    "needle_grammar_schema": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "needle_grammar_clone": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "needle_grammar_free": (None, [C.c_void_p]),
    "needle_grammar_feed": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int32, C.POINTER(C.c_int32)]),
    "needle_grammar_complete": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "needle_grammar_result": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int32, C.POINTER(C.c_int32)]),
    "needle_vocab_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_int32), C.c_int32, C.POINTER(C.c_void_p)]),
    "needle_vocab_free": (None, [C.c_void_p]),
    "needle_grammar_allowed": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(C.c_uint32), C.c_int32,
                                         C.POINTER(C.c_int32)]),
    "needle_grammar_allowed_batch": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(C.c_int64), C.c_int32, C.c_void_p,
                                               C.c_int32, C.POINTER(C.c_uint32), C.c_int32, C.POINTER(C.c_int32)]),
    "needle_mask_cache_open": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.POINTER(C.c_void_p)]),
    "needle_mask_cache_free": (None, [C.c_void_p]),
    "needle_mask_cache_table": (C.c_int, [C.c_void_p, C.POINTER(C.POINTER(C.c_uint32)), C.POINTER(C.c_int32)]),
    "needle_mask_cache_lookup": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(C.c_int64), C.c_int32,
                                           C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_int32)]),
    "needle_mask_cache_stats": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64), C.POINTER(C.c_int64),
                                          C.POINTER(C.c_int64)]),
}

_lib = None


def lib():
    """Loads libneedle_cuda.so; raises NeedleError(BACKEND_UNAVAILABLE) when it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NeedleError("BACKEND_UNAVAILABLE",
                              f"{LIB_PATH} is missing: build it with needle_b200.build.build()")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in EXPORTS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != 0:
        msg = lib().needle_cuda_last_error().decode(errors="replace")
        code = CODES[rc - 1] if 1 <= rc <= len(CODES) else "BACKEND_UNAVAILABLE"
        raise NeedleError(code, msg)


def ptr(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def default_opts(**kw) -> Opts:
    o = Opts()
    check(lib().needle_cuda_default_opts(C.byref(o)))
    for k, v in kw.items():
        setattr(o, k, v)
    return o
