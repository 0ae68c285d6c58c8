"""ctypes binding of the CPU oracle (libneedle_ref.so).  TEST INFRASTRUCTURE ONLY.

The oracle restates the needle.js TypeScript CPU decode path (see needle_ref.h for the file:line
map).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg / reference arm use
this module, always as the checker or the timed CPU baseline -- never as the engine.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "libneedle_ref.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++ only)."""
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < max(
            os.path.getmtime(os.path.join(_HERE, f)) for f in ("needle_ref.cpp", "needle_ref.h")):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "libneedle_ref.so"], check=True)
    return _SO


class RefError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{code}] {message}")
        self.code = code
        self.message = message


class CqDesc(C.Structure):
    _fields_ = [("rows", C.c_int32), ("input_size", C.c_int32), ("group_size", C.c_int32),
                ("bits", C.c_int32), ("packed", C.c_void_p), ("norms", C.c_void_p),
                ("cb2", C.c_void_p), ("cb3", C.c_void_p), ("cb4", C.c_void_p)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = C.CDLL(_SO)
        L.ref_last_error.restype = C.c_char_p
        L.ref_float16_to_number.restype = C.c_double
        L.ref_float16_to_number.argtypes = [C.c_uint32]
        L.ref_number_to_float16.restype = C.c_uint32
        L.ref_number_to_float16.argtypes = [C.c_double]
        L.ref_model_num_tensors.argtypes = [C.c_void_p]
        L.ref_runtime_position.argtypes = [C.c_void_p]
        L.ref_runtime_kv_allocation.argtypes = [C.c_void_p]
        L.ref_model_close.argtypes = [C.c_void_p]
        L.ref_runtime_free.argtypes = [C.c_void_p]
        L.ref_sched_free.argtypes = [C.c_void_p]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _check(rc: int):
    if rc != 0:
        raise RefError(rc, lib().ref_last_error().decode())


def float16_to_number(h: int) -> float:
    return lib().ref_float16_to_number(h)


def number_to_float16(v: float) -> int:
    return lib().ref_number_to_float16(v)


def fwht(values: np.ndarray) -> np.ndarray:
    v = np.ascontiguousarray(values, dtype=np.float32).copy()
    _check(lib().ref_fwht(_p(v), C.c_int32(v.size)))
    return v


class CqMatrix:
    """A free-standing CQ matrix: rows x input_size, packed bitstream + fp16 norms + codebooks."""

    def __init__(self, rows, input_size, group_size, bits, packed, norms, cb2, cb3, cb4):
        self.packed = np.ascontiguousarray(packed, dtype=np.uint8)
        self.norms = np.ascontiguousarray(norms).view(np.uint8)
        self.cb2 = np.ascontiguousarray(cb2, dtype=np.float32)
        self.cb3 = np.ascontiguousarray(cb3, dtype=np.float32)
        self.cb4 = np.ascontiguousarray(cb4, dtype=np.float32)
        self.rows, self.input_size, self.group_size, self.bits = rows, input_size, group_size, bits
        self.desc = CqDesc(rows, input_size, group_size, bits, self.packed.ctypes.data,
                           self.norms.ctypes.data, self.cb2.ctypes.data, self.cb3.ctypes.data,
                           self.cb4.ctypes.data)

    @property
    def input_padded(self):
        g = self.group_size
        return -(-self.input_size // g) * g

    def matvec(self, x, row_start=0, row_count=None):
        if row_count is None:
            row_count = self.rows - row_start
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(row_count, dtype=np.float32)
        _check(lib().ref_cq_matvec_desc(C.byref(self.desc), _p(x), C.c_int32(row_start),
                                        C.c_int32(row_count), _p(y)))
        return y

    def prepare(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.zeros(self.input_padded, dtype=np.float32)
        _check(lib().ref_cq_prepare_desc(C.byref(self.desc), _p(x), _p(out)))
        return out

    def row(self, r):
        out = np.zeros(self.input_size, dtype=np.float32)
        _check(lib().ref_cq_row_desc(C.byref(self.desc), C.c_int32(r), _p(out)))
        return out


class Model:
    """parseCact + CpuBackend operators on an archive (cact.ts:189-562, cpu.ts:12-30)."""

    def __init__(self, archive: bytes):
        self._bytes = np.frombuffer(archive, dtype=np.uint8)
        h = C.c_void_p()
        _check(lib().ref_model_open(_p(self._bytes), C.c_size_t(self._bytes.size), C.byref(h)))
        self.h = h
        f = np.zeros(32, dtype=np.int32)
        theta = C.c_float()
        _check(lib().ref_model_geometry(self.h, _p(f), C.byref(theta)))
        self.fields = f
        self.rope_theta = theta.value
        self.vocab = int(f[5])
        self.dim = int(f[6])
        self.layers = int(f[9])
        self.kv_heads = int(f[8])
        self.head_dim = int(f[10])
        self.lanes = int(f[13])

    def close(self):
        if getattr(self, "h", None):
            lib().ref_model_close(self.h)
            self.h = None

    __del__ = close

    def num_tensors(self):
        return lib().ref_model_num_tensors(self.h)

    def record(self, i):
        info = np.zeros(8, dtype=np.int32)
        off, n = C.c_uint64(), C.c_uint64()
        _check(lib().ref_model_record(self.h, C.c_int32(i), _p(info), C.byref(off), C.byref(n)))
        return dict(dtype=int(info[0]), rank=int(info[1]), shape=tuple(int(s) for s in info[2:2 + info[1]]),
                    group=int(info[6]), bits=int(info[7]), offset=off.value, length=n.value)

    def matvec(self, tensor, x, row_start=0, row_count=None):
        rec = self.record(tensor)
        if row_count is None:
            row_count = rec["shape"][0] - row_start
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(row_count, dtype=np.float32)
        _check(lib().ref_model_matvec(self.h, C.c_int32(tensor), _p(x), C.c_int32(row_start),
                                      C.c_int32(row_count), _p(y)))
        return y

    def row(self, tensor, r):
        rec = self.record(tensor)
        out = np.zeros(rec["shape"][1], dtype=np.float32)
        _check(lib().ref_model_row(self.h, C.c_int32(tensor), C.c_int32(r), _p(out)))
        return out

    def generate_greedy(self, prompt, steps, sink=0, want_logits=True):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        ids = np.zeros(steps, dtype=np.int32)
        lp = np.zeros(steps, dtype=np.float64)
        logits = np.zeros((steps, self.vocab), dtype=np.float32) if want_logits else None
        _check(lib().ref_generate_greedy(self.h, _p(prompt), C.c_int32(prompt.size), C.c_int32(steps),
                                         C.c_int32(sink), _p(ids), _p(lp), _p(logits)))
        return ids, lp, logits

    def decode_many(self, prompts, gen_steps, n_threads, seconds=False):
        offsets = np.zeros(len(prompts) + 1, dtype=np.int32)
        offsets[1:] = np.cumsum([len(p) for p in prompts])
        flat = np.ascontiguousarray(np.concatenate(prompts), dtype=np.int32)
        steps = np.ascontiguousarray(gen_steps, dtype=np.int32)
        last = np.zeros(len(prompts), dtype=np.int32)
        secs = np.zeros(len(prompts), dtype=np.float64)
        processed = C.c_int64()
        _check(lib().ref_decode_many(self.h, C.c_int32(len(prompts)), _p(offsets), _p(flat), _p(steps),
                                     C.c_int32(n_threads), _p(last), C.byref(processed), _p(secs)))
        if seconds:
            return last, processed.value, secs
        return last, processed.value


class Runtime:
    """NeedleRuntime restated (runtime.ts:108-878)."""

    def __init__(self, model: Model, kv_mode: int = 0, collect_confidence: bool = False):
        self.model = model
        h = C.c_void_p()
        _check(lib().ref_runtime_new(model.h, C.c_int32(kv_mode), C.c_int32(int(collect_confidence)),
                                     C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            lib().ref_runtime_free(self.h)
            self.h = None

    __del__ = close

    def reset(self, maximum_length, sink_length=0):
        _check(lib().ref_runtime_reset(self.h, C.c_int32(maximum_length), C.c_int32(sink_length)))

    @property
    def position(self):
        return lib().ref_runtime_position(self.h)

    @property
    def kv_allocation(self):
        return lib().ref_runtime_kv_allocation(self.h)

    def step(self, token, want_logits=True):
        logits = np.zeros(self.model.vocab, dtype=np.float32) if want_logits else None
        _check(lib().ref_runtime_step(self.h, C.c_int32(token), _p(logits)))
        return logits

    def step_selected(self, token, allowed=None):
        a = None if allowed is None else np.ascontiguousarray(allowed, dtype=np.uint32)
        i, lp = C.c_int32(), C.c_double()
        _check(lib().ref_runtime_step_selected(self.h, C.c_int32(token), _p(a),
                                               C.c_int32(0 if a is None else a.size), C.byref(i), C.byref(lp)))
        return i.value, lp.value

    def read_kv(self, layer):
        alloc = self.kv_allocation
        hk, hd = self.model.kv_heads, self.model.head_dim
        kc = np.zeros((hk, alloc, hd), dtype=np.int8)
        vc = np.zeros((hk, alloc, hd), dtype=np.int8)
        ks = np.zeros((hk, alloc), dtype=np.float32)
        vs = np.zeros((hk, alloc), dtype=np.float32)
        _check(lib().ref_runtime_read_kv(self.h, C.c_int32(layer), _p(kc), _p(vc), _p(ks), _p(vs)))
        return kc, vc, ks, vs

    def read_kv_f32(self, layer):
        alloc = self.kv_allocation
        hk, hd = self.model.kv_heads, self.model.head_dim
        k = np.zeros((hk, alloc, hd), dtype=np.float32)
        v = np.zeros((hk, alloc, hd), dtype=np.float32)
        _check(lib().ref_runtime_read_kv_f32(self.h, C.c_int32(layer), _p(k), _p(v)))
        return k, v

    def read_lanes(self):
        out = np.zeros(self.model.lanes * self.model.dim, dtype=np.float32)
        _check(lib().ref_runtime_read_lanes(self.h, _p(out)))
        return out

    def confidence(self):
        v = C.c_double()
        _check(lib().ref_runtime_confidence(self.h, C.byref(v)))
        return v.value


def attention_int8(q, key_codes, key_scales, value_codes, value_scales, heads=8, kv_heads=4, head_dim=64):
    """Decode attention with kvWindow = 0 semantics over `count` cached positions."""
    count = key_codes.shape[1]
    q = np.ascontiguousarray(q, dtype=np.float32)
    kc = np.ascontiguousarray(key_codes, dtype=np.int8)
    vc = np.ascontiguousarray(value_codes, dtype=np.int8)
    ks = np.ascontiguousarray(key_scales, dtype=np.float32)
    vs = np.ascontiguousarray(value_scales, dtype=np.float32)
    out = np.zeros(heads * head_dim, dtype=np.float32)
    _check(lib().ref_attention_int8(C.c_int32(heads), C.c_int32(kv_heads), C.c_int32(head_dim), C.c_int32(count),
                                    _p(q), _p(kc), _p(ks), _p(vc), _p(vs), _p(out)))
    return out


def quantize_kv_head(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.size, dtype=np.int8)
    s = C.c_float()
    _check(lib().ref_quantize_kv_head(_p(x), C.c_int32(x.size), _p(codes), C.byref(s)))
    return codes, s.value


class Sched:
    """Host continuous batching (ref_sched_*): the CPU counterpart of the device scheduler."""

    def __init__(self, model: Model, n_slots, prompts, gen_steps, n_threads):
        self.model = model
        offsets = np.zeros(len(prompts) + 1, dtype=np.int32)
        offsets[1:] = np.cumsum([len(p) for p in prompts])
        flat = np.ascontiguousarray(np.concatenate(prompts) if len(prompts) else np.zeros(0), dtype=np.int32)
        steps = np.ascontiguousarray(gen_steps, dtype=np.int32)
        self.n_seqs = len(prompts)
        h = C.c_void_p()
        _check(lib().ref_sched_new(model.h, C.c_int32(n_slots), _p(offsets), _p(flat), _p(steps),
                                   C.c_int32(len(prompts)), C.c_int32(n_threads), C.byref(h)))
        self.h = h

    def step(self, steps=1):
        _check(lib().ref_sched_step(self.h, C.c_int32(steps)))

    def status(self):
        p, g, f = C.c_int64(), C.c_int64(), C.c_int32()
        last = np.zeros(max(self.n_seqs, 1), dtype=np.int32)
        _check(lib().ref_sched_status(self.h, C.byref(p), C.byref(g), C.byref(f), _p(last)))
        return p.value, g.value, f.value, last[:self.n_seqs]

    def close(self):
        if getattr(self, "h", None):
            lib().ref_sched_free(self.h)
            self.h = None

    __del__ = close
