"""Host-side mirror of the needle.js backend interface over libneedle_cuda.so.

needle.js is TypeScript and its runtime cannot run in this environment, so the adapter it would
use (a bun:ffi `CudaBackend` over the same C-ABI) is mirrored here in Python with the same names,
argument meanings and error behaviour:

* `CudaBackend`         -- InferenceBackend (packages/needle.js/src/backends/backend.ts:83-110):
                            matvec / matvec_batch / row / create_resident_session / dispose.
                            CQ matrices are addressed by archive record index
                            (CqMatrix.record.index, cact.ts:61-75).
* `NeedleRuntime`       -- NeedleRuntime (packages/needle.js/src/model/runtime.ts:108-583):
                            reset / prefill / prefill_selected / step / step_selected over one
                            sequence slot of the engine, token loop entirely on the GPU.
* `CudaEngine`          -- the batched engine itself: many slots stepped together (the ragged
                            batch API that the single-sequence reference has no counterpart for).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import native
from .native import NeedleError, check, lib, ptr


@dataclass
class StepRequest:
    """One slot's work in a batched step."""
    seq: int
    token: int = native.TOKEN_PENDING
    select: bool = False
    allowed: Optional[np.ndarray] = None  # None: unmasked argmax
    mask_slot: Optional[int] = None       # a slot of the device mask pool instead of `allowed`


class CudaEngine:
    """One engine context on one GPU (needle_cuda_open .. needle_cuda_close)."""

    def __init__(self, archive: bytes, device: int = 0, max_seqs: int = 1, max_len: int = 2048,
                 max_sink: int = 160, kv_cache: str = "int8", numerics: str = "exact", micro_batches: int = 0,
                 sched_chunk: int = 0, sched_items: int = 0):
        if kv_cache not in ("int8", "float32"):
            raise NeedleError("BACKEND_UNAVAILABLE", f"unknown kvCache {kv_cache!r}")
        modes = {"exact": native.NUMERICS_EXACT, "fast": native.NUMERICS_FAST,
                 "fast_attention": native.NUMERICS_FAST_ATTENTION}
        if numerics not in modes:
            raise NeedleError("BACKEND_UNAVAILABLE", f"unknown numerics {numerics!r}")
        self._archive = np.frombuffer(archive, dtype=np.uint8)
        opts = native.default_opts(device=device, max_seqs=max_seqs, max_len=max_len, max_sink=max_sink,
                                   kv_mode=native.KV_FLOAT32 if kv_cache == "float32" else native.KV_INT8,
                                   numerics=modes[numerics],
                                   micro_batches=micro_batches, sched_chunk=sched_chunk,
                                   sched_items=sched_items)
        self.numerics = numerics
        self.kv_cache = kv_cache
        h = C.c_void_p()
        check(lib().needle_cuda_open(ptr(self._archive), self._archive.size, C.byref(opts), C.byref(h)))
        self.h = h
        g = native.Geometry()
        check(lib().needle_cuda_geometry(self.h, C.byref(g)))
        self.geometry = g
        self.vocab = g.vocabulary_size
        self.layers = g.layers
        self.max_seqs = max_seqs
        self.kv_window = g.kv_window

    def close(self):
        if getattr(self, "h", None):
            check(lib().needle_cuda_close(self.h))
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def stream(self) -> int:
        return lib().needle_cuda_stream(self.h) or 0

    def reset(self, seq: int, maximum_length: int, sink_length: int = 0, collect_confidence: bool = False):
        check(lib().needle_cuda_seq_reset_ex(self.h, seq, maximum_length, sink_length, int(collect_confidence)))

    def confidence(self, seq: int) -> float:
        v = C.c_double()
        check(lib().needle_cuda_confidence(self.h, seq, C.byref(v)))
        return v.value

    def read_kv_f32(self, seq: int, layer: int):
        alloc = C.c_int32()
        check(lib().needle_cuda_read_kv_f32(self.h, seq, layer, None, None, C.byref(alloc)))
        hk, hd = self.geometry.kv_heads, self.geometry.head_dimension
        k = np.zeros((hk, alloc.value, hd), dtype=np.float32)
        v = np.zeros((hk, alloc.value, hd), dtype=np.float32)
        check(lib().needle_cuda_read_kv_f32(self.h, seq, layer, ptr(k), ptr(v), None))
        return k, v

    def position(self, seq: int) -> int:
        p = C.c_int32()
        check(lib().needle_cuda_seq_position(self.h, seq, C.byref(p)))
        return p.value

    @staticmethod
    def _items(requests: Sequence[StepRequest]):
        """The requests as a needle_step_item array (int32 seq, token, select, allowed_count,
        uint32 allowed_offset; filled column by column) and their allowed ids, concatenated."""
        n = len(requests)
        items = np.zeros((max(n, 1), 5), dtype=np.int32)
        if n:
            items[:n, 0] = [r.seq for r in requests]
            items[:n, 1] = [r.token for r in requests]
            masked = [r.select and r.allowed is not None and r.mask_slot is None for r in requests]
            pooled = [r.select and r.mask_slot is not None for r in requests]
            items[:n, 2] = [1 if r.select else 0 for r in requests]
            counts = np.array([r.allowed.size if m else -1 for r, m in zip(requests, masked)], dtype=np.int64)
            sizes = np.maximum(counts, 0)
            offsets = np.cumsum(sizes) - sizes
            for i, p in enumerate(pooled):
                if p:
                    counts[i], offsets[i] = native.ALLOWED_MASK, requests[i].mask_slot
            items[:n, 3] = counts
            items[:n, 4] = offsets.astype(np.uint32).view(np.int32)
        parts = [np.asarray(r.allowed, dtype=np.uint32) for r, m in zip(requests, masked) if m] if n else []
        allowed = np.ascontiguousarray(np.concatenate(parts)) if parts else None
        return items, allowed

    def step(self, requests: Sequence[StepRequest], want_logits: bool = False):
        """One batched step; returns (selected list of (id, logprob) or None per request, logits)."""
        n = len(requests)
        items, allowed = self._items(requests)
        sel = (native.Selected * max(n, 1))()
        logits = np.zeros((n, self.vocab), dtype=np.float32) if want_logits else None
        check(lib().needle_cuda_step(self.h, ptr(items), n, ptr(allowed),
                                     0 if allowed is None else allowed.size, C.cast(sel, C.c_void_p),
                                     ptr(logits)))
        out = [(sel[i].id, sel[i].log_probability) if r.select else None for i, r in enumerate(requests)]
        return out, logits

    def step_begin(self, requests: Sequence[StepRequest], items: Optional[np.ndarray] = None):
        """First half of a step (needle_cuda_step_begin): the layers are enqueued and this returns at
        once; the requests' allowed lists are not read.  step_end must follow before any other call.
        `items`: the requests already packed by `_items` (e.g. while the previous step ran)."""
        if items is None:
            items, _ = self._items(requests)
        check(lib().needle_cuda_step_begin(self.h, ptr(items), len(requests)))

    def step_end(self, requests: Sequence[StepRequest]):
        """Second half: the same requests (a select may be cleared), now with their allowed lists;
        returns the selections as step does."""
        n = len(requests)
        items, allowed = self._items(requests)
        sel = (native.Selected * max(n, 1))()
        check(lib().needle_cuda_step_end(self.h, ptr(items), n, ptr(allowed),
                                         0 if allowed is None else allowed.size, C.cast(sel, C.c_void_p)))
        return [(sel[i].id, sel[i].log_probability) if r.select else None for i, r in enumerate(requests)]

    def mask_pool(self, capacity: int):
        """(Re)allocates the device mask pool (needle_cuda_mask_pool): `capacity` empty slots."""
        check(lib().needle_cuda_mask_pool(self.h, int(capacity)))

    def masks_put(self, slots, table: np.ndarray):
        """Copies the listed slots' masks from `table` ([capacity][words] uint32, indexed by slot) into
        the device pool (needle_cuda_masks_put); allowed between step_begin and step_end."""
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        if slots.size == 0:
            return
        table = np.ascontiguousarray(table, dtype=np.uint32)
        check(lib().needle_cuda_masks_put(self.h, ptr(slots), slots.size, ptr(table)))

    def prefill(self, seq: int, ids, want_logits: bool = True):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        logits = np.zeros(self.vocab, dtype=np.float32) if want_logits else None
        check(lib().needle_cuda_prefill(self.h, seq, ptr(ids), ids.size, ptr(logits)))
        return logits

    def read_kv(self, seq: int, layer: int):
        g = self.geometry
        alloc = C.c_int32()
        check(lib().needle_cuda_read_kv(self.h, seq, layer, None, None, None, None, C.byref(alloc)))
        a = alloc.value
        kc = np.zeros((g.kv_heads, a, g.head_dimension), dtype=np.int8)
        vc = np.zeros_like(kc)
        ks = np.zeros((g.kv_heads, a), dtype=np.float32)
        vs = np.zeros_like(ks)
        check(lib().needle_cuda_read_kv(self.h, seq, layer, ptr(kc), ptr(vc), ptr(ks), ptr(vs), C.byref(alloc)))
        return kc, vc, ks, vs

    def read_lanes(self, seq: int):
        out = np.zeros(self.geometry.mhc_lanes * self.geometry.model_dimension, dtype=np.float32)
        check(lib().needle_cuda_read_lanes(self.h, seq, ptr(out)))
        return out

    def matvec(self, tensor: int, x, row_start: int = 0, row_count: Optional[int] = None):
        x = np.ascontiguousarray(x, dtype=np.float32)
        batch = 1 if x.ndim == 1 else x.shape[0]
        if row_count is None:
            raise ValueError("row_count is required")
        y = np.zeros((batch, row_count), dtype=np.float32)
        check(lib().needle_cuda_matvec(self.h, tensor, row_start, row_count, ptr(x), batch, ptr(y)))
        return y[0] if x.ndim == 1 else y

    def row(self, tensor: int, row: int, width: int):
        out = np.zeros(width, dtype=np.float32)
        check(lib().needle_cuda_row(self.h, tensor, row, ptr(out)))
        return out

    # device-resident continuous batching -------------------------------------------------
    def sched_load(self, n_slots: int, prompts, gen_steps):
        offsets = np.zeros(len(prompts) + 1, dtype=np.int32)
        offsets[1:] = np.cumsum([len(p) for p in prompts])
        flat = np.ascontiguousarray(np.concatenate(prompts) if prompts else np.zeros(0), dtype=np.int32)
        steps = np.ascontiguousarray(gen_steps, dtype=np.int32)
        check(lib().needle_cuda_sched_load(self.h, n_slots, ptr(offsets), ptr(flat), ptr(steps), len(prompts)))
        self._n_seqs = len(prompts)

    def sched_step(self, steps: int = 1):
        check(lib().needle_cuda_sched_step(self.h, steps))

    def sched_status(self):
        """(tokens processed, tokens generated, sequences finished, last ids per sequence)."""
        tokens, generated, finished = C.c_int64(), C.c_int64(), C.c_int32()
        last = np.zeros(max(self._n_seqs, 1), dtype=np.int32)
        check(lib().needle_cuda_sched_status(self.h, C.byref(tokens), C.byref(generated), C.byref(finished),
                                             ptr(last)))
        return tokens.value, generated.value, finished.value, last[:self._n_seqs]

    def sched_ids(self):
        """Every selected id of the loaded queue, split per sequence (-1 where not generated yet)."""
        total = C.c_size_t()
        check(lib().needle_cuda_sched_ids(self.h, None, 0, C.byref(total)))
        flat = np.zeros(max(total.value, 1), dtype=np.int32)
        check(lib().needle_cuda_sched_ids(self.h, ptr(flat), total.value, None))
        return flat[:total.value]

    def sched_slot(self, slot: int):
        """(sequence id, position, busy) of a scheduler slot."""
        sid, pos, busy = C.c_int32(), C.c_int32(), C.c_int32()
        check(lib().needle_cuda_sched_slot(self.h, slot, C.byref(sid), C.byref(pos), C.byref(busy)))
        return sid.value, pos.value, bool(busy.value)

    def damaged_guards(self) -> int:
        """Guards after the context's device buffers that no longer hold their pattern (0: no
        kernel wrote past those buffers; needle_cuda_check_guards)."""
        n = C.c_int32()
        check(lib().needle_cuda_check_guards(self.h, C.byref(n)))
        return n.value

    def kernel_launches(self) -> int:
        n = C.c_int64()
        check(lib().needle_cuda_kernel_launches(self.h, C.byref(n)))
        return n.value

    # per-kernel-class event timing ----------------------------------------------------------
    def profile(self, enable: bool):
        check(lib().needle_cuda_profile(self.h, 1 if enable else 0))

    def profile_read(self):
        n = 16
        names = (C.c_char_p * n)()
        ms = (C.c_double * n)()
        launches = (C.c_int64 * n)()
        count = C.c_int32()
        check(lib().needle_cuda_profile_read(self.h, n, names, ms, launches, C.byref(count)))
        return {names[i].decode(): (ms[i], launches[i]) for i in range(count.value)}


class CudaBackend:
    """InferenceBackend over one engine context (backend.ts:83-110)."""

    kind = "cuda"
    name = "CUDA sm_100a (B200)"

    def __init__(self, archive: bytes, device: int = 0, max_seqs: int = 1, max_len: int = 2048,
                 max_sink: int = 160, kv_cache: str = "int8"):
        self.weights = archive
        self.engine = CudaEngine(archive, device=device, max_seqs=max_seqs, max_len=max_len, max_sink=max_sink,
                                 kv_cache=kv_cache)
        self._free = list(range(max_seqs))

    def matvec(self, tensor: int, input, range: Optional[dict] = None):
        """matvec(matrix, input, range?) with the matrix given by its archive record index."""
        rows = self._rows(tensor)
        start = (range or {}).get("rowStart", 0)
        count = (range or {}).get("rowCount", rows - start)
        return self.engine.matvec(tensor, input, start, count)

    def matvec_batch(self, requests):
        """matvecBatch(requests): one (tensor, input, range) per request."""
        return [self.matvec(t, x, r) for (t, x, r) in requests]

    def row(self, tensor: int, row: int):
        return self.engine.row(tensor, row, self._width(tensor))

    def create_resident_session(self) -> "CudaResidentSession":
        if not self._free:
            raise NeedleError("BACKEND_UNAVAILABLE", "all sequence slots of the CUDA backend are in use")
        return CudaResidentSession(self, self._free.pop(0))

    def dispose(self):
        self.engine.close()

    def _record(self, tensor):
        import struct
        a = self.weights
        n, cbl = struct.unpack_from("<II", a, 4)
        off = 120 + cbl * 4 + tensor * 44
        dtype, rank = a[off], a[off + 1]
        dims = struct.unpack_from("<4I", a, off + 4)
        return dtype, dims[:rank]

    def _rows(self, tensor):
        return self._record(tensor)[1][0]

    def _width(self, tensor):
        return self._record(tensor)[1][1]


class CudaResidentSession:
    """ResidentExecutionSession (backend.ts:66-80) bound to one engine slot, implementing the whole-
    token calls NeedleRuntime.step makes (runtime.ts:314-372) with the arguments it passes them.
    reset() returns True for supported options and raises NeedleError(BACKEND_UNAVAILABLE) otherwise:
    unlike the reference's optional sessions, this backend never hands the step back to a CPU loop.
    prepareResidentEngrams and beginResidentToken keep their arguments; forwardResidentToken runs the
    token on the GPU (needle_cuda_resident_forward); finishResidentToken / selectResidentToken end it."""

    def __init__(self, backend: CudaBackend, slot: int):
        self.backend = backend
        self.engine = backend.engine
        self.slot = slot
        self._lanes = None
        self._engrams = None

    def reset(self, options: dict) -> bool:
        """reset({maximumLength, sinkLength, kvCache, collectConfidence})."""
        kv_cache = options.get("kvCache", "int8")
        if kv_cache != self.engine.kv_cache:
            raise NeedleError("BACKEND_UNAVAILABLE",
                              f"this CUDA backend context holds a {self.engine.kv_cache} KV cache")
        self.engine.reset(self.slot, options["maximumLength"], options.get("sinkLength", 0),
                          bool(options.get("collectConfidence", False)))
        self._lanes = self._engrams = None
        return True

    def forward(self, request):
        raise NeedleError("BACKEND_UNAVAILABLE", "the CUDA session runs whole tokens (forwardResidentToken)")

    def prepare_resident_engrams(self, request: dict) -> bool:
        """prepareResidentEngrams({indices, valid, position})."""
        self._engrams = (np.ascontiguousarray(request["indices"], dtype=np.uint32),
                         np.ascontiguousarray(request["valid"], dtype=np.uint32), int(request["position"]))
        return True

    def begin_resident_token(self, lanes) -> bool:
        """beginResidentToken(x): the token's lanes (mhcLanes copies of the scaled embedding row)."""
        self._lanes = np.ascontiguousarray(lanes, dtype=np.float32)
        return True

    def forward_resident_token(self, request: dict) -> None:
        """forwardResidentToken({position, engramKeys, engramValues}): every layer and the vocabulary
        projection, enqueued on the GPU."""
        if self._lanes is None:
            raise NeedleError("BACKEND_UNAVAILABLE", "beginResidentToken must precede forwardResidentToken")
        idx, valid, epos = self._engrams if self._engrams is not None else (None, None, int(request["position"]))
        lanes, self._lanes, self._engrams = self._lanes, None, None
        check(lib().needle_cuda_resident_forward(self.engine.h, self.slot, int(request["position"]), ptr(lanes),
                                                 ptr(idx), ptr(valid), 0 if idx is None else idx.size, epos))

    def finish_resident_token(self, want_logits: bool):
        """finishResidentToken(wantLogits): the logits (or None) and the slot advanced."""
        logits = np.zeros(self.engine.vocab, dtype=np.float32) if want_logits else None
        check(lib().needle_cuda_resident_finish(self.engine.h, self.slot, ptr(logits)))
        return logits

    def finish_resident_token_for_selection(self) -> None:
        """finishResidentTokenForSelection(): nothing to do, forward already projected the vocabulary."""

    def select_resident_token(self, allowed=None):
        """selectResidentToken(allowedTokenIds?) -> (id, logProbability)."""
        a = None if allowed is None else np.ascontiguousarray(allowed, dtype=np.uint32)
        sel = native.Selected()
        check(lib().needle_cuda_resident_select(self.engine.h, self.slot, ptr(a), -1 if a is None else a.size,
                                                C.byref(sel)))
        return sel.id, sel.log_probability

    def resident_layers_enabled(self) -> bool:
        return True

    def resident_confidence(self) -> float:
        return self.engine.confidence(self.slot)

    def read_resident_lanes(self):
        return self.engine.read_lanes(self.slot)

    def dispose(self):
        self.backend._free.append(self.slot)


ENGRAM_SEED = 0x9E3779B9   # runtime.ts:22
ENGRAM_PRIME = 0x01000193  # runtime.ts:23
EMBEDDING = 0              # canonical tensor order: the embedding is record 0 (cact.ts:403-536)


def _imul(a: int, b: int) -> int:
    return (a * b) & 0xFFFFFFFF


class NeedleRuntime:
    """NeedleRuntime (runtime.ts:108-583) restated over a resident session: the host side of step()
    is the reference's -- embedding row through backend.row, the scaled lanes, #engramLookup on the
    token history -- and every token goes through the session calls in the reference's order
    (prepareResidentEngrams, beginResidentToken, forwardResidentToken, then finishResidentToken or
    finishResidentTokenForSelection + selectResidentToken).  prefill runs step once per token, as
    runtime.ts:227-243 does; `chunked_prefill` (an extension) sends a prompt through the engine's
    batched prefill (needle_cuda_prefill) instead, with the same result."""

    def __init__(self, backend: CudaBackend, kv_cache: str = "int8", collect_confidence: bool = True):
        self.backend = backend
        self.options = {"kvCache": kv_cache, "collectConfidence": collect_confidence}
        self.session = backend.create_resident_session()
        self.engine = backend.engine
        g = self.engine.geometry
        self.dimension, self.lanes = g.model_dimension, g.mhc_lanes
        self.vocab = g.vocabulary_size
        self.orders = list(g.engram_orders[:g.engram_order_count])
        self.tables, self.slots = g.engram_tables, g.engram_slots
        self.sites = g.engram_site_count
        self._max = 0
        self._position = 0
        self._history: list[int] = []
        self._engram_position = 0
        self._selection_request = None
        self._selection_active = False
        self._selection_result = None

    @property
    def position(self) -> int:
        return self._position

    @property
    def maximum_length(self) -> int:
        return self._max

    def reset(self, maximum_length: int, sink_length: int = 0):
        if not (isinstance(maximum_length, int) and 0 < maximum_length <= self.engine.geometry.maximum_sequence_length):
            raise NeedleError("CONTEXT_OVERFLOW", f"Runtime length {maximum_length} is outside model limit "
                                                  f"{self.engine.geometry.maximum_sequence_length}")
        self._max = maximum_length
        sink = min(max(sink_length, 0), maximum_length)
        self._position = 0
        self._history = []
        self._engram_position = 0
        self._selection_active = False
        self.session.reset({"maximumLength": maximum_length, "sinkLength": sink, "kvCache": self.options["kvCache"],
                            "collectConfidence": self.options["collectConfidence"] is not False})

    def confidence(self) -> float:
        """NeedleRuntime.confidence (runtime.ts:634-645): NaN unless collecting."""
        return self.session.resident_confidence()

    def prefill(self, tokens, chunked_prefill: bool = False) -> np.ndarray:
        if len(tokens) == 0:
            raise NeedleError("INVALID_CACT", "Cannot prefill an empty token sequence")
        if self._max < len(tokens):
            raise NeedleError("CONTEXT_OVERFLOW", f"Prompt has {len(tokens)} tokens but runtime holds {self._max}")
        if chunked_prefill:
            logits = self.engine.prefill(self.slot_index, tokens, want_logits=True)
            self._history.extend(int(t) for t in tokens)
            self._position += len(tokens)
            self._engram_position += len(tokens)
            return logits
        logits = None
        for i, t in enumerate(tokens):
            logits = self.step(int(t), want_logits=i == len(tokens) - 1)
        return logits

    def prefill_selected(self, tokens, allowed=None):
        if len(tokens) == 0:
            raise NeedleError("INVALID_CACT", "Cannot prefill an empty token sequence")
        for t in tokens[:-1]:
            self.step(int(t), want_logits=False)
        return self.step_selected(int(tokens[-1]), allowed)

    def step_selected(self, token: int, allowed=None):
        if self._selection_active:
            raise NeedleError("BACKEND_UNAVAILABLE", "Selection is already active")
        self._selection_active = True
        self._selection_request = None if allowed is None else np.asarray(allowed, dtype=np.uint32)
        self._selection_result = None
        try:
            self.step(token)
            if self._selection_result is None:
                raise NeedleError("BACKEND_UNAVAILABLE", "Token selection did not produce a result")
            return self._selection_result
        finally:
            self._selection_active = False
            self._selection_request = None
            self._selection_result = None

    def _engram_lookup(self):
        """#engramLookup (runtime.ts:788-818): per order and head an FNV-style hash of the last
        `order` tokens of the history (missing tokens hash as 0), valid when the history reaches back
        that far."""
        per_order = self.tables // len(self.orders)
        indices = np.zeros(self.tables, dtype=np.uint32)
        valid = np.zeros(self.tables, dtype=np.uint32)
        table = 0
        for oi, order in enumerate(self.orders):
            for head in range(per_order):
                h = _imul(ENGRAM_SEED, oi * per_order + head + 1)
                ok = True
                for off in range(order):
                    hi = len(self._history) - 1 - off
                    tok = self._history[hi] if hi >= 0 else 0
                    h = _imul((h ^ tok) & 0xFFFFFFFF, ENGRAM_PRIME)
                    if off == order - 1:
                        ok = hi >= 0
                h = (h ^ (h >> 15)) & 0xFFFFFFFF
                indices[table] = h % self.slots
                valid[table] = 1 if ok else 0
                table += 1
        return indices, valid

    def step(self, token: int, want_logits: bool = True):
        if self._max <= 0:
            raise NeedleError("INVALID_CACT", "Call runtime.reset() before decoding")
        if self._position >= self._max:
            raise NeedleError("CONTEXT_OVERFLOW", f"Position {self._position} reached runtime limit {self._max}")
        if not (0 <= int(token) < self.vocab):
            raise NeedleError("INVALID_CACT", f"Token {token} is outside the vocabulary")
        position = self._position
        self._history.append(int(token))
        embedding = self.backend.row(EMBEDDING, int(token))
        scaled = (embedding.astype(np.float64) * np.sqrt(float(self.dimension))).astype(np.float32)
        x = np.tile(scaled, self.lanes)
        if self.sites > 0:
            indices, valid = self._engram_lookup()
            if self.session.prepare_resident_engrams({"indices": indices, "valid": valid,
                                                      "position": self._engram_position}):
                self._engram_position += 1
        self.session.begin_resident_token(x)
        self.session.forward_resident_token({"position": position, "engramKeys": [], "engramValues": []})
        logits = None
        if self._selection_active:
            self.session.finish_resident_token_for_selection()
        else:
            logits = self.session.finish_resident_token(want_logits is not False)
        self._position += 1
        if self._selection_active:
            self._selection_result = self.session.select_resident_token(self._selection_request)
            return None
        return logits if want_logits is not False else None

    @property
    def slot_index(self) -> int:
        return self.session.slot

    def dispose(self):
        self.session.dispose()
