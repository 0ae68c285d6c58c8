"""Host-side constrained tool-call grammar (include/needle_grammar.h) and the constrained loop.

`ToolCallGrammar` / `JsonSchemaGrammar` mirror packages/needle.js/src/tools/grammar.ts (same
constructor arguments, `feed`, `clone`, `complete`, `value` / `calls`); `Vocabulary` holds the
pieces the loop may emit (tokenizer.pieceBytes of the Normal and Byte pieces,
packages/needle.js/src/model/tokenizer.ts:257-282); `allowed` / `allowed_batch` return the ids the
grammar accepts next, ascending, as the loop's scan over the vocabulary does
(packages/needle.js/src/tools/agent.ts:165-176).
"""
from __future__ import annotations

import ctypes as C
import json
from typing import List, Optional, Sequence

import numpy as np

from .native import check, lib

MAX_OUTPUT_BYTES = 65_536  # agent.ts:171
META_SPACE = "▁"

# TokenPieceType (tokenizer.ts:21-27)
NORMAL, UNKNOWN, CONTROL, USER_DEFINED, BYTE = 0, 1, 2, 3, 4


class _Grammar:
    def __init__(self, handle: C.c_void_p):
        self._h = handle

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().needle_grammar_free(h)
            self._h = None

    @property
    def handle(self) -> C.c_void_p:
        return self._h

    def clone(self):
        out = C.c_void_p()
        check(lib().needle_grammar_clone(self._h, C.byref(out)))
        c = object.__new__(type(self))
        _Grammar.__init__(c, out)
        return c

    def feed(self, data: bytes) -> bool:
        ok = C.c_int32()
        check(lib().needle_grammar_feed(self._h, bytes(data), len(data), C.byref(ok)))
        return bool(ok.value)

    @property
    def complete(self) -> bool:
        v = C.c_int32()
        check(lib().needle_grammar_complete(self._h, C.byref(v)))
        return bool(v.value)

    def _result(self):
        n = C.c_int32()
        check(lib().needle_grammar_result(self._h, None, 0, C.byref(n)))
        buf = C.create_string_buffer(n.value + 1)
        check(lib().needle_grammar_result(self._h, buf, n.value + 1, C.byref(n)))
        text = buf.raw[:n.value].decode("utf-8", "surrogatepass")
        return json.loads(text) if text else None


class JsonSchemaGrammar(_Grammar):
    """grammar.ts:258: a byte grammar of one compact JSON value conforming to `schema`."""

    def __init__(self, schema):
        out = C.c_void_p()
        check(lib().needle_grammar_schema(json.dumps(schema).encode(), C.byref(out)))
        super().__init__(out)

    @property
    def value(self):
        return self._result()


class ToolCallGrammar(_Grammar):
    """grammar.ts:655: `[{"name":...,"arguments":...}, ...]` over normalised tools."""

    def __init__(self, tools: Sequence[dict], maximum_calls: int = 4):
        out = C.c_void_p()
        check(lib().needle_grammar_tools(json.dumps(list(tools)).encode(), int(maximum_calls), C.byref(out)))
        super().__init__(out)

    @property
    def calls(self):
        return self._result() or []


def piece_bytes(piece: str, kind: int) -> bytes:
    """tokenizer.pieceBytes (tokenizer.ts:257-282)."""
    if kind in (CONTROL, UNKNOWN):
        return b""
    if kind == BYTE:
        if len(piece) == 6 and piece.startswith("<0x") and piece.endswith(">"):
            try:
                return bytes([int(piece[3:5], 16)])
            except ValueError:
                return b""
        return b""
    return piece.replace(META_SPACE, " ").encode("utf-8")


class Vocabulary:
    """The pieces the constrained loop may emit: Normal and Byte pieces with non-empty bytes
    (agent.ts:168-170); every other id is never allowed."""

    def __init__(self, pieces: Sequence[str], types: Sequence[int]):
        chunks, offsets = [], [0]
        for p, t in zip(pieces, types):
            b = piece_bytes(p, t) if t in (NORMAL, BYTE) else b""
            chunks.append(b)
            offsets.append(offsets[-1] + len(b))
        self.piece = chunks
        blob = b"".join(chunks)
        off = (C.c_int32 * len(offsets))(*offsets)
        out = C.c_void_p()
        check(lib().needle_vocab_open(blob, off, len(chunks), C.byref(out)))
        self._h = out
        self.size = len(chunks)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().needle_vocab_free(h)
            self._h = None


def allowed(grammar: _Grammar, vocab: Vocabulary, output_bytes: int = 0) -> np.ndarray:
    ids = np.empty(vocab.size, dtype=np.uint32)
    n = C.c_int32()
    check(lib().needle_grammar_allowed(grammar.handle, vocab._h, int(output_bytes),
                                       ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size, C.byref(n)))
    return ids[:n.value].copy()


def allowed_batch(grammars: Sequence[Optional[_Grammar]], output_bytes: Sequence[int], vocab: Vocabulary,
                  threads: int = 8) -> List[np.ndarray]:
    n = len(grammars)
    if n == 0:
        return []
    hs = (C.c_void_p * n)(*[g.handle if g is not None else None for g in grammars])
    ob = (C.c_int64 * n)(*[int(v) for v in output_bytes])
    ids = np.empty((n, vocab.size), dtype=np.uint32)
    counts = np.empty(n, dtype=np.int32)
    check(lib().needle_grammar_allowed_batch(hs, ob, n, vocab._h, int(threads),
                                             ids.ctypes.data_as(C.POINTER(C.c_uint32)), vocab.size,
                                             counts.ctypes.data_as(C.POINTER(C.c_int32))))
    return [ids[k, :counts[k]].copy() for k in range(n)]


class MaskCache:
    """Allowed-token masks per grammar state (needle_mask_cache_*, include/needle_grammar.h) for the
    clones of one template grammar: `lookup` gives each grammar's table slot and allowed count,
    scanning only states not seen before; `table` is the [capacity][words] host table the slots
    index (the masks a device pool copies, CudaEngine.masks_put)."""

    def __init__(self, template: _Grammar, vocab: Vocabulary, capacity: int = 4096):
        out = C.c_void_p()
        check(lib().needle_mask_cache_open(template.handle, vocab._h, int(capacity), C.byref(out)))
        self._h = out
        self._vocab = vocab  # the cache reads it: keep it alive as long as the cache
        self.capacity = int(capacity)
        p = C.POINTER(C.c_uint32)()
        words = C.c_int32()
        check(lib().needle_mask_cache_table(self._h, C.byref(p), C.byref(words)))
        self.words = words.value
        self.table = np.ctypeslib.as_array(p, shape=(self.capacity, self.words))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self.table = None
            lib().needle_mask_cache_free(h)
            self._h = None

    def lookup(self, grammars: Sequence[Optional[_Grammar]], output_bytes: Sequence[int], threads: int = 8):
        """(slots, counts, filled): per grammar its table slot (-1 for None) and allowed count, and the
        slots this call (re)filled."""
        n = len(grammars)
        slots = np.empty(max(n, 1), dtype=np.int32)
        counts = np.empty(max(n, 1), dtype=np.int32)
        filled = np.empty(max(n, 1), dtype=np.int32)
        n_filled = C.c_int32()
        hs = (C.c_void_p * max(n, 1))(*[g.handle if g is not None else None for g in grammars])
        ob = (C.c_int64 * max(n, 1))(*[int(v) for v in output_bytes])
        check(lib().needle_mask_cache_lookup(self._h, hs, ob, n, int(threads), slots.ctypes.data,
                                             counts.ctypes.data, filled.ctypes.data, C.byref(n_filled)))
        return slots[:n], counts[:n], filled[:n_filled.value].copy()

    def ids(self, slot: int) -> np.ndarray:
        """The ascending ids of a slot's mask."""
        bits = np.unpackbits(self.table[slot].view(np.uint8), bitorder="little")
        return np.flatnonzero(bits[:self._vocab.size]).astype(np.uint32)

    @property
    def stats(self):
        h, m, e = C.c_int64(), C.c_int64(), C.c_int64()
        check(lib().needle_mask_cache_stats(self._h, C.byref(h), C.byref(m), C.byref(e)))
        return {"hits": h.value, "misses": m.value, "evictions": e.value}
