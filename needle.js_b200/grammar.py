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
