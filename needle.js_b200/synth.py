"""Synthetic Needle 2 `.cact` archives: the build's own CQ quantizer and archive writer.

needle.js ships only readers for the `.cact` format (packages/needle.js/src/model/cact.ts:189-562);
its official archive is downloaded at run time and is not available offline.  This module writes
archives with the same layout (apps/website/src/content/docs/tutorials/cact-format.mdx):

* a 120-byte header, the 28-entry f32 codebook, 44-byte tensor records, 64-byte aligned blobs in
  the canonical tensor order (cact.ts:403-536);
* Cactus-Quant matrices quantised as the format tutorial describes (cact-format.mdx:195-205):
  rotate each 128-group with the normalised Walsh-Hadamard transform, store its L2 norm as fp16,
  and replace the unit-norm rotated values by their nearest codebook level;
* a RAW SentencePiece tokenizer blob in the layout read by tokenizer.ts:45-91.

Random numbers: one PCG64 stream per tensor, seeded with (seed, tensor index), and numpy's
ziggurat normal sampler.  The quantiser itself uses only IEEE-754 +, -, *, / and sqrt with a
fixed summation order, so the archive bytes are identical on every CPU running this image.

Codebook: the Lloyd-Max minimum-MSE quantiser levels of the standard normal distribution for 4, 8
and 16 levels (J. Max, "Quantizing for minimum distortion", IRE Trans. IT-6, 1960), divided by
sqrt(128) as the format requires (cact-format.mdx:78-86).  Ternary matrices use the analytic
levels {-1.2240064, 0, +1.2240064}/sqrt(group) of cq.ts:5-6.

Bit-width assignment (not stated by the reference; ~2.5 bits/weight overall like the official
13.7 MB archive): embedding CQ4; Q/K/V/gate CQ2; output projection CQ3; mHC phi CQ4; engram
tables CQ2; engram key/value projections ternary.  All four record widths are exercised.
"""
from __future__ import annotations

import dataclasses
import math
import struct

import numpy as np

CACT_TAG = 0x05E12A83
HEADER_BYTES = 120
RECORD_BYTES = 44
DT_F16, DT_F32, DT_CQ, DT_RAW = 1, 2, 3, 4
TERNARY_BITS = 5
TERNARY_CENTROID = 1.2240064

_LLOYD_MAX = {
    2: [0.4528, 1.5104],
    3: [0.2451, 0.7560, 1.3440, 2.1520],
    4: [0.1284, 0.3881, 0.6568, 0.9424, 1.2562, 1.6181, 2.0690, 2.7326],
}


def lloyd_max_codebook(group: int = 128) -> np.ndarray:
    """28 f32 levels: CQ2 (4) + CQ3 (8) + CQ4 (16), ascending, divided by sqrt(group)."""
    out = []
    for bits in (2, 3, 4):
        half = np.asarray(_LLOYD_MAX[bits], dtype=np.float64)
        levels = np.concatenate([-half[::-1], half]) / np.sqrt(float(group))
        out.append(levels)
    return np.concatenate(out).astype(np.float32)


# ------------------------------------------------------------------ deterministic RNG

_GAMMA = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def splitmix64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n outputs of splitmix64 whose state starts at a (seed, stream) dependent value."""
    base = (int(seed) * 0x2545F4914F6CDD1D + int(stream) * 0xD1B54A32D192ED03 + 0x632BE59BD9B4E019)
    base &= (1 << 64) - 1
    with np.errstate(over="ignore"):
        z = np.uint64(base) + (np.arange(1, n + 1, dtype=np.uint64) * _GAMMA)
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        z = z ^ (z >> np.uint64(31))
    return z


def normal(seed: int, n: int, stream: int = 0, std: float = 1.0) -> np.ndarray:
    """n N(0, std^2) doubles from numpy's PCG64 bit generator seeded with (seed, stream) and its
    ziggurat normal sampler.  The bit stream is platform independent; the sampler only consults
    libm's exp in its rare wedge test, so the draws are identical on every machine running the
    same numpy."""
    rng = np.random.Generator(np.random.PCG64([int(seed), int(stream)]))
    return rng.standard_normal(n) * std


def integers(seed: int, n: int, high: int, stream: int = 0) -> np.ndarray:
    """n uniform integers in [0, high) from PCG64 seeded with (seed, stream)."""
    rng = np.random.Generator(np.random.PCG64([int(seed), int(stream)]))
    return rng.integers(0, high, size=n, dtype=np.int64)


# ------------------------------------------------------------------ Cactus-Quant quantiser


def fwht_rows(values: np.ndarray) -> np.ndarray:
    """Unnormalised Walsh-Hadamard transform along the last axis (power-of-two length)."""
    v = np.array(values, dtype=np.float64, copy=True)
    n = v.shape[-1]
    h = 1
    while h < n:
        v = v.reshape(v.shape[:-1] + (n // (2 * h), 2, h))
        a = v[..., 0, :].copy()
        b = v[..., 1, :].copy()
        v[..., 0, :] = a + b
        v[..., 1, :] = a - b
        v = v.reshape(v.shape[:-3] + (n,))
        h *= 2
    return v


def pack_indices(indices: np.ndarray, bits: int) -> np.ndarray:
    """Little-endian bitstream per row: index k occupies bits [k*bits, (k+1)*bits)."""
    rows, cols = indices.shape
    if bits in (2, 4) and cols % (8 // bits) == 0:
        per = 8 // bits
        v = indices.astype(np.uint8).reshape(rows, cols // per, per)
        out = v[..., 0].copy()
        for k in range(1, per):
            out |= v[..., k] << np.uint8(k * bits)
        return out
    shifts = np.arange(bits, dtype=np.uint32)
    bitplane = ((indices.astype(np.uint32)[:, :, None] >> shifts) & 1).astype(np.uint8)
    flat = bitplane.reshape(rows, cols * bits)
    return np.packbits(flat, axis=1, bitorder="little")


def quantize_cq(weights: np.ndarray, bits: int, codebook: np.ndarray, group: int = 128):
    """Quantise a float64 [rows, input] matrix; returns (packed bytes, fp16 norms bytes)."""
    rows, inputs = weights.shape
    padded = -(-inputs // group) * group
    w = np.zeros((rows, padded), dtype=np.float64)
    w[:, :inputs] = weights
    groups = w.reshape(rows, padded // group, group)
    rotated = fwht_rows(groups) / np.sqrt(float(group))
    sq = rotated * rotated
    total = np.zeros(sq.shape[:-1], dtype=np.float64)
    for k in range(group):  # fixed summation order
        total = total + sq[..., k]
    norm = np.sqrt(total)
    unit = rotated / np.where(norm > 0, norm, 1.0)[..., None]
    if bits == TERNARY_BITS:
        c = TERNARY_CENTROID / np.sqrt(float(group))
        levels = np.array([-c, 0.0, c])
    else:
        start = {2: 0, 3: 4, 4: 12}[bits]
        levels = codebook[start:start + (1 << bits)].astype(np.float64)
    # Nearest level; a value exactly between two levels takes the lower one.
    midpoints = (levels[1:] + levels[:-1]) * 0.5
    idx = np.searchsorted(midpoints, unit.reshape(-1), side="left").reshape(rows, padded)
    if bits == TERNARY_BITS:
        # trit index 0 (-c), 1 (0), 2 (+c) -> crumbs 3, 0, 1 (packages/needle.js/tests/cq.test.ts:26-27)
        idx = np.where(idx == 0, 3, idx - 1)
        packed = pack_indices(idx, 2)
    else:
        packed = pack_indices(idx, bits)
    norms16 = norm.astype(np.float16).reshape(-1)
    return packed.reshape(-1).tobytes(), norms16.astype("<f2").tobytes()


# ------------------------------------------------------------------ tokenizer blob

CHAT_MARKERS = ["<|im_start|>", "<|im_end|>", "<think>", "</think>", "<tools>", "</tools>",
                "<tool_call>", "</tool_call>", "<tool_result>", "</tool_result>"]


def tokenizer_pieces(vocab: int, seed: int = 0):
    """(pieces, types, scores): 4 controls, chat markers, 256 byte pieces, then ASCII pieces.

    Modelled on the synthetic vocabulary of packages/needle.js/tests/tokenizer.test.ts:4-52.
    """
    pieces = ["<pad>", "</s>", "<s>", "<unk>"]
    types = [2, 2, 2, 1]
    pieces += CHAT_MARKERS
    types += [3] * len(CHAT_MARKERS)
    for b in range(256):
        pieces.append("<0x%02X>" % b)
        types.append(4)
    seen = set(pieces)
    singles = [chr(c) for c in range(33, 127)] + ["▁"]
    for s in singles:
        if len(pieces) >= vocab:
            break
        pieces.append(s)
        types.append(0)
        seen.add(s)
    alphabet = list("abcdefghijklmnopqrstuvwxyz") + list("0123456789") + list('{}[]":,_ -.')
    r = splitmix64(seed, 8 * vocab + 64, stream=0xC0FFEE)
    k = 0
    while len(pieces) < vocab:
        length = 2 + int(r[k % len(r)] % np.uint64(6))
        k += 1
        chars = []
        for _ in range(length):
            chars.append(alphabet[int(r[k % len(r)] % np.uint64(len(alphabet)))])
            k += 1
        s = ("▁" if int(r[k % len(r)] & np.uint64(3)) == 0 else "") + "".join(chars)
        k += 1
        if s in seen:
            s = s + str(len(pieces))
        seen.add(s)
        pieces.append(s)
        types.append(0)
    scores = np.zeros(vocab, dtype=np.float32)
    for i in range(vocab):
        if types[i] == 0:
            scores[i] = -float(i) / 100.0
    return pieces[:vocab], types[:vocab], scores


def tokenizer_blob(vocab: int, seed: int = 0) -> bytes:
    pieces, types, scores = tokenizer_pieces(vocab, seed)
    out = bytearray(struct.pack("<5I", len(pieces), 0, 1, 2, 3))
    out += struct.pack("<BBH", 1, 1, 0)
    for p, t, s in zip(pieces, types, scores):
        raw = p.encode("utf-8")
        out += struct.pack("<fBH", float(s), t, len(raw)) + raw
    return bytes(out)


# ------------------------------------------------------------------ archive writer


@dataclasses.dataclass(frozen=True)
class Geometry:
    vocab: int = 8192
    dim: int = 512
    heads: int = 8
    kv_heads: int = 4
    layers: int = 27
    head_dim: int = 64
    max_seq: int = 2048
    hadamard: int = 512
    lanes: int = 4
    engram_slots: int = 8192
    engram_sub: int = 128
    engram_tables: int = 4
    engram_taps: int = 4
    engram_dilation: int = 3
    engram_orders: tuple = (2, 3)
    engram_sites: tuple = (2, 15)
    rope_theta: float = 10000.0
    kv_window: int = 256
    kv_bits: int = 8
    group: int = 128


NEEDLE2 = Geometry()


def small_geometry(layers: int = 3, vocab: int = 512, kv_window: int = 8,
                   engram_slots: int = 64) -> Geometry:
    """A Needle-shaped geometry with fewer layers/vocabulary for fast CPU tests."""
    sites = tuple(s for s in (1, 2) if s < layers)
    return dataclasses.replace(NEEDLE2, layers=layers, vocab=vocab, kv_window=kv_window,
                               engram_slots=engram_slots, engram_sites=sites, max_seq=512)


class _Writer:
    def __init__(self, seed: int, codebook: np.ndarray, group: int):
        self.seed = seed
        self.codebook = codebook
        self.group = group
        self.records = []  # (dtype, shape, blob, group, bits)

    def _normal(self, shape, std=0.02):
        n = int(np.prod(shape))
        return normal(self.seed, n, stream=len(self.records) + 1, std=std).reshape(shape)

    def dense(self, shape, dtype=DT_F32, values=None):
        v = self._normal(shape) if values is None else np.asarray(values, dtype=np.float64).reshape(shape)
        blob = v.astype("<f2").tobytes() if dtype == DT_F16 else v.astype("<f4").tobytes()
        self.records.append((dtype, tuple(shape), blob, 0, 0))

    def cq(self, rows, inputs, bits):
        w = self._normal((rows, inputs))
        packed, norms = quantize_cq(w, bits, self.codebook, self.group)
        self.records.append((DT_CQ, (rows, inputs), packed + norms, self.group, bits))

    def raw(self, blob: bytes):
        self.records.append((DT_RAW, (len(blob),), blob, 0, 0))

    def finish(self, g: Geometry) -> bytes:
        n = len(self.records)
        header = [0] * 29
        header[0] = CACT_TAG
        header[1] = n
        header[2] = len(self.codebook)
        header[3] = g.kv_window
        header[4] = g.kv_bits
        header[5] = g.vocab
        header[6] = g.dim
        header[7] = g.heads
        header[8] = g.kv_heads
        header[9] = g.layers
        header[10] = g.head_dim
        header[11] = g.max_seq
        header[12] = g.hadamard
        header[13] = g.lanes
        header[14] = g.engram_slots
        header[15] = g.engram_sub
        header[16] = g.engram_tables
        header[17] = g.engram_taps
        header[18] = g.engram_dilation
        header[19] = len(g.engram_orders)
        for i, o in enumerate(g.engram_orders):
            header[20 + i] = o
        header[24] = len(g.engram_sites)
        for i, s in enumerate(g.engram_sites):
            header[25 + i] = s
        out = bytearray(struct.pack("<29I", *header) + struct.pack("<f", g.rope_theta))
        assert len(out) == HEADER_BYTES
        out += self.codebook.astype("<f4").tobytes()
        directory_at = len(out)
        out += bytes(RECORD_BYTES * n)
        offsets = []
        for dtype, shape, blob, group, bits in self.records:
            out += bytes((-len(out)) % 64)
            offsets.append(len(out))
            out += blob
        for i, (dtype, shape, blob, group, bits) in enumerate(self.records):
            dims = list(shape) + [0] * (4 - len(shape))
            rec = struct.pack("<BBH4IQQII", dtype, len(shape), 0, *dims, offsets[i], len(blob), group, bits)
            assert len(rec) == RECORD_BYTES
            out[directory_at + i * RECORD_BYTES: directory_at + (i + 1) * RECORD_BYTES] = rec
        return bytes(out)


def build_archive(seed: int = 0, geometry: Geometry = NEEDLE2, probe_heads: bool = True) -> bytes:
    """A complete synthetic archive: every tensor N(0, 0.02) from `seed`, CQ-quantised."""
    g = geometry
    codebook = lloyd_max_codebook(g.group)
    w = _Writer(seed, codebook, g.group)
    d, hd = g.dim, g.head_dim
    w.cq(g.vocab, d, 4)  # tied embedding
    for _ in range(g.layers):
        w.dense((d,), DT_F16)                 # input norm
        w.cq(g.heads * hd, d, 2)              # query projection
        w.cq(g.kv_heads * hd, d, 2)           # key projection
        w.cq(g.kv_heads * hd, d, 2)           # value projection
        w.dense((hd,), DT_F16)                # query norm
        w.dense((hd,), DT_F16)                # key norm
        w.cq(g.heads * hd, d, 2)              # gate projection
        w.cq(d, g.heads * hd, 3)              # output projection
        w.dense((d,), DT_F16)                 # post-attention norm
        w.dense((1,), DT_F32)                 # attention gate
        w.dense((d,), DT_F16)                 # pre-Hadamard norm
        w.dense((g.hadamard,), DT_F32)        # d1
        w.dense((g.hadamard,), DT_F32)        # d2
        w.dense((g.hadamard,), DT_F32)        # d3
    L, lanes = g.layers, g.lanes
    w.dense((L,))                             # a_pre
    w.dense((L,))                             # a_post
    w.dense((L,))                             # a_res
    w.dense((L * lanes,))                     # b_pre
    w.dense((L * lanes,))                     # b_post
    w.dense((L * lanes * lanes,))             # b_res
    w.cq(L * lanes, lanes * d, 4)             # phi_pre
    w.cq(L * lanes, lanes * d, 4)             # phi_post
    w.cq(L * lanes * lanes, lanes * d, 4)     # phi_res
    for _ in g.engram_sites:
        w.cq(g.engram_tables * g.engram_slots, g.engram_sub, 2)   # tables
        w.cq(d, g.engram_tables * g.engram_sub, TERNARY_BITS)     # key projection
        w.cq(d, g.engram_tables * g.engram_sub, TERNARY_BITS)     # value projection
        w.dense((g.engram_taps, d))                               # taps
    w.dense((d,), DT_F16)                     # final norm
    if probe_heads:
        w.dense((2,), DT_F32, values=[1.0, 2.0])     # manifest: contrastive, confidence
        w.dense((4, d))                              # contrastive probes
        w.dense((64, 4 * d))                         # contrastive projection
        w.dense((64,))                               # contrastive bias
        w.dense((8, d))                              # confidence probes
        w.dense((1, 8 * d))                          # confidence projection
        w.dense((1,))                                # confidence bias
    w.raw(tokenizer_blob(g.vocab, seed))
    return w.finish(g)


def random_cq_matrix(rows: int, inputs: int, bits: int, seed: int = 2, group: int = 128):
    """Isolated-matvec operands: uniform indices (ternary crumbs uniform over {0,1,3}) and fp16
    norms |N(0,1)|*0.01, returned as (packed, norms16) byte arrays."""
    padded = -(-inputs // group) * group
    n = rows * padded
    if bits == TERNARY_BITS:
        crumbs = np.array([0, 1, 3], dtype=np.uint32)
        idx = crumbs[integers(seed, n, 3, stream=bits)].reshape(rows, padded)
        packed = pack_indices(idx, 2)
    else:
        idx = integers(seed, n, 1 << bits, stream=bits).astype(np.uint32).reshape(rows, padded)
        packed = pack_indices(idx, bits)
    norms = np.abs(normal(seed, rows * (padded // group), stream=100 + bits)) * 0.01
    return packed.reshape(-1), norms.astype("<f2").view(np.uint8)
