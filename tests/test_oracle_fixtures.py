"""Pins the CPU oracle against the reference's own unit fixtures.

Restates, case for case, packages/needle.js/tests/cq.test.ts:8-99, fp16.test.ts:4-21 and
cact.test.ts:4-21 (the reference runs them under bun:test; no JS runtime exists here).
"""
import math
import struct

import numpy as np
import pytest


def pack(indices, bits):
    """cq.test.ts:8-18: little-endian bit packing."""
    out = bytearray(math.ceil(len(indices) * bits / 8))
    for index, value in enumerate(indices):
        bit = index * bits
        byte, shift = bit >> 3, bit & 7
        out[byte] |= (value << shift) & 0xFF
        if shift + bits > 8:
            out[byte + 1] |= value >> (8 - shift)
    return np.frombuffer(bytes(out), dtype=np.uint8)


def fixture_matrix(oracle, bits):
    """cq.test.ts:20-61: 2 rows, group 8, norms 1.25 / 0.75, hand-written codebooks."""
    group, rows = 8, 2
    source_bits = 2 if bits == 5 else bits
    mx = 3 if bits == 5 else 1 << bits
    indices = [i % mx for i in range(rows * group)]
    encoded = [3 if i == 0 else i - 1 for i in indices] if bits == 5 else indices
    packed = pack(encoded, source_bits)
    norms = np.array([oracle.number_to_float16(1.25), oracle.number_to_float16(0.75)], dtype="<u2")
    cb2 = np.array([-0.5, -0.15, 0.15, 0.5], dtype=np.float32)
    cb3 = np.array([-0.6, -0.4, -0.2, -0.05, 0.05, 0.2, 0.4, 0.6], dtype=np.float32)
    cb4 = np.array([(i - 7.5) / 12 for i in range(16)], dtype=np.float32)
    return oracle.CqMatrix(rows, group, group, bits, packed, norms, cb2, cb3, cb4)


def test_fwht_is_self_inverse_up_to_n(oracle):
    values = np.arange(1, 9, dtype=np.float32)
    twice = oracle.fwht(oracle.fwht(values))
    np.testing.assert_allclose(twice, values * 8, atol=5e-6)


def test_batched_projections_equal_individual_calls(oracle):
    m = fixture_matrix(oracle, 2)
    x = np.cos(np.arange(8) + 0.5).astype(np.float32)
    full = m.matvec(x)
    np.testing.assert_array_equal(m.matvec(x, 1, 1), full[1:2])


@pytest.mark.parametrize("bits", [2, 3, 4, 5])
def test_direct_matvec_equals_dequantized_row_dot(oracle, bits):
    m = fixture_matrix(oracle, bits)
    x = np.sin(np.arange(8) + 0.25).astype(np.float32)
    direct = m.matvec(x)
    for row in range(2):
        w = m.row(row)
        expected = sum(float(a) * float(b) for a, b in zip(w, x))
        assert abs(direct[row] - expected) < 0.5e-4  # toBeCloseTo(expected, 4)


def test_float16_known_bit_patterns(oracle):
    assert oracle.float16_to_number(0x0000) == 0
    neg_zero = oracle.float16_to_number(0x8000)
    assert neg_zero == 0 and math.copysign(1.0, neg_zero) < 0
    assert oracle.float16_to_number(0x3C00) == 1
    assert oracle.float16_to_number(0xC000) == -2
    assert oracle.float16_to_number(0x7C00) == math.inf
    assert math.isnan(oracle.float16_to_number(0x7E00))
    assert abs(oracle.float16_to_number(0x0001) - 2 ** -24) < 0.5e-12


@pytest.mark.parametrize("value", [0, -0.0, 1, -2, 0.33325, 65504, 2 ** -14, 2 ** -24])
def test_float16_round_trip(oracle, value):
    decoded = oracle.float16_to_number(oracle.number_to_float16(value))
    digits = 10 if abs(value) < 1e-4 else 3
    assert abs(decoded - value) < 0.5 * 10 ** -digits


def test_float16_matches_numpy_rne(oracle):
    """numberToFloat16 rounds to nearest even, like IEEE binary16 conversion of the f32 value."""
    rng = np.random.default_rng(7)
    vals = np.concatenate([rng.standard_normal(2000) * 10.0 ** rng.integers(-8, 5, 2000),
                           [65519.0, 65520.0, 6.1e-5, 5.96e-8, 2.98e-8]]).astype(np.float32)
    for v in vals:
        assert oracle.number_to_float16(float(v)) == int(np.float16(v).view(np.uint16))


def _err(oracle, data):
    with pytest.raises(oracle.RefError) as e:
        oracle.Model(bytes(data))
    return e.value


def test_cact_rejects_truncated_header(oracle):
    e = _err(oracle, bytearray(12))
    assert "header" in e.message.lower() and e.code == 1


def test_cact_rejects_bad_magic(oracle):
    e = _err(oracle, bytearray(120))
    assert "tag" in e.message.lower() and e.code == 1


def test_cact_validates_codebook_before_directory(oracle):
    data = bytearray(120)
    struct.pack_into("<III", data, 0, 0x05E12A83, 1, 4)
    e = _err(oracle, data)
    assert "codebook" in e.message.lower() and e.code == 2
