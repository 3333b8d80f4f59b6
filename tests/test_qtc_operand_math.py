"""Exactness of the integer encodings the tcgen05 quantized product feeds its
tensor cores (voxtral.cpp_b200/csrc/vxk_qmm_tc.cu, vxk_qtc_quant.h), checked
exhaustively on the CPU over every value the formats allow.

- Q6_K: one 32-bit multiply-add per pair word turns two 6-bit quants q6 of a
  sub-block with int8 scale sc into 4 p + 32768 (p = sc (q6 - 32)) in each
  16-bit half with no carry between the halves; the high byte with bit 7
  flipped is floor(p / 64) as s8 and the low byte is 4 (p mod 64) as u8, and
  64 hi + (4 lo) / 4 gives p back.
- Q4_K: a 4-bit quant spliced under the f16 exponent of 1024 (as 1024 + q,
  or 1024 + 16 q for the high nibble) and one f16 fused multiply-add with the
  6-bit sub-block scale give q * sc exactly; every f16 constant involved is
  exact and below f16's largest finite value.
- Q4_K mins: a sub-block sum s of 32 int8 activations is 128 h + l with
  h, l exact f16 values, and the mins product sum_j m_j s_j over a unit's 8
  sub-blocks stays below 2^24, so an fp32 accumulator holds it exactly in any
  order.  The main Q4_K accumulator (sum over 256 columns of q sc x) is exact
  while its partial sums stay below 2^24: true of rows whose quantized
  magnitudes average under 70 (random rows average ~30), not of a row of
  equal magnitudes (up to 256 * 945 * 127).
"""
from __future__ import annotations

import numpy as np

F16_MAX = 65504.0


def _byte(x, k):
    return (x >> np.uint32(8 * k)) & np.uint32(0xFF)


def _byte_perm(a, b, sel):
    """__byte_perm(a, b, sel) for selector nibbles < 8 (no sign replication)."""
    out = np.zeros_like(a)
    for k in range(4):
        s = (sel >> (4 * k)) & 7
        src = _byte(a, s) if s < 4 else _byte(b, s - 4)
        out |= src << np.uint32(8 * k)
    return out


def test_q6k_pair_word_split_is_exact():
    q6 = np.arange(64, dtype=np.uint32)
    b0, b2 = np.meshgrid(q6, q6, indexing="ij")
    b0, b2 = b0.ravel(), b2.ravel()
    for sc in range(-128, 128):
        m4 = np.uint32((4 * sc) & 0xFFFFFFFF)
        c4 = np.uint32((((32768 - 128 * sc) & 0xFFFFFFFF) * 0x00010001) & 0xFFFFFFFF)
        with np.errstate(over="ignore"):
            r = (b0 | (b2 << np.uint32(16))) * m4 + c4  # uint32 wrap-around, as the device
        for q, half in ((b0, r & np.uint32(0xFFFF)), (b2, r >> np.uint32(16))):
            p = sc * (q.astype(np.int64) - 32)
            assert half.min() >= 16384 and half.max() <= 49152
            assert np.array_equal(half.astype(np.int64), 4 * p + 32768)  # no carry between halves
            hi = ((half >> np.uint32(8)) ^ np.uint32(0x80)).astype(np.uint8).view(np.int8).astype(np.int64)
            lo4 = (half & np.uint32(0xFF)).astype(np.int64)
            assert np.array_equal(hi, np.floor_divide(p, 64))
            assert np.array_equal(lo4, 4 * np.mod(p, 64))
            assert np.array_equal(64 * hi + (lo4 >> 2), p)


def test_q6k_word_gather_puts_elements_in_natural_order():
    rng = np.random.default_rng(5)
    w = rng.integers(0, 64, size=(4096, 4), dtype=np.uint32)
    word = w[:, 0] | (w[:, 1] << np.uint32(8)) | (w[:, 2] << np.uint32(16)) | (w[:, 3] << np.uint32(24))
    for sc in (-128, -77, -1, 0, 1, 42, 127):
        m4 = np.uint32((4 * sc) & 0xFFFFFFFF)
        c4 = np.uint32((((32768 - 128 * sc) & 0xFFFFFFFF) * 0x00010001) & 0xFFFFFFFF)
        with np.errstate(over="ignore"):
            r02 = (word & np.uint32(0x00FF00FF)) * m4 + c4
            r13 = _byte_perm(word, np.zeros_like(word), 0x4341) * m4 + c4
        hi = _byte_perm(r02, r13, 0x7351) ^ np.uint32(0x80808080)
        lo = _byte_perm(r02, r13, 0x6240)
        for e in range(4):
            p = sc * (w[:, e].astype(np.int64) - 32)
            he = _byte(hi, e).astype(np.uint8).view(np.int8).astype(np.int64)
            assert np.array_equal(he, np.floor_divide(p, 64))
            assert np.array_equal(_byte(lo, e).astype(np.int64), 4 * np.mod(p, 64))


def _f16(bits):
    return float(np.array([bits], np.uint16).view(np.float16)[0])


def _round_f16(x):
    return float(np.float16(x))


def test_q4k_f16_splice_and_fma_give_q_times_scale():
    for s in range(64):
        # the scale as (s, s): bits 0x6400 | s is 1024 + s, minus 1024
        scl = _round_f16(_f16(0x6400 | s) - 1024.0)
        assert scl == s
        sch = _round_f16(scl * _f16(0x2C00))             # s / 16
        blo = _round_f16(scl * _f16(0xE400))             # -1024 s
        bhi = _round_f16(scl * _f16(0xD400))             # -64 s
        assert sch == s / 16 and blo == -1024 * s and bhi == -64 * s
        assert abs(blo) <= F16_MAX
        for q in range(16):
            lo_in = _f16(0x6400 | q)                     # low nibble spliced: 1024 + q
            hi_in = _f16(0x6400 | (q << 4))              # high nibble in place: 1024 + 16 q
            assert lo_in == 1024 + q and hi_in == 1024 + 16 * q
            # fused multiply-add: exact product and sum, one rounding to f16
            assert _round_f16(lo_in * scl + blo) == q * s
            assert _round_f16(hi_in * sch + bhi) == q * s


def test_q4k_mins_operands_and_sum_are_exact():
    s = np.arange(-32 * 127, 32 * 127 + 1)          # sums of 32 int8 activations in [-127, 127]
    h = np.floor_divide(s, 128)
    l = np.mod(s, 128)
    assert h.min() >= -32 and h.max() <= 31 and l.min() >= 0 and l.max() <= 127
    assert np.array_equal(128 * h + l, s)
    # every operand is an f16 integer: m, 128 m (m <= 63), l, h
    for v in (np.arange(64), 128 * np.arange(64), l, h):
        assert np.array_equal(v.astype(np.float16).astype(np.int64), v)
    # the largest |sum_j m_j s_j| of a unit's 8 sub-blocks, in any order of the 16 products
    assert 8 * 63 * 32 * 127 < 2**24


def test_q4k_main_accumulator_bound():
    # |q sc| <= 15 * 63; a unit's partial sums are integers bounded by 945 * sum |x|
    assert 15 * 63 == 945
    assert 945 * 256 * 69 < 2**24 < 945 * 256 * 70      # exact while mean |x| < 70
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (2000, 256))
    q8 = np.clip(np.rint(x * 127 / np.abs(x).max(axis=1, keepdims=True)), -127, 127)
    assert np.abs(q8).mean(axis=1).max() < 70            # Q8_K rows of random data (~30)
