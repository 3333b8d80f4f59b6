"""Quantized-weight product, CPU side: the oracle and the host repack.

- The oracle's GGUF block decoders (oracle/vx_qmm.c) equal gguf 0.19.0's
  dequantize (gguf.quants, an independent numpy implementation of the same
  Q8_0 / Q4_K / Q6_K layouts) bit for bit.
- quantize_row_q8_K restated: max by magnitude with the first index winning
  ties, iscale = -127/max, round-half-to-even, clamp at 127, d = 1/iscale,
  bsums of 16; zero rows give d = 0.
- The oracle product equals the float64 product of its own dequantized
  operands up to fp32 rounding (an algebraic identity of the integer path).
- vxk_qweight_repack writes the record layout include/vxk.h and
  csrc/vxk_qmm_host.cpp document: decoded here independently, every record
  reproduces gguf's dequantized weights.
"""
from __future__ import annotations

import numpy as np
import pytest

import vx_oracle as vo
Q8_0, Q4_K, Q6_K = 8, 12, 14
TYPES = [Q8_0, Q4_K, Q6_K]


def gguf_dequant(t, blocks):
    gguf = pytest.importorskip("gguf")
    from gguf import quants

    gt = {Q8_0: gguf.GGMLQuantizationType.Q8_0, Q4_K: gguf.GGMLQuantizationType.Q4_K,
          Q6_K: gguf.GGMLQuantizationType.Q6_K}[t]
    return quants.dequantize(blocks, gt)


@pytest.mark.parametrize("t", TYPES)
def test_oracle_block_decoders_match_gguf(t):
    rng = np.random.default_rng(10 + t)
    w = vo.random_qblocks(t, 8, 1024, rng)
    ref = gguf_dequant(t, w)
    mine = np.stack([vo.dequantize_w(t, w[i], 1024) for i in range(8)])
    np.testing.assert_array_equal(mine, ref.astype(np.float32))


def test_q8_K_quantizer_rules():
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, 512).astype(np.float32)
    x[300] = -5.0
    x[301] = 5.0          # same magnitude, later: the first one (negative) sets the sign
    x[10:14] = [0.5, 1.5, 2.5, -2.5] / np.float32(127 / 5.0)  # exact halves after scaling
    d, q, bs = vo.quantize_q8_K(x)
    amax_blk1 = x[256:]
    iscale = np.float32(-127.0) / np.float32(-5.0)
    assert d[1] == np.float32(1.0) / iscale
    want = np.minimum(127, np.rint((iscale * amax_blk1).astype(np.float32))).astype(np.int8)
    np.testing.assert_array_equal(q[256:], want)
    np.testing.assert_array_equal(bs, q.reshape(-1, 16).astype(np.int32).sum(1).astype(np.int16))
    d0, q0, bs0 = vo.quantize_q8_K(np.zeros(256, np.float32))
    assert d0[0] == 0.0 and not q0.any() and not bs0.any()


@pytest.mark.parametrize("t", TYPES)
def test_oracle_product_is_the_integer_path(t):
    rng = np.random.default_rng(20 + t)
    n, k, rows = 32, 512, 3
    w = vo.random_qblocks(t, n, k, rng)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    y, mag, terms = vo.qmatmul(t, w, n, k, x)
    wf = np.stack([vo.dequantize_w(t, w[i], k) for i in range(n)]).astype(np.float64)
    if t == Q8_0:
        xq = np.stack([vo.row_to_f32(vo.quantize_q8_0(x[r]), 8, 1, k) for r in range(rows)])
    else:
        xq = []
        for r in range(rows):
            d, q, _ = vo.quantize_q8_K(x[r])
            xq.append(np.repeat(d, 256).astype(np.float64) * q.astype(np.float64))
        xq = np.stack(xq)
    exact = xq.astype(np.float64) @ wf.T
    # the oracle rounds each block's scale product to fp32 like ggml
    assert np.all(np.abs(y - exact) <= 64 * 2.0**-24 * (mag + np.abs(exact)))


def _decode_records(t, packed, n, k):
    """Independent numpy reading of the record layout -> dequantized fp32."""
    units = k // 256
    rec = {Q8_0: 4352, Q4_K: 2368, Q6_K: 3360}[t]
    packed = packed.reshape(n // 16, units, rec)
    out = np.zeros((n, k), np.float64)
    L = np.arange(32)
    g, c = L // 4, L % 4
    f16 = lambda b: b.view(np.float16).astype(np.float64)
    for T in range(n // 16):
        for u in range(units):
            r = packed[T, u]
            vals = np.zeros((16, 256), np.int64)
            if t == Q8_0:
                q = r[:4096].reshape(8, 32, 4, 4).view(np.int8)
                for i in range(4):
                    for b in range(4):
                        for j in range(8):
                            vals[g + 8 * (i & 1), 32 * j + 4 * c + 16 * (i >> 1) + b] = q[j, :, i, b]
                d = f16(r[4096:4352].copy()).reshape(8, 8, 2)       # [block][g][row g, row g+8]
                for j in range(8):
                    for rr in range(16):
                        out[16 * T + rr, 256 * u + 32 * j: 256 * u + 32 * j + 32] = \
                            vals[rr, 32 * j: 32 * j + 32] * d[j, rr % 8, rr // 8]
            elif t == Q4_K:
                q = r[:2048].reshape(4, 32, 4, 4)
                for p in range(4):
                    for i in range(4):
                        for b in range(4):
                            rows = g + 8 * (i & 1)
                            kk = 4 * c + 16 * (i >> 1) + b
                            vals[rows, 32 * (2 * p) + kk] = q[p, :, i, b] & 15
                            vals[rows, 32 * (2 * p + 1) + kk] = q[p, :, i, b] >> 4
                dd = f16(r[2048:2112].copy()).reshape(16, 2)
                sc = r[2112:2240].reshape(16, 8).astype(np.float64)
                mn = r[2240:2368].reshape(16, 8).astype(np.float64)
                for rr in range(16):
                    for j in range(8):
                        dsc = np.float32(np.float32(dd[rr, 0]) * np.float32(sc[rr, j]))
                        dm = np.float32(np.float32(dd[rr, 1]) * np.float32(mn[rr, j]))
                        out[16 * T + rr, 256 * u + 32 * j: 256 * u + 32 * j + 32] = \
                            (dsc * vals[rr, 32 * j: 32 * j + 32].astype(np.float32) - dm)
            else:
                lo = r[:2048].reshape(4, 32, 4, 4)
                hi = r[2048:3072].reshape(2, 32, 4, 4)
                for tt in range(16):
                    for b in range(4):
                        kk = 16 * tt + 4 * c + b
                        byte = lo[tt >> 2, :, tt & 3, b]
                        vals[g, kk] = byte & 15
                        vals[g + 8, kk] = byte >> 4
                for P in range(8):
                    for b in range(4):
                        k0 = 16 * (2 * P) + 4 * c + b
                        hb = hi[P >> 2, :, P & 3, b]
                        vals[g, k0] |= (hb & 3) << 4
                        vals[g + 8, k0] |= ((hb >> 2) & 3) << 4
                        vals[g, k0 + 16] |= ((hb >> 4) & 3) << 4
                        vals[g + 8, k0 + 16] |= ((hb >> 6) & 3) << 4
                sc = r[3072:3328].view(np.int8).reshape(16, 16).astype(np.float64)
                d = f16(r[3328:3360].copy())
                for rr in range(16):
                    for e in range(256):
                        out[16 * T + rr, 256 * u + e] = np.float32(
                            np.float32(np.float32(d[rr]) * np.float32(sc[rr, e // 16])) * np.float32(vals[rr, e] - 32))
    return out


@pytest.mark.parametrize("t", TYPES)
def test_repack_layout_reproduces_gguf_weights(t, vxk):
    rng = np.random.default_rng(30 + t)
    n, k = 64, 512
    w = vo.random_qblocks(t, n, k, rng)
    packed = vxk.qweight_repack(t, n, k, w)
    assert packed.size == (n // 16) * (k // 256) * {Q8_0: 4352, Q4_K: 2368, Q6_K: 3360}[t]
    got = _decode_records(t, packed, n, k)
    ref = gguf_dequant(t, w).astype(np.float64)
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-6 * np.abs(ref).max())


def test_repack_rejects_bad_shapes(vxk):
    w = vo.random_qblocks(Q4_K, 64, 512, np.random.default_rng(1))
    for n, k in ((48, 512), (64, 500), (64, 0)):
        with pytest.raises(vxk.VxkError):
            vxk.qweight_repack(Q4_K, n, k, w)
    with pytest.raises(vxk.VxkError):
        vxk.qweight_repack(Q4_K, 64, 768, w)      # byte count does not match the shape
