"""Pins the CPU oracle before it is trusted as the parity checker.

* f16 / bf16 round-to-nearest-even against numpy (tests/golden/f16_bf16.npz)
* q8_0 against gguf 0.19.0's restatement of ggml quantize_row_q8_0_ref
  (tests/golden/q8_0_blocks.npz)
* RoPE mode 0: the rotation arithmetic against an independent numpy float32
  restatement built on the oracle's cos/sin cache, and the cache itself
  against float64 cos/sin of the float32 theta chain
* attention against an independent numpy float64 softmax(QK^T)V
RoPE rounding inside ggml itself cannot be pinned here (ggml is absent).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_f16_matches_numpy(oracle):
    d = np.load(GOLDEN / "f16_bf16.npz")
    got = oracle.f32_to_f16_bits(d["x"])
    np.testing.assert_array_equal(got, d["f16"])


def test_bf16_matches_reference_rounding(oracle):
    d = np.load(GOLDEN / "f16_bf16.npz")
    got = oracle.f32_to_bf16_bits(d["x"])
    np.testing.assert_array_equal(got, d["bf16"])


def test_q8_0_matches_gguf(oracle):
    d = np.load(GOLDEN / "q8_0_blocks.npz")
    got = oracle.quantize_q8_0(d["x"])
    np.testing.assert_array_equal(got, d["blocks"])


def test_q8_0_ties_round_away_from_zero(oracle):
    # amax 127 -> d = 1, id = 1: x*id lands exactly on .5
    x = np.zeros(32, dtype=np.float32)
    x[0] = 127.0
    x[1], x[2], x[3], x[4] = 0.5, 2.5, -0.5, -2.5
    b = oracle.quantize_q8_0(x[None, :])[0]
    qs = b[2:].view(np.int8)
    assert list(qs[:5]) == [127, 1, 3, -1, -3]


def test_rope_cache_theta_chain(oracle):
    base, n_dims = np.float32(1e6), 128
    for pos in (0, 1, 7, 391, 8191, 22499, 32767):
        cs = oracle.rope_cache(pos, n_dims, float(base))
        theta_scale = np.float32(base) ** np.float32(-2.0 / n_dims)
        theta = np.float32(pos)
        for i in range(n_dims // 2):
            # libm cosf/sinf are within an ulp of the float64 value of the same theta
            assert abs(float(cs[2 * i]) - np.cos(np.float64(theta))) <= 2.0 ** -23
            assert abs(float(cs[2 * i + 1]) - np.sin(np.float64(theta))) <= 2.0 ** -23
            theta = np.float32(theta * theta_scale)


def test_rope_rotation_is_separately_rounded(oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 0.5, size=(8, 128)).astype(np.float32)
    for pos in (0, 5, 1000, 20000):
        cs = oracle.rope_cache(pos, 128, 1e6)
        c, s = cs[0::2], cs[1::2]
        x0, x1 = x[:, 0::2], x[:, 1::2]
        want = np.empty_like(x)
        want[:, 0::2] = (x0 * c).astype(np.float32) - (x1 * s).astype(np.float32)
        want[:, 1::2] = (x0 * s).astype(np.float32) + (x1 * c).astype(np.float32)
        got = oracle.rope_apply(x, pos, 1e6)
        np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))


def _numpy_attention(qr, k, v, group, scale):
    out = np.empty(qr.shape, dtype=np.float64)
    for h in range(qr.shape[0]):
        kv = h // group
        s = (k[:, kv, :].astype(np.float64) @ qr[h].astype(np.float64)) * float(scale)
        p = np.exp(s - s.max())
        out[h] = (p @ v[:, kv, :].astype(np.float64)) / p.sum()
    return out


def test_attention_matches_numpy_fp64(oracle):
    rng = np.random.default_rng(11)
    n_q, n_kv, hd, n = 32, 8, 128, 77
    q = rng.normal(0, 0.5, size=(n_q, hd)).astype(np.float32)
    kf = rng.normal(0, 0.5, size=(n, n_kv, hd)).astype(np.float32)
    vf = rng.normal(0, 0.5, size=(n, n_kv, hd)).astype(np.float32)
    k16 = oracle.f32_to_f16_bits(kf).reshape(n, -1).view(np.uint8)
    v16 = oracle.f32_to_f16_bits(vf).reshape(n, -1).view(np.uint8)
    scale = np.float32(1.0 / np.sqrt(128.0))
    got = oracle.attn_row(q, 500, 1e6, k16, v16, oracle.F16, n_kv, float(scale), rope_q=False)
    kd = oracle.f32_to_f16_bits(kf).view(np.float16).astype(np.float32)
    vd = oracle.f32_to_f16_bits(vf).view(np.float16).astype(np.float32)
    want = _numpy_attention(q, kd, vd, n_q // n_kv, scale)
    np.testing.assert_allclose(got, want, atol=1e-6, rtol=0)


def test_q8_0_row_roundtrip_within_half_step(oracle):
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.5, size=(1024,)).astype(np.float32)
    b = oracle.quantize_q8_0(x[None, :])[0]
    y = oracle.row_to_f32(b, oracle.Q8_0, 8, 128)
    d = b.reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    err = np.abs(y - x).reshape(-1, 32)
    # half a step, plus |q| <= 127 times the f16 rounding of d (2^-11 relative)
    assert np.all(err <= d[:, None] * (0.5 + 127 * 2.0 ** -11) + 1e-6)


def test_cpu_step_matches_oracle_for_f16_and_q8_0(oracle):
    """The timed CPU step (bench's cpu_baseline / reference arm) computes the
    same cache bytes and attention as the oracle, for both cache formats."""
    rng = np.random.default_rng(5)
    n_q, n_kv, hd, cap, ctx = 32, 8, 128, 64, 37
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    rope = oracle.rope_table(cap + 1, hd, 1e6)
    for dtype in (1, 8):
        rb = oracle.row_bytes(dtype, 1, hd)
        kc = np.zeros((1, 1, n_kv, cap, rb), dtype=np.uint8)
        vc = np.zeros_like(kc)
        rows_k, rows_v = [], []
        for p in range(ctx + 1):
            k = rng.standard_normal((n_kv, hd)).astype(np.float32) * 0.5
            v = rng.standard_normal((n_kv, hd)).astype(np.float32) * 0.5
            kr, vr = oracle.kv_row(k, v, p, 1e6, dtype)
            rows_k.append(kr)
            rows_v.append(vr)
            if p < ctx:
                kc[0, 0, :, p] = kr.reshape(n_kv, rb)
                vc[0, 0, :, p] = vr.reshape(n_kv, rb)
        q = rng.standard_normal((1, 1, n_q, hd)).astype(np.float32) * 0.5
        out = oracle.cpu_decode_step(dtype, kc, vc, q, k[None, None], v[None, None],
                                     np.array([ctx], dtype=np.int64), np.zeros(1, dtype=np.int64),
                                     rope, scale, 2)
        np.testing.assert_array_equal(kc[0, 0, :, ctx].reshape(-1), rows_k[ctx])
        np.testing.assert_array_equal(vc[0, 0, :, ctx].reshape(-1), rows_v[ctx])
        want = oracle.attn_row(q[0, 0], ctx, 1e6, np.stack(rows_k), np.stack(rows_v), dtype, n_kv, scale)
        assert np.max(np.abs(out[0, 0] - want)) < 1e-4, dtype
