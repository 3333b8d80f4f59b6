"""CPU checks of the whole-decoder restatement (oracle/vx_decoder.py) and of
the decoder entry points' argument checks, no GPU.

Row independence: every node of the step acts on one row at a time (the
products quantize each row on its own), so the last row of a 3-token
prefill equals the third of three single-token steps, bit for bit; and a
stream's result does not depend on the other streams of its batch.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np
import pytest

import vx_decoder as vd


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    pytest.importorskip("gguf")
    import decoder_model

    path = tmp_path_factory.mktemp("dec") / "tiny.gguf"
    t = decoder_model.build(path, 5, n_layers=1, dim=256, hidden=256, vocab=512, enc_dim=64)
    return path, t


def test_time_embedding_matches_formula():
    te = vd.time_embedding(6.0, 3072)
    half = 1536
    i = np.arange(half)
    ang = 6.0 * np.exp(-math.log(10000.0) * i / half)
    np.testing.assert_allclose(te[:half], np.cos(ang), atol=2e-6)
    np.testing.assert_allclose(te[half:], np.sin(ang), atol=2e-6)


def test_act_roundtrip_rules():
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, 512).astype(np.float32)
    # Q8_K: values are d * q with |q| <= 127 and the block maximum exactly -127 * d or 127 * d
    y = vd.act_roundtrip(vd.Q4_K, x)
    for b in range(2):
        blk = x[256 * b:256 * b + 256]
        m = blk[np.argmax(np.abs(blk))]
        assert abs(y[256 * b + np.argmax(np.abs(blk))] - m) <= abs(m) * 1e-6
    assert np.abs(y - x).max() <= np.abs(x).max() / 127
    assert np.array_equal(vd.act_roundtrip(vd.F16, x), x.astype(np.float16).astype(np.float32))
    z = vd.act_roundtrip(vd.Q8_0, x)
    assert np.abs(z - x).max() <= np.abs(x).max() / 100


def test_prefill_row_equals_single_steps(tiny):
    _, t = tiny
    rng = np.random.default_rng(1)
    toks = [int(v) for v in rng.integers(0, 512, 3)]
    audio = rng.normal(0, 0.05, (3, 256)).astype(np.float32)
    a = vd.Decoder(t, 1)
    ha, la, _ = a.forward([(0, toks)], audio)
    b = vd.Decoder(t, 1)
    for i in range(3):
        hb, lb, _ = b.forward([(0, [toks[i]])], audio[i:i + 1])
    assert np.array_equal(ha, hb)
    assert np.array_equal(la, lb)


def test_batch_neighbours_do_not_change_a_stream(tiny):
    _, t = tiny
    rng = np.random.default_rng(2)
    audio = rng.normal(0, 0.05, (4, 256)).astype(np.float32)
    a = vd.Decoder(t, 1)
    ha, _, _ = a.forward([(0, [7]), (1, [9])], audio[:2])
    b = vd.Decoder(t, 1)
    hb, _, _ = b.forward([(1, [9])], audio[1:2])
    assert np.array_equal(ha[1], hb[0])


def test_adapter_restatement_shapes(tiny):
    _, t = tiny
    d = vd.Decoder(t, 1)
    rng = np.random.default_rng(3)
    y = d.adapt(rng.normal(0, 1, (2, 4, 64)).astype(np.float32))
    assert y.shape == (2, 256) and np.isfinite(y).all()


def test_decoder_entry_points_check_arguments(vxk):
    lib = vxk.load()
    h = C.c_void_p()
    assert lib.vxk_decoder_create(None, None, None, C.byref(h)) == vxk.INVALID_ARGUMENT
    buf = C.create_string_buffer(256)
    lib.vxk_decoder_last_error(None, buf, 256)
    assert b"null" in buf.value
    assert lib.vxk_decoder_forward(None, None, None, None, None, None, None) == vxk.INVALID_ARGUMENT
    assert lib.vxk_decoder_sync(None, None, 10) == vxk.INVALID_ARGUMENT
    info = vxk.DecoderInfo()
    assert lib.vxk_decoder_get_info(None, C.byref(info)) == vxk.INVALID_ARGUMENT
    c = lib.vxk_decoder_default_config()
    assert (c.audio_capacity, c.enc_capacity, c.time_value) == (256, 256, 6.0)
