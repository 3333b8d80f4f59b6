"""CPU properties of the oracle's streaming encoder (oracle/vx_decoder.py
Encoder, the restatement of build_encoder_steady_graph, src/voxtral.cpp:2386-2511).

Streaming invariance: a stream's encoder rows do not depend on how its mel
frames are grouped into chunks, because every piece of the step is causal
per row:
- the conv stem's new rows read conv0 outputs 3 .. of their window, never the
  padded edge (causal_conv1d_graph, src/voxtral.cpp:1767-1814);
- norms, quantized products (each row quantized on its own) and biases work
  on one row;
- attention reads the stream's cached K/V of positions max(0, q - window + 1)
  .. q, all appended before the row attends (src/voxtral.cpp:2474-2487, mask
  4104-4119).

So the rows of the same positions must be bit-identical across chunkings,
with windows shorter than the sequence so that the window's lower bound moves.
Two streams interleaved in one batch must not see each other's history.
"""
from __future__ import annotations

import numpy as np
import pytest

BF16, F16 = 30, 1


def _run(t, mel, chunks, window, dtype, n_layers=2, n_heads=4):
    """Rows of positions 0 .. sum(chunks) - 1 of one stream, chunk by chunk."""
    import decoder_model
    import vx_decoder as vd

    enc = vd.Encoder(t, n_layers, n_heads, cache_dtype=dtype, window=window)
    rows, q0 = [], 0
    for n in chunks:
        rows.append(enc.forward([(0, q0, n, decoder_model.mel_window(mel, q0, n))]))
        q0 += n
    return np.concatenate(rows)


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    pytest.importorskip("gguf")
    import decoder_model

    path = tmp_path_factory.mktemp("enc") / "enc.gguf"
    t = decoder_model.build_encoder(path, 5, n_layers=2, dim=256, n_heads=4, hidden=512, n_mel=32)
    mel = np.random.default_rng(6).normal(0, 1, (32, 48)).astype(np.float32)
    return t, mel


@pytest.mark.parametrize("dtype", [BF16, F16])
@pytest.mark.parametrize("window", [5, 750])
def test_rows_do_not_depend_on_chunking(model, dtype, window):
    t, mel = model
    ref = _run(t, mel, [4, 4, 4, 4], window, dtype)
    assert ref.shape == (16, 256) and np.isfinite(ref).all()
    for chunks in ([8, 8], [1, 3, 4, 8], [5, 2, 9]):
        got = _run(t, mel, chunks, window, dtype)
        np.testing.assert_array_equal(got, ref, err_msg=f"chunks {chunks}")


def test_window_bounds_what_a_row_sees(model):
    # two streams that differ only in mel frames 0-3: a stem row at position p
    # reads frames from 2 p - 3 on, so with one layer and a window of 5 the
    # rows from position 8 on (attending positions 4 ..) read none of them and
    # agree; with the full window they keep differing
    t, mel = model
    other = mel.copy()
    other[:, :4] = np.random.default_rng(7).normal(0, 1, (32, 4)).astype(np.float32)

    def rows(window, m):
        return _run(t, m, [4, 4, 4, 4], window, BF16, n_layers=1)

    a, b = rows(5, mel), rows(5, other)
    assert not np.array_equal(a[:4], b[:4])
    np.testing.assert_array_equal(a[8:], b[8:])
    full_a, full_b = rows(750, mel), rows(750, other)
    assert not np.array_equal(full_a[8:], full_b[8:])


def test_interleaved_streams_keep_their_own_history(model):
    import decoder_model
    import vx_decoder as vd

    t, mel = model
    mel_b = np.random.default_rng(8).normal(0, 1, mel.shape).astype(np.float32)
    alone_a = _run(t, mel, [4, 4, 4], 750, BF16)
    alone_b = _run(t, mel_b, [4, 4, 4], 750, BF16)
    enc = vd.Encoder(t, 2, 4, cache_dtype=BF16, window=750)
    got_a, got_b = [], []
    for q0 in (0, 4, 8):
        out = enc.forward([(0, q0, 4, decoder_model.mel_window(mel, q0, 4)),
                           (1, q0, 4, decoder_model.mel_window(mel_b, q0, 4))])
        got_a.append(out[:4])
        got_b.append(out[4:])
    np.testing.assert_array_equal(np.concatenate(got_a), alone_a)
    np.testing.assert_array_equal(np.concatenate(got_b), alone_b)
