"""The device-resident pipeline of the realtime model, end to end on the GPU:
Mel windows -> encoder stack (vxk_encoder_forward) -> encoder-output ring
(vxk_decoder_write_enc) -> adapter (vxk_decoder_adapt) -> audio-embedding
ring -> decoder step (vxk_decoder_forward) -> greedy token, for several
streams per batch (src/voxtral.cpp: run_encoder_steady_batch 4072-4160,
build_adapter_ring_graph_reusable 2589-2620, the step graph 3047-3104),
against the oracle's encoder, adapter and decoder chained the same way.

The chain re-quantizes activations to 8 bits in every product, so it is
compared at the cascade bar of the decoder and encoder tests (5e-2 of the
largest value), with greedy tokens equal wherever the oracle's top-2 logit gap
exceeds twice the step's own logit error.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BF16 = 30
BAR = 5e-2


def test_mel_to_token_pipeline(vxk, tmp_path):
    import torch
    import decoder_model
    import vx_decoder as vd

    enc_dim = 512
    tdec = decoder_model.build(tmp_path / "dec.gguf", 41, enc_dim=enc_dim)
    tenc = decoder_model.build_encoder(tmp_path / "enc.gguf", 42, dim=enc_dim)
    epool = vxk.EncPool(n_layers=2, n_heads=8, head_dim=64, window=750, capacity=878, max_streams=4, max_new=8,
                        dtype=BF16, max_position=4096)
    dpool = vxk.Pool(n_layers=2, n_blocks=64, capacity=512, max_streams=4, max_rows=64, max_position=1024, dtype=1)
    ge, gd = vxk.Gguf(tmp_path / "enc.gguf"), vxk.Gguf(tmp_path / "dec.gguf")
    enc = vxk.Encoder(ge, epool, max_rows=16)
    dec = vxk.Decoder(gd, dpool, audio_capacity=32, enc_capacity=16)
    ge.close()
    gd.close()
    assert dec.info["enc_dim"] == enc_dim
    oenc = vd.Encoder(tenc, 2, 8, cache_dtype=BF16)
    odec = vd.Decoder(tdec, 2, capacity=512)
    rng = np.random.default_rng(43)
    n_streams = 3
    es = [epool.open_stream() for _ in range(n_streams)]
    ds = [dpool.open_stream() for _ in range(n_streams)]
    mel = [rng.normal(0, 1, (128, 64)).astype(np.float32) for _ in range(n_streams)]
    cs = torch.cuda.current_stream().cuda_stream
    tokens = [int(t) for t in rng.integers(0, dec.info["vocab"], n_streams)]
    worst = 0.0
    for chunk in range(4):
        q0 = 4 * chunk
        # encoder: 4 new frames per stream
        rows = epool.plan(es, [4] * n_streams, cs)
        wins = [decoder_model.mel_window(m, q0, 4) for m in mel]
        dmel = torch.from_numpy(np.concatenate([w.reshape(-1) for w in wins])).cuda()
        eout = torch.empty((rows, enc_dim), device="cuda")
        enc.forward(dmel.data_ptr(), eout.data_ptr(), cs)
        enc.sync(cs)
        epool.commit()
        want_enc = oenc.forward([(s, q0, 4, w) for s, w in zip(es, wins)])
        # adapter: the 4 frames of each stream -> audio position `chunk`
        for i, s in enumerate(ds):
            dec.write_enc(s, q0, 4, eout[4 * i:4 * i + 4].data_ptr(), cs)
        dec.adapt(ds, [q0] * n_streams, [chunk] * n_streams, cs)
        want_audio = odec.adapt(want_enc.reshape(n_streams, 4, enc_dim))
        # decoder: one token per stream with that audio row
        dpool.plan(ds, [1] * n_streams, cs)
        amax = torch.zeros(n_streams, dtype=torch.int32, device="cuda")
        logits = torch.empty((n_streams, dec.info["vocab"]), device="cuda")
        dec.forward(tokens, [chunk % 32] * n_streams, amax.data_ptr(), logits.data_ptr(), 0, cs)
        dec.sync(cs)
        dpool.commit()
        _, ref_l, ref_a = odec.forward([(s, [t]) for s, t in zip(ds, tokens)], want_audio)
        got_l = logits.cpu().numpy().astype(np.float64)
        got_a = amax.cpu().numpy()
        err = float(np.abs(got_l - ref_l).max() / np.abs(ref_l).max())
        e_enc = float(np.abs(eout.cpu().numpy() - want_enc).max() / np.abs(want_enc).max())
        print(f"\nchunk {chunk}: encoder rel err {e_enc:.3g}, logits rel err {err:.3g}")
        assert e_enc <= BAR and err <= BAR
        gap_bar = 2 * np.abs(got_l - ref_l).max()
        for r in range(n_streams):
            top2 = np.sort(ref_l[r])[-2:]
            if top2[1] - top2[0] > gap_bar:
                assert got_a[r] == ref_a[r]
        worst = max(worst, err)
        tokens = [int(t) for t in got_a]   # greedy feedback, as the stream decoder does
    enc.close()
    dec.close()
    epool.close()
    dpool.close()
