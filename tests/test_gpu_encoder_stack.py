"""GPU parity of the streaming encoder stack (vxk_encoder_forward) through the
C ABI against the oracle's restatement (oracle/vx_decoder.py, Encoder) on the
same seeded GGUF model: conv stem, layers with biases, final norm.

As for the decoder step, every product re-quantizes its input to 8 bits, so a
last-bit difference can move one activation by a quantization step and
decorrelate the rest at the 1e-2 level; each step is compared at 5e-2 of the
largest value against the fp64 oracle and against the oracle started from the
device's own conv stem output with the device attention plugged in, and the
first step (new streams) must match the latter to 1e-4.  The conv stem itself
is checked at 2e-4 of its largest value: fp32 sums of 1536 f16 products, and
conv1 rounds its inputs to f16, so a last-bit difference in a conv0 output can
round one input to the neighbouring f16 (~5e-4 of that input; observed 3.6e-5
of the largest output).
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BF16, F16, F32 = 30, 1, 0
STEP_BAR = 5e-2
EXACT_BAR = 1e-4
STEM_BAR = 2e-4


class DeviceEncAttention:
    def __init__(self, vxk, cfg):
        import torch

        self.torch = torch
        self.pool = vxk.EncPool(**cfg)
        self.ids = {}

    def begin(self, batch):
        for s, _ in batch:
            if s not in self.ids:
                self.ids[s] = self.pool.open_stream()
        self.pool.plan([self.ids[s] for s, _ in batch], [n for _, n in batch])

    def layer(self, l, q, k, v):
        torch = self.torch
        dq, dk, dv = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda() for a in (q, k, v))
        out = torch.empty_like(dq)
        self.pool.layer(l, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr())
        torch.cuda.synchronize()
        return out.cpu().numpy()

    def end(self):
        self.pool.commit()

    def close(self):
        self.pool.close()


@pytest.mark.parametrize("dtype,kind", [(BF16, "q4_k_m"), (F16, "q4_k_m"), (F32, "q4_k_m"), (BF16, "q8_0")])
def test_encoder_stack_matches_oracle(vxk, tmp_path, dtype, kind):
    # q4_k_m: the products on the tcgen05 kernel, the q/v biases added in its
    # store; q8_0: every product on the int8 mma.sync kernel, biases added by
    # the separate bias kernel after it
    import torch
    import decoder_model
    import vx_decoder as vd

    path = tmp_path / "enc.gguf"
    types = decoder_model.Q4_K_M if kind == "q4_k_m" else decoder_model.Q8_0_ALL
    t = decoder_model.build_encoder(path, 21, types=types)
    cfg = dict(n_layers=2, n_heads=8, head_dim=64, window=750, capacity=878, max_streams=4, max_new=8, dtype=dtype,
               max_position=4096)
    pool = vxk.EncPool(**cfg)
    g = vxk.Gguf(path)
    enc = vxk.Encoder(g, pool, max_rows=32)
    g.close()
    dev = DeviceEncAttention(vxk, cfg)
    comp = vd.Encoder(t, 2, 8, cache_dtype=dtype, attention=dev)
    e2e = vd.Encoder(t, 2, 8, cache_dtype=dtype)
    rng = np.random.default_rng(8)
    streams = [pool.open_stream() for _ in range(3)]
    mel = {s: rng.normal(0, 1, (128, 400)).astype(np.float32) for s in streams}
    nxt = {s: 0 for s in streams}
    cs = torch.cuda.current_stream().cuda_stream
    schedule = [[(0, 4), (1, 4), (2, 4)], [(0, 4), (2, 4)], [(1, 8), (0, 1)], [(2, 4), (1, 4), (0, 4)]]
    errs = []
    for step in schedule:
        ids = [streams[i] for i, _ in step]
        ns = [n for _, n in step]
        rows = pool.plan(ids, ns, cs)
        batch = [(s, nxt[s], n, decoder_model.mel_window(mel[s], nxt[s], n)) for s, n in zip(ids, ns)]
        dmel = torch.from_numpy(np.concatenate([b[3].reshape(-1) for b in batch])).cuda()
        stem = torch.full((rows, enc.info["dim"]), float("nan"), device="cuda")
        enc.stem(dmel.data_ptr(), stem.data_ptr(), cs)
        out = torch.full((rows, enc.info["dim"]), float("nan"), device="cuda")
        enc.forward(dmel.data_ptr(), out.data_ptr(), cs)
        enc.sync(cs)
        pool.commit()
        got, got_stem = out.cpu().numpy(), stem.cpu().numpy()
        # the conv stem: fp32 sums of 384 / 1536 f16 products against fp64
        want_stem = np.concatenate([e2e.stem(b[3], b[2]) for b in batch])
        es = float(np.abs(got_stem - want_stem).max() / np.abs(want_stem).max())
        assert es <= STEM_BAR, f"stem rel err {es:.3g}"
        want_c = comp.forward(batch, x0=got_stem)
        want_e = e2e.forward(batch)
        ec = float(np.abs(got - want_c).max() / np.abs(want_c).max())
        ee = float(np.abs(got - want_e).max() / np.abs(want_e).max())
        print(f"\nstep {step}: stem {es:.3g}, composition {ec:.3g}, end to end {ee:.3g}")
        assert np.isfinite(got).all()
        assert ec <= STEP_BAR and ee <= STEP_BAR
        errs.append(ec)
        for s, n in zip(ids, ns):
            nxt[s] += n
    assert errs[0] <= EXACT_BAR
    dev.close()
    enc.close()
    pool.close()


def test_encoder_rejects_bad_calls(vxk, tmp_path):
    import torch
    import decoder_model

    path = tmp_path / "enc2.gguf"
    decoder_model.build_encoder(path, 22)
    g = vxk.Gguf(path)
    pool = vxk.EncPool(n_layers=2, n_heads=8, head_dim=64, window=750, capacity=878, max_streams=2, max_new=8,
                       dtype=BF16, max_position=4096)
    enc = vxk.Encoder(g, pool, max_rows=4)
    out = torch.zeros((16, 512), device="cuda")
    mel = torch.zeros(128 * 20 * 2, device="cuda")
    with pytest.raises(vxk.VxkError):     # nothing planned
        enc.forward(mel.data_ptr(), out.data_ptr())
    s0, s1 = pool.open_stream(), pool.open_stream()
    pool.plan([s0, s1], [4, 4])
    with pytest.raises(vxk.VxkError):     # 8 rows > max_rows 4
        enc.forward(mel.data_ptr(), out.data_ptr())
    pool.commit()
    other = vxk.EncPool(n_layers=3, n_heads=8, head_dim=64, window=750, capacity=878, max_streams=2, max_new=8,
                        dtype=BF16, max_position=4096)
    with pytest.raises(vxk.VxkError):     # layer count differs from the model's
        vxk.Encoder(g, other)
    other.close()
    g.close()
    enc.close()
    pool.close()
