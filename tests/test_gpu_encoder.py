"""GPU parity of the streaming-encoder window attention (config 4 semantics)
through the C-ABI against the oracle: ring bytes bit-exact (bf16/f16 RNE, or
the fp32 values, of the rotated K and of V at slot abs % 878), outputs within
2e-3.  f32 is the reference's default encoder cache (src/voxtral.cpp:100-105)."""
from __future__ import annotations

import numpy as np
import pytest

from gpu_harness import ATOL, rand

pytestmark = pytest.mark.gpu

BF16, F16, F32 = 30, 1, 0


@pytest.mark.parametrize("dtype", [BF16, F16, F32])
def test_encoder_chunks_across_ring_wrap(vxk, oracle, dtype):
    import torch

    H, HD, L, WIN, CAP = 20, 64, 2, 750, 878
    pool = vxk.EncPool(n_layers=L, n_heads=H, head_dim=HD, window=WIN, capacity=CAP, max_streams=4,
                       max_new=128, dtype=dtype, max_position=8192)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(41)
    streams = [pool.open_stream() for _ in range(3)]
    hist = {(s, l): {} for s in streams for l in range(L)}
    nxt = {s: 0 for s in streams}
    scale = float(np.float32(1.0 / 8.0))
    # a 128-frame first block, large chunks to reach the wrap, then 80 ms chunks of 4
    schedule = [[128, 128, 64]] + [[128, 128, 128]] * 6 + [[4, 4, 4]] * 6 + [[1, 4, 8]] * 2
    worst = 0.0
    for chunk in schedule:
        n_rows = pool.plan(streams, chunk, stream)
        rows = [(s, nxt[s] + t) for s, n in zip(streams, chunk) for t in range(n)]
        assert n_rows == len(rows)
        check = len(rows) <= 32 or chunk == schedule[0]
        for layer in range(L):
            q, k, v = (rand(rng, n_rows, H, HD) for _ in range(3))
            dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
            dout = torch.full((n_rows, H, HD), float("nan"), device="cuda")
            pool.layer(layer, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dout.data_ptr(), stream)
            for r, (s, pos) in enumerate(rows):
                hist[(s, layer)][pos] = oracle.kv_row(k[r], v[r], pos, 1e6, dtype)
            if check:
                out = dout.cpu().numpy()
                for r, (s, pos) in enumerate(rows):
                    if chunk == schedule[0] and r % 17:
                        continue
                    ws = max(0, pos - (WIN - 1))
                    kk = np.stack([hist[(s, layer)][p][0] for p in range(ws, pos + 1)])
                    vv = np.stack([hist[(s, layer)][p][1] for p in range(ws, pos + 1)])
                    want = oracle.attn_row(q[r], pos, 1e6, kk, vv, dtype, H, scale)
                    worst = max(worst, float(np.max(np.abs(out[r] - want))))
        torch.cuda.synchronize()
        pool.commit()
        for s, n in zip(streams, chunk):
            nxt[s] += n
    assert worst <= ATOL
    for s in streams:
        head, evicted = pool.position(s)
        assert head == nxt[s]
        assert evicted == max(0, head - WIN)
        for layer in range(L):
            k, v = pool.read_slots(layer, s, 0, CAP, stream)
            for slot in range(CAP):
                # newest absolute frame stored in this slot
                a = slot + ((head - 1 - slot) // CAP) * CAP
                if a < 0 or a >= head or a < head - WIN:
                    continue
                wk, wv = hist[(s, layer)][a]
                np.testing.assert_array_equal(k[slot].view(np.uint8), wk, err_msg=f"K slot {slot}")
                np.testing.assert_array_equal(v[slot].view(np.uint8), wv, err_msg=f"V slot {slot}")
