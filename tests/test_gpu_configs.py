"""GPU parity of the decoder KV path at the benchmark configurations' own sizes,
through the C-ABI (libvxk.so) against the CPU oracle on identical seeded inputs.

- config 1 in full: one stream, 30 layers, a 391-position prefill (375 audio
  + 16 prompt positions) and then 128 single-token decode steps, every layer of
  every step checked, cache bytes of all 30 layers compared at the end;
- config 5's context range: q8_0 (and f16) caches with contexts seeded
  uniform in [8192, 32768] plus the edges of that range, so that rows are cut
  into many splits and splits end on odd page counts;
- config 3's ring: one realtime stream with an 8192-slot ring driven through
  the reference's 30-minute sequence (a 38-position prefill, then 22,511
  single-token steps = 22,549 positions), whose counters the reference
  reports as 2 wraps, 14,357 evictions and 0 bytes moved
  (docs/session8-findings.md:97-106; ring rules src/voxtral.cpp:413-427,
  1604-1656); attention is checked just before and after each wrap;
- config 2's load: 64 streams with contexts seeded uniform in [400, 4096] in
  16-token pages with a random block table.

Bar: cache bytes bit-exact (f16 RNE / ggml q8_0 blocks / f32); attention outputs
within max-abs 2e-3 of the fp64 oracle.
"""
from __future__ import annotations

import numpy as np
import pytest

from gpu_harness import ATOL, Driver, max_err, rand

pytestmark = pytest.mark.gpu

F32, F16, Q8 = 0, 1, 8


def _cfg(**kw):
    base = dict(n_layers=2, n_q_heads=32, n_kv_heads=8, head_dim=128, block_tokens=16, capacity=8192,
                n_blocks=1024, max_streams=16, max_rows=4096, max_position=32768, dtype=F16)
    base.update(kw)
    return base


@pytest.mark.parametrize("dtype", [F16, Q8, F32])
def test_config1_in_full(vxk, oracle, dtype):
    """30 layers, prefill 391, then 128 decode steps with every step checked."""
    d = Driver(vxk, oracle, seed=101, **_cfg(n_layers=30, dtype=dtype, n_blocks=64, max_rows=512))
    s = d.open()
    got, want = d.step([s], [391], check_rows=list(range(0, 391, 13)) + [390])
    assert max_err(got, want) <= ATOL
    worst = 0.0
    for _ in range(128):
        g, w = d.step([s], [1])
        assert len(g) == 30
        worst = max(worst, max_err(g, w))
    assert worst <= ATOL, worst
    d.check_cache(s)
    r = d.pool.ring(s)
    assert (r.used, r.next_absolute_position, r.wraps, r.evictions, r.bytes_moved) == (519, 519, 0, 0, 0)


@pytest.mark.parametrize("dtype", [Q8, F16])
def test_config5_context_range(vxk, oracle, dtype):
    """Contexts of config 5 (seeded U[8192, 32768]) and its edges: rows of
    up to 2,048 pages split over many work items, odd page counts, a window
    ending mid-page; several decode steps with every stream checked."""
    rng = np.random.default_rng(505)
    ctx = [int(c) for c in rng.integers(8192, 32769, size=3)] + [32768, 8193]
    steps = 3
    cap = 32768 + 64
    pages = sum((c + steps) // 16 + 2 for c in ctx)
    d = Driver(vxk, oracle, seed=55, **_cfg(dtype=dtype, capacity=cap, n_blocks=pages + 16, max_streams=8,
                                            max_position=cap + 64, alloc_seed=31))
    streams = [d.open() for _ in ctx]
    for s, n in zip(streams, ctx):
        d.fill(s, n)
    assert {(n + 15) // 16 % 2 for n in ctx} == {0, 1}
    worst = 0.0
    for _ in range(steps):
        g, w = d.step(streams, [1] * len(streams))
        worst = max(worst, max_err(g, w))
    assert worst <= ATOL, worst
    for s in streams:
        d.check_cache(s)


def test_config3_thirty_minute_ring(vxk, oracle):
    """The reference's 30-minute realtime stream on an 8192-slot ring:
    38 + 22,511 positions, 2 wraps, 14,357 evictions, no bytes moved."""
    import torch

    cap, prefill, n_steps, L = 8192, 38, 22511, 2
    total = prefill + n_steps
    d = Driver(vxk, oracle, seed=303, **_cfg(n_layers=L, capacity=cap, n_blocks=cap // 16 + 8, max_streams=2,
                                             max_rows=64, max_position=total + 64))
    c = d.pool.config
    s = d.open()
    ring = oracle.DecRing()
    ring.capacity = cap

    def expect(n):
        ok, p = oracle.dec_plan(ring, ring.next, n)
        assert ok
        oracle.dec_commit(ring, p)

    def counters(r):
        return (r.used, r.oldest_absolute_position, r.next_absolute_position, r.wraps, r.evictions)

    g, w = d.step([s], [prefill], check_rows=[0, prefill - 1])
    assert max_err(g, w) <= ATOL
    expect(prefill)
    # every decode step's K/V (both layers) resident on the device; one query per layer
    rng = np.random.default_rng(304)
    k = rand(rng, L, n_steps, c.n_kv_heads, c.head_dim)
    v = rand(rng, L, n_steps, c.n_kv_heads, c.head_dim)
    q = rand(rng, L, c.n_q_heads, c.head_dim)
    for layer in range(L):
        d.mirror.append_many(s, layer, prefill, k[layer], v[layer])
    dk, dv, dq = (torch.from_numpy(a).cuda() for a in (k, v, q))
    check = [prefill, cap - 2, cap - 1, cap, cap + 1, 2 * cap - 1, 2 * cap, 2 * cap + 1, total - 1]
    out = torch.full((len(check), L, c.n_q_heads, c.head_dim), float("nan"), device="cuda")
    scratch = torch.empty((L, c.n_q_heads, c.head_dim), device="cuda")
    row_b = c.n_kv_heads * c.head_dim * 4
    seen = {}
    for i in range(n_steps):
        pos = prefill + i
        d.pool.plan([s], [1], d.stream)
        slot = check.index(pos) if pos in check else -1
        for layer in range(L):
            dst = out[slot, layer] if slot >= 0 else scratch[layer]
            d.pool.decode_layer(layer, dq[layer].data_ptr(), dk[layer].data_ptr() + i * row_b,
                                dv[layer].data_ptr() + i * row_b, dst.data_ptr(), d.stream)
        d.pool.commit()
        expect(1)
        if slot >= 0:
            seen[pos] = (counters(d.pool.ring(s)), (ring.used, ring.oldest, ring.next, ring.wraps, ring.evictions))
    d.pool.sync(d.stream)
    d.mirror.advance(s, total - prefill)
    for pos, (got_c, want_c) in seen.items():
        assert got_c == want_c, (pos, got_c, want_c)
    r = d.pool.ring(s)
    assert (r.wraps, r.evictions, r.bytes_moved, r.used) == (2, 14357, 0, cap)
    assert (r.oldest_absolute_position, r.next_absolute_position) == (total - cap, total)
    assert d.pool.stats().bytes_moved == 0
    o = out.cpu().numpy()
    worst = 0.0
    for j, pos in enumerate(check):
        ws = max(0, pos - cap + 1)
        for layer in range(L):
            want = d.mirror.attend(s, layer, pos, ws, q[layer])
            worst = max(worst, float(np.max(np.abs(o[j, layer] - want))))
    assert worst <= ATOL, worst
    d.check_cache(s)


@pytest.mark.parametrize("dtype", [F16, Q8])
def test_config2_load(vxk, oracle, dtype):
    """64 streams, contexts seeded U[400, 4096], random block table, every
    stream checked on two decode steps."""
    rng = np.random.default_rng(202)
    ctx = [int(c) for c in rng.integers(400, 4097, size=64)]
    pages = sum(c // 16 + 3 for c in ctx)
    d = Driver(vxk, oracle, seed=22, **_cfg(n_layers=2, dtype=dtype, n_blocks=pages + 64, max_streams=64,
                                            alloc_seed=77))
    streams = [d.open() for _ in ctx]
    for s, n in zip(streams, ctx):
        d.fill(s, n)
    worst = 0.0
    for _ in range(2):
        g, w = d.step(streams, [1] * len(streams), check_layers=[0, 1])
        worst = max(worst, max_err(g, w))
    assert worst <= ATOL, worst
    for s in streams[::9]:
        d.check_cache(s)
