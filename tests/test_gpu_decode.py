"""GPU parity of the decoder KV path through the C-ABI (libvxk.so) against the
CPU oracle on identical seeded inputs.

Bar: cache bytes bit-exact (f16 RNE / ggml q8_0 blocks / f32); attention outputs
within max-abs 2e-3 of the fp64 oracle.  Shapes are the 3B/4B decoder's
(32 q heads, 8 kv heads, head_dim 128, 16-token pages, RoPE theta 1e6);
layer counts are trimmed where the oracle would take minutes.
"""
from __future__ import annotations

import numpy as np
import pytest

from gpu_harness import ATOL, Driver, max_err, rand

pytestmark = pytest.mark.gpu

F32, F16, Q8 = 0, 1, 8


def _cfg(**kw):
    base = dict(n_layers=2, n_q_heads=32, n_kv_heads=8, head_dim=128, block_tokens=16, capacity=8192,
                n_blocks=1024, max_streams=16, max_rows=512, max_position=32768, dtype=F16)
    base.update(kw)
    return base


@pytest.mark.parametrize("dtype", [F16, Q8, F32])
def test_config1_prefill_then_decode(vxk, oracle, dtype):
    """Config 1 shape: one stream, prefill 391 positions, then decode steps."""
    d = Driver(vxk, oracle, seed=1, **_cfg(n_layers=3, dtype=dtype))
    s = d.open()
    got, want = d.step([s], [391], check_rows=list(range(0, 391, 29)) + [390])
    assert max_err(got, want) <= ATOL
    allg, allw = [], []
    for _ in range(32):
        g, w = d.step([s], [1])
        allg += g
        allw += w
    assert max_err(allg, allw) <= ATOL
    d.check_cache(s)
    r = d.pool.ring(s)
    assert (r.used, r.next_absolute_position, r.wraps, r.evictions) == (423, 423, 0, 0)


def test_fused_matches_unfused(vxk, oracle):
    d1 = Driver(vxk, oracle, seed=5, **_cfg())
    d2 = Driver(vxk, oracle, seed=5, **_cfg())
    s1, s2 = d1.open(), d2.open()
    d1.step([s1], [100], check_layers=[])
    d2.step([s2], [100], check_layers=[])
    for _ in range(5):
        g1, _ = d1.step([s1], [1], fused=True)
        g2, _ = d2.step([s2], [1], fused=False)
        for a, b in zip(g1, g2):
            np.testing.assert_array_equal(a, b)
    d1.check_cache(s1)
    d2.check_cache(s2)


@pytest.mark.parametrize("dtype", [F16, Q8, F32])
def test_many_streams_random_block_table(vxk, oracle, dtype):
    """Config 2 in miniature: uneven contexts, seeded random page order."""
    d = Driver(vxk, oracle, seed=2, **_cfg(dtype=dtype, n_blocks=2048, alloc_seed=99, max_rows=2048))
    rng = np.random.default_rng(22)
    streams = [d.open() for _ in range(8)]
    ctx = rng.integers(400, 1200, size=len(streams))
    # interleave prefills so pages of different streams are mixed
    for s, n in zip(streams, ctx):
        d.step([s], [int(n)], check_layers=[])
    allg, allw = [], []
    for _ in range(6):
        g, w = d.step(streams, [1] * len(streams))
        allg += g
        allw += w
    assert max_err(allg, allw) <= ATOL
    for s in streams[:3]:
        d.check_cache(s)


@pytest.mark.parametrize("dtype", [F16, Q8, F32])
def test_ring_wrap_sliding_window(vxk, oracle, dtype):
    """Realtime ring semantics with a small capacity: slots overwrite in place,
    wraps/evictions follow the reference planner, attention sees the window."""
    cap = 64
    d = Driver(vxk, oracle, seed=3, **_cfg(dtype=dtype, capacity=cap, n_blocks=64))
    a, b = d.open(), d.open()
    d.step([a], [20], check_layers=[])
    allg, allw = [], []
    for i in range(150):
        g, w = d.step([a, b], [1, 1], check_layers=[i % 2])
        allg += g
        allw += w
    assert max_err(allg, allw) <= ATOL
    ra, rb = d.pool.ring(a), d.pool.ring(b)
    # the reference planner's counters for the same sequence of appends
    ring = oracle.DecRing()
    ring.capacity = cap
    for n in [20] + [1] * 150:
        ok, p = oracle.dec_plan(ring, ring.next, n)
        assert ok
        oracle.dec_commit(ring, p)
    assert (ra.used, ra.oldest_absolute_position, ra.next_absolute_position, ra.wraps, ra.evictions) == \
        (ring.used, ring.oldest, ring.next, ring.wraps, ring.evictions)
    assert (rb.wraps, rb.evictions, rb.used) == (2, 150 - cap, cap)
    assert ra.bytes_moved == 0
    d.check_cache(a)
    d.check_cache(b)


def test_long_context_many_splits(vxk, oracle):
    d = Driver(vxk, oracle, seed=4, **_cfg(n_layers=1, n_blocks=600, max_rows=2048))
    s = d.open()
    for _ in range(3):
        d.step([s], [2000], check_layers=[])
    g, w = d.step([s], [1])
    assert max_err(g, w) <= ATOL
    g, w = d.step([s], [1])
    assert max_err(g, w) <= ATOL


def test_compaction_moves_pages_and_keeps_data(vxk, oracle):
    d = Driver(vxk, oracle, seed=6, **_cfg(n_blocks=256))
    streams = [d.open() for _ in range(4)]
    for rep in range(3):
        for s in streams:
            d.step([s], [40], check_layers=[])
    # close two streams: their pages leave holes in the pool
    d.pool.close_stream(streams[0])
    d.pool.close_stream(streams[2])
    st0 = d.pool.stats()
    moved, moved_bytes = d.pool.compact(d.stream)
    st1 = d.pool.stats()
    assert moved > 0
    page_bytes = 2 * 8 * 16 * 128 * 2 * d.pool.config.n_layers
    assert moved_bytes == moved * page_bytes
    assert st1.pages_used == st0.pages_used
    assert st1.pages_high_water == st1.pages_used
    assert st1.bytes_moved == moved_bytes
    assert sum(d.pool.ring(s).bytes_moved for s in (streams[1], streams[3])) == moved_bytes
    for s in (streams[1], streams[3]):
        d.check_cache(s)
    g, w = d.step([streams[1], streams[3]], [1, 1])
    assert max_err(g, w) <= ATOL


def test_explicit_eviction_releases_pages(vxk, oracle):
    d = Driver(vxk, oracle, seed=7, **_cfg(n_blocks=128))
    s = d.open()
    d.step([s], [300], check_layers=[])
    used0 = d.pool.stats().pages_used
    d.pool.evict(s, 200)
    d.mirror.oldest[s] = 200
    assert d.pool.stats().pages_used == used0 - 200 // 16
    r = d.pool.ring(s)
    assert (r.oldest_absolute_position, r.used, r.evictions) == (200, 100, 200)
    g, w = d.step([s], [1])
    assert max_err(g, w) <= ATOL
    d.check_cache(s)


def test_errors_are_statuses_not_faults(vxk, oracle):
    d = Driver(vxk, oracle, seed=8, **_cfg(n_blocks=8, capacity=64))
    s = d.open()
    with pytest.raises(vxk.VxkError) as e:
        d.pool.plan([s], [200])  # > capacity
    assert e.value.status == vxk.INVALID_ARGUMENT
    t = d.open()
    d.pool.plan([s, t], [64, 64])
    d.pool.abort()
    with pytest.raises(vxk.VxkError) as e:
        d.pool.plan([s, t], [64, 65])  # more pages than the pool has / over capacity
    assert e.value.status in (vxk.INVALID_ARGUMENT, vxk.OUT_OF_MEMORY)
    with pytest.raises(vxk.VxkError) as e:
        d.pool.plan([s, s], [1, 1])
    assert e.value.status == vxk.INVALID_ARGUMENT
    d.pool.plan([s], [10])
    with pytest.raises(vxk.VxkError) as e:
        d.pool.decode_layer(0, 0, 0, 0, 0)  # multi-token batch cannot use the fused step
    assert e.value.status == vxk.INVALID_STATE
    d.pool.abort()
    # exhaust the pool: s and t take all 8 pages, u needs a ninth
    u = d.open()
    d.pool.plan([s, t], [64, 64])
    d.pool.commit()
    assert d.pool.stats().pages_used == 8
    with pytest.raises(vxk.VxkError) as e:
        d.pool.plan([u], [16])
    assert e.value.status == vxk.OUT_OF_MEMORY
    assert d.pool.stats().pages_used == 8
    # the pool still works after the failed plan
    d.pool.sync(d.stream)
    d.pool.reset_stream(s)
    d.mirror.open(s)
    g, w = d.step([u], [20])
    assert max_err(g, w) <= ATOL


def test_device_wait_timeout_is_reported_and_the_pool_recovers(vxk, oracle):
    """A bounded device wait that runs out (a barrier nothing completes) is
    reported by the next sync as a timeout, and the pool keeps working."""
    d = Driver(vxk, oracle, seed=9, **_cfg(n_blocks=64, capacity=256))
    s = d.open()
    g, w = d.step([s], [30])
    assert max_err(g, w) <= ATOL
    d.pool.probe_wait_timeout(50, d.stream)
    with pytest.raises(vxk.VxkError) as e:
        d.pool.sync(d.stream)
    assert e.value.status == vxk.TIMEOUT
    d.pool.sync(d.stream)  # the error word was cleared
    for _ in range(2):
        g, w = d.step([s], [1])
        assert max_err(g, w) <= ATOL
    with pytest.raises(vxk.VxkError) as e:
        d.pool.probe_wait_timeout(0, d.stream)
    assert e.value.status == vxk.INVALID_ARGUMENT


@pytest.mark.parametrize("dtype", [F16, Q8, F32])
def test_back_to_back_layers(vxk, oracle, dtype):
    """All layers of a step launched back to back with no host sync between
    them (the decode launches after the first overlap their predecessor)."""
    import torch

    d = Driver(vxk, oracle, seed=12, **_cfg(n_layers=6, dtype=dtype, n_blocks=2048, max_rows=2048))
    streams = [d.open() for _ in range(6)]
    rng = np.random.default_rng(13)
    for s in streams:
        d.step([s], [int(rng.integers(300, 1500))], check_layers=[])
    c = d.pool.config
    for _ in range(3):
        n = len(streams)
        rows = d.pool.plan(streams, [1] * n, d.stream)
        q = rand(rng, c.n_layers, n, c.n_q_heads, c.head_dim)
        k = rand(rng, c.n_layers, n, c.n_kv_heads, c.head_dim)
        v = rand(rng, c.n_layers, n, c.n_kv_heads, c.head_dim)
        dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
        out = torch.full((c.n_layers, n, c.n_q_heads, c.head_dim), float("nan"), device="cuda")
        torch.cuda.synchronize()
        for layer in range(c.n_layers):
            d.pool.decode_layer(layer, dq[layer].data_ptr(), dk[layer].data_ptr(), dv[layer].data_ptr(),
                                out[layer].data_ptr(), d.stream)
        d.pool.sync(d.stream)
        d.pool.commit()
        o = out.cpu().numpy()
        worst = 0.0
        for layer in range(c.n_layers):
            for r, s in enumerate(streams):
                pos = d.mirror.next[s]
                d.mirror.append(s, layer, pos, k[layer, r], v[layer, r])
                want = d.mirror.attend(s, layer, pos, max(0, pos - c.capacity + 1), q[layer, r])
                worst = max(worst, float(np.max(np.abs(o[layer, r] - want))))
        for s in streams:
            d.mirror.advance(s, 1)
        assert rows == n and worst <= ATOL
    for s in streams[:2]:
        d.check_cache(s)


@pytest.mark.parametrize("n_layers", [3, 11])
def test_end_to_end_host_step_matches_device_path(vxk, oracle, n_layers):
    """11 layers: the inputs go up in runs [0, 1), [1, 3), [3, 7), [7, 11) and
    the outputs come down in runs ending at layers 3, 7, 9 and 10."""
    import torch

    cfg = _cfg(n_layers=n_layers)
    d = Driver(vxk, oracle, seed=9, **cfg)
    streams = [d.open() for _ in range(4)]
    for s in streams:
        d.step([s], [257], check_layers=[])
    c = d.pool.config
    rng = np.random.default_rng(10)
    n = len(streams)
    for step in range(2):  # the second step reuses the staging of the first
        q = torch.from_numpy(rand(rng, c.n_layers, n, c.n_q_heads, c.head_dim)).pin_memory()
        k = torch.from_numpy(rand(rng, c.n_layers, n, c.n_kv_heads, c.head_dim)).pin_memory()
        v = torch.from_numpy(rand(rng, c.n_layers, n, c.n_kv_heads, c.head_dim)).pin_memory()
        out = torch.full((c.n_layers, n, c.n_q_heads, c.head_dim), float("nan")).pin_memory()
        d.pool.decode_step_host(streams, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), d.stream)
        for layer in range(c.n_layers):
            for r, s in enumerate(streams):
                pos = d.mirror.next[s]
                d.mirror.append(s, layer, pos, k[layer, r].numpy(), v[layer, r].numpy())
                want = d.mirror.attend(s, layer, pos, max(0, pos - c.capacity + 1), q[layer, r].numpy())
                assert np.max(np.abs(out[layer, r].numpy() - want)) <= ATOL
        for s in streams:
            d.mirror.advance(s, 1)
            assert d.pool.ring(s).next_absolute_position == 258 + step
            d.check_cache(s)
