"""vxk_decode_layer_static_scratch: the decode entry point for callers that
cannot allocate device memory on their decode path (real-time audio threads,
where cudaMalloc may synchronise the device and has no latency bound, and
hosts whose device memory is owned by another allocator).  Its split scratch
is a fixed array inside libvxk.so instead of memory the library allocates.

Checked through the C ABI, for f16, q8_0 and f32 caches, on two pools holding the
same caches: on consecutive calls (the shared array keeps the previous call's
contents) its outputs agree with vxk_decode_layer's and with the CPU oracle
within the attention tolerance, the appended cache bytes are the oracle's,
and the device's free memory does not shrink across the calls.  Batches
larger than the array are refused with an error instead of running.

This file is collected last so that a run stopping at the first failure has
run every other test before it.
"""
from __future__ import annotations

import numpy as np
import pytest

from gpu_harness import ATOL, DecoderMirror

pytestmark = pytest.mark.gpu

F32, F16, Q8 = 0, 1, 8
CFG = dict(n_layers=2, n_q_heads=32, n_kv_heads=8, head_dim=128, block_tokens=16, capacity=8192,
           n_blocks=1024, max_streams=8, max_rows=4096, max_position=16384, alloc_seed=5)


def _filled_pools(vxk, oracle, ctx, seed, dtype, split_pages=0):
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    a = vxk.Pool(dtype=dtype, **CFG)
    b = vxk.Pool(dtype=dtype, split_pages=split_pages, **CFG)
    c = b.config
    mirror = DecoderMirror(oracle, c.n_layers, c.n_q_heads, c.n_kv_heads, c.head_dim, dtype, c.capacity,
                           c.rope_theta)
    rng = np.random.default_rng(seed)
    sa = [a.open_stream() for _ in ctx]
    sb = [b.open_stream() for _ in ctx]
    for i, n in enumerate(ctx):
        mirror.open(sb[i])
        k = rng.normal(0, 0.5, (n, 8, 128)).astype(np.float32)
        v = rng.normal(0, 0.5, (n, 8, 128)).astype(np.float32)
        dk, dv = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
        for pool, s in ((a, sa[i]), (b, sb[i])):
            pool.plan([s], [n], stream)
            for layer in range(CFG["n_layers"]):
                pool.append_layer(layer, dk.data_ptr(), dv.data_ptr(), stream)
            pool.commit()
        for layer in range(CFG["n_layers"]):
            mirror.append_many(sb[i], layer, 0, k, v)
        mirror.advance(sb[i], n)
    torch.cuda.synchronize()
    return a, b, sa, sb, mirror, stream, rng


@pytest.mark.parametrize("dtype", [F16, Q8, F32])
def test_static_scratch_matches_allocating_entry_point_and_oracle(vxk, oracle, dtype):
    import torch

    a, b, sa, sb, mirror, stream, rng = _filled_pools(vxk, oracle, [900, 1500, 333, 2048], 77, dtype)
    n = len(sa)
    L = CFG["n_layers"]
    calls = 3  # the first call on the device looks up the array's address
    q = torch.from_numpy(rng.normal(0, 0.5, (calls, L, n, 32, 128)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.normal(0, 0.5, (calls, L, n, 8, 128)).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.normal(0, 0.5, (calls, L, n, 8, 128)).astype(np.float32)).cuda()
    out_a = torch.full((calls, L, n, 32, 128), float("nan"), device="cuda")
    out_b = torch.full((calls, L, n, 32, 128), float("nan"), device="cuda")
    free_before = None
    for i in range(calls):
        a.plan(sa, [1] * n, stream)
        b.plan(sb, [1] * n, stream)
        torch.cuda.synchronize()
        if i == 1:
            free_before = torch.cuda.mem_get_info()[0]
        for layer in range(L):
            a.decode_layer(layer, q[i, layer].data_ptr(), k[i, layer].data_ptr(), v[i, layer].data_ptr(),
                           out_a[i, layer].data_ptr(), stream)
            b.decode_layer_static_scratch(layer, q[i, layer].data_ptr(), k[i, layer].data_ptr(),
                                          v[i, layer].data_ptr(), out_b[i, layer].data_ptr(), stream)
        torch.cuda.synchronize()
        a.sync(stream)
        b.sync(stream)
        a.commit()
        b.commit()
    # calls after the first allocate nothing on the device
    assert torch.cuda.mem_get_info()[0] >= free_before
    assert bool(torch.isfinite(out_b).all())
    assert float((out_a - out_b).abs().max()) <= ATOL
    qh, kh, vh, ob = (t.cpu().numpy() for t in (q, k, v, out_b))
    worst = 0.0
    for i in range(calls):
        for layer in range(L):
            for r, s in enumerate(sb):
                pos = mirror.next[s] + i
                mirror.append(s, layer, pos, kh[i, layer, r], vh[i, layer, r])
                want = mirror.attend(s, layer, pos, 0, qh[i, layer, r])
                worst = max(worst, float(np.max(np.abs(ob[i, layer, r] - want))))
    assert worst <= ATOL, worst
    for s in sb:
        mirror.advance(s, calls)
    for sx, sy in zip(sa, sb):
        for layer in range(L):
            end = b.ring(sy).next_absolute_position
            ka, va = a.read_rows(layer, sx, 0, end, stream)
            kb, vb = b.read_rows(layer, sy, 0, end, stream)
            np.testing.assert_array_equal(ka, kb)
            np.testing.assert_array_equal(va, vb)
            wk, wv = mirror.window(sy, layer, 0, end)
            np.testing.assert_array_equal(kb, wk)
            np.testing.assert_array_equal(vb, wv)


def test_static_scratch_refuses_batches_beyond_its_size(vxk, oracle):
    import torch

    # 4 streams x 200 pages split one page per work item: 800 splits > 512
    a, b, sa, sb, mirror, stream, rng = _filled_pools(vxk, oracle, [3199] * 4, 78, F16, split_pages=1)
    b.plan(sb, [1] * 4, stream)
    q = torch.zeros((4, 32, 128), device="cuda")
    kv = torch.zeros((4, 8, 128), device="cuda")
    out = torch.zeros((4, 32, 128), device="cuda")
    with pytest.raises(vxk.VxkError) as e:
        b.decode_layer_static_scratch(0, q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), stream)
    assert e.value.status == vxk.INVALID_ARGUMENT
    assert "static scratch" in str(e.value)
    b.abort()
