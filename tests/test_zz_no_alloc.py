"""vxk_decode_layer_static_scratch: the decode entry point for callers that
cannot allocate device memory on their decode path (real-time audio threads,
hosts whose device memory is owned by another allocator).  Its split scratch
is a fixed array inside libvxk.so instead of memory the library allocates.

Checked through the C ABI against vxk_decode_layer on two pools holding the
same caches: outputs agree within the attention tolerance on consecutive
calls (the shared array keeps the previous call's contents), and batches
larger than the array are refused with an error instead of running.
"""
from __future__ import annotations

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 2e-3
CFG = dict(n_layers=2, n_q_heads=32, n_kv_heads=8, head_dim=128, block_tokens=16, capacity=8192,
           n_blocks=1024, max_streams=8, max_rows=4096, max_position=16384, alloc_seed=5)


def _filled_pools(vxk, ctx, seed):
    import torch

    stream = torch.cuda.current_stream().cuda_stream
    a, b = vxk.Pool(**CFG), vxk.Pool(**CFG)
    rng = np.random.default_rng(seed)
    sa = [a.open_stream() for _ in ctx]
    sb = [b.open_stream() for _ in ctx]
    for i, n in enumerate(ctx):
        k = torch.from_numpy(rng.normal(0, 0.5, (n, 8, 128)).astype(np.float32)).cuda()
        v = torch.from_numpy(rng.normal(0, 0.5, (n, 8, 128)).astype(np.float32)).cuda()
        for pool, s in ((a, sa[i]), (b, sb[i])):
            pool.plan([s], [n], stream)
            for layer in range(CFG["n_layers"]):
                pool.append_layer(layer, k.data_ptr(), v.data_ptr(), stream)
            pool.commit()
    torch.cuda.synchronize()
    return a, b, sa, sb, stream, rng


def test_static_scratch_matches_allocating_entry_point(vxk):
    import torch

    a, b, sa, sb, stream, rng = _filled_pools(vxk, [900, 1500, 333, 2048], seed=77)
    n = len(sa)
    for _ in range(2):  # two calls in a row per layer, sharing the fixed array
        a.plan(sa, [1] * n, stream)
        b.plan(sb, [1] * n, stream)
        for layer in range(CFG["n_layers"]):
            q = torch.from_numpy(rng.normal(0, 0.5, (n, 32, 128)).astype(np.float32)).cuda()
            k = torch.from_numpy(rng.normal(0, 0.5, (n, 8, 128)).astype(np.float32)).cuda()
            v = torch.from_numpy(rng.normal(0, 0.5, (n, 8, 128)).astype(np.float32)).cuda()
            out_a = torch.full((n, 32, 128), float("nan"), device="cuda")
            out_b = torch.full((n, 32, 128), float("nan"), device="cuda")
            a.decode_layer(layer, q.data_ptr(), k.data_ptr(), v.data_ptr(), out_a.data_ptr(), stream)
            b.decode_layer_static_scratch(layer, q.data_ptr(), k.data_ptr(), v.data_ptr(), out_b.data_ptr(), stream)
            torch.cuda.synchronize()
            assert bool(torch.isfinite(out_b).all())
            assert float((out_a - out_b).abs().max()) <= ATOL
        a.sync(stream)
        b.sync(stream)
        a.commit()
        b.commit()
    for sx, sy in zip(sa, sb):
        ka, va = a.read_rows(0, sx, 0, a.ring(sx).next_absolute_position, stream)
        kb, vb = b.read_rows(0, sy, 0, b.ring(sy).next_absolute_position, stream)
        np.testing.assert_array_equal(ka, kb)
        np.testing.assert_array_equal(va, vb)


def test_static_scratch_refuses_batches_beyond_its_size(vxk):
    import torch

    # 4 streams x 200 pages split one page per work item: 800 splits > 512
    a, b, sa, sb, stream, rng = _filled_pools(vxk, [3199] * 4, seed=78)
    old = os.environ.get("VXK_CHUNK_PAGES")
    os.environ["VXK_CHUNK_PAGES"] = "1"
    try:
        b.plan(sb, [1] * 4, stream)
    finally:
        if old is None:
            del os.environ["VXK_CHUNK_PAGES"]
        else:
            os.environ["VXK_CHUNK_PAGES"] = old
    q = torch.zeros((4, 32, 128), device="cuda")
    kv = torch.zeros((4, 8, 128), device="cuda")
    out = torch.zeros((4, 32, 128), device="cuda")
    with pytest.raises(vxk.VxkError) as e:
        b.decode_layer_static_scratch(0, q.data_ptr(), kv.data_ptr(), kv.data_ptr(), out.data_ptr(), stream)
    assert e.value.status == vxk.INVALID_ARGUMENT
    assert "static scratch" in str(e.value)
    b.abort()
