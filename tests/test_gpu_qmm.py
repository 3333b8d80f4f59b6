"""GPU parity of the quantized-weight product (vxk_qweight_matmul) through
the C ABI against the oracle's restatement of ggml's CPU arithmetic
(oracle/vx_qmm.c): activations quantized to Q8_0 / Q8_K exactly as ggml's
reference quantizers do, exact integer block dots, block scales in fp32.

Bar: |y - y_oracle| <= (2 * terms + 8) * 2^-24 * mag, mag = the sum of the
block terms' magnitudes: what fp32 summation of the same terms in another
order may differ by.  A single activation quantized one step differently
moves an output by ~1e-4 * mag, far outside the bar, so the bar also pins
the device quantizers.  Shapes: small ones (every batch size class, the
split-K path), and the decoder's own projections (src/voxtral.cpp:2659-2661,
2857) at the Q4_K_M types (attn_q/k/o Q4_K, attn_v Q6_K,
src/voxtral-quantize.cpp:146-158) and Q8_0.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q8_0, Q4_K, Q6_K = 8, 12, 14


def _run(vxk, w_blocks, t, n, k, x, max_batch=64, repeat=1):
    import torch

    qw = vxk.QWeight(w_blocks, type=t, n_rows=n, n_cols=k, max_batch=max_batch)
    xd = torch.from_numpy(x).cuda()
    outs = []
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(repeat):
        y = torch.full((x.shape[0], n), float("nan"), device="cuda")
        qw.matmul(xd.data_ptr(), x.shape[0], y.data_ptr(), stream)
        qw.sync(stream)
        outs.append(y.cpu().numpy())
    qw.close()
    return outs


def _check(oracle, t, w, n, k, x, got):
    ref, mag, terms = oracle.qmatmul(t, w, n, k, x)
    bound = (2 * terms + 8) * 2.0**-24 * mag + 1e-30
    err = np.abs(got.astype(np.float64) - ref)
    assert np.isfinite(got).all()
    worst = float((err / bound).max())
    assert worst <= 1.0, f"worst error / bound = {worst:.3g}"


@pytest.mark.parametrize("t", [Q8_0, Q4_K, Q6_K])
@pytest.mark.parametrize("rows", [1, 7, 16, 40, 64])
def test_small_shapes_every_batch_class(vxk, oracle, t, rows):
    rng = np.random.default_rng(100 * t + rows)
    n, k = 128, 512
    w = oracle.random_qblocks(t, n, k, rng)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    (got,) = _run(vxk, w, t, n, k, x)
    _check(oracle, t, w, n, k, x, got)


@pytest.mark.parametrize("t,n,k,rows", [
    (Q4_K, 4096, 3072, 64),   # attn_q, 64 batched streams
    (Q4_K, 1024, 3072, 1),    # attn_k, one stream
    (Q6_K, 1024, 3072, 64),   # attn_v
    (Q4_K, 3072, 4096, 33),   # attn_o
    (Q8_0, 4096, 3072, 16),   # attn_q of a Q8_0 model
])
def test_decoder_projection_shapes(vxk, oracle, t, n, k, rows):
    rng = np.random.default_rng(7 + n + k + rows + t)
    w = oracle.random_qblocks(t, n, k, rng)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    a, b = _run(vxk, w, t, n, k, x, repeat=2)
    np.testing.assert_array_equal(a, b)   # splits are summed in a fixed order
    _check(oracle, t, w, n, k, x, a)


def test_activation_edge_rows(vxk, oracle):
    # a zero row (d = 0), a row whose largest magnitude appears twice with
    # both signs (the first sets the scale's sign) and a row of one spike
    rng = np.random.default_rng(5)
    n, k = 64, 512
    x = rng.normal(0, 1, (3, k)).astype(np.float32)
    x[0] = 0.0
    x[1, 17] = -7.0
    x[1, 200] = 7.0
    x[2] = 0.0
    x[2, 300] = 3.0
    for t in (Q8_0, Q4_K, Q6_K):
        w = oracle.random_qblocks(t, n, k, rng)
        (got,) = _run(vxk, w, t, n, k, x, max_batch=3)
        _check(oracle, t, w, n, k, x, got)
        assert not got[0].any()


def test_rejects_bad_calls(vxk, oracle):
    import torch

    rng = np.random.default_rng(9)
    w = oracle.random_qblocks(Q4_K, 64, 256, rng)
    with pytest.raises(vxk.VxkError):
        vxk.QWeight(w, type=Q4_K, n_rows=64, n_cols=256, max_batch=513)
    with pytest.raises(vxk.VxkError):
        vxk.QWeight(w[:32], type=Q4_K, n_rows=64, n_cols=256, max_batch=4)
    qw = vxk.QWeight(w, type=Q4_K, n_rows=64, n_cols=256, max_batch=4)
    x = torch.zeros((8, 256), device="cuda")
    y = torch.zeros((8, 64), device="cuda")
    for rows in (0, 5):
        with pytest.raises(vxk.VxkError):
            qw.matmul(x.data_ptr(), rows, y.data_ptr())
    with pytest.raises(vxk.VxkError):
        qw.matmul(0, 1, y.data_ptr())
    with pytest.raises(vxk.VxkError):        # x not 16-byte aligned
        qw.matmul(x.data_ptr() + 4, 1, y.data_ptr())
    qw.close()


def test_group_of_q_k_v_matches_separate_products(vxk, oracle):
    """q, k, v of one layer (Q4_K, Q4_K, Q6_K) from one quantization of x in
    one launch: within the bar of the oracle, like the three separate
    products (which split the columns differently, so their fp32 sums may
    round differently)."""
    import torch

    rng = np.random.default_rng(21)
    k, rows = 3072, 64
    spec = [(Q4_K, 4096), (Q4_K, 1024), (Q6_K, 1024)]
    blocks = [oracle.random_qblocks(t, n, k, rng) for t, n in spec]
    mats = [vxk.QWeight(b, type=t, n_rows=n, n_cols=k, max_batch=rows) for b, (t, n) in zip(blocks, spec)]
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    ys = [torch.full((rows, n), float("nan"), device="cuda") for _, n in spec]
    vxk.qweight_matmul_group(mats, xd.data_ptr(), rows, [y.data_ptr() for y in ys], stream)
    mats[0].sync(stream)
    sep = [torch.full((rows, n), float("nan"), device="cuda") for _, n in spec]
    for m, y in zip(mats, sep):
        m.matmul(xd.data_ptr(), rows, y.data_ptr(), stream)
    mats[0].sync(stream)
    for (t, n), b, yg, ys_ in zip(spec, blocks, ys, sep):
        _check(oracle, t, b, n, k, x, yg.cpu().numpy())
        _check(oracle, t, b, n, k, x, ys_.cpu().numpy())
    for m in mats:
        m.close()


def test_group_rejects_mixed_families_and_shapes(vxk, oracle):
    import torch

    rng = np.random.default_rng(22)
    a = vxk.QWeight(oracle.random_qblocks(Q4_K, 64, 512, rng), type=Q4_K, n_rows=64, n_cols=512, max_batch=8)
    b = vxk.QWeight(oracle.random_qblocks(Q8_0, 64, 512, rng), type=Q8_0, n_rows=64, n_cols=512, max_batch=8)
    c = vxk.QWeight(oracle.random_qblocks(Q6_K, 64, 256, rng), type=Q6_K, n_rows=64, n_cols=256, max_batch=8)
    x = torch.zeros((8, 512), device="cuda")
    y = torch.zeros((8, 64), device="cuda")
    for group in ([a, b], [a, c]):
        with pytest.raises(vxk.VxkError):
            vxk.qweight_matmul_group(group, x.data_ptr(), 8, [y.data_ptr()] * len(group))
    for m in (a, b, c):
        m.close()


def test_qweight_from_gguf_file(vxk, oracle, tmp_path):
    """A model file's tensors straight to the device (vxk_qweight_create_from_gguf):
    the product of each quantized tensor matches the oracle on the same bytes."""
    gguf = pytest.importorskip("gguf")
    import torch

    rng = np.random.default_rng(31)
    path = tmp_path / "m.gguf"
    w = gguf.GGUFWriter(str(path), "voxtral_realtime")
    spec = {"dec.blk.0.attn_q.weight": (Q4_K, gguf.GGMLQuantizationType.Q4_K),
            "dec.blk.0.attn_v.weight": (Q6_K, gguf.GGMLQuantizationType.Q6_K),
            "adapter.0.weight": (Q8_0, gguf.GGMLQuantizationType.Q8_0)}
    n, k, rows = 256, 1024, 24
    blocks = {}
    for name, (t, gt) in spec.items():
        blocks[name] = oracle.random_qblocks(t, n, k, rng)
        w.add_tensor(name, blocks[name], raw_dtype=gt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    g = vxk.Gguf(path)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    xd = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    for name, (t, _) in spec.items():
        qw = g.qweight(name, max_batch=rows)
        y = torch.full((rows, n), float("nan"), device="cuda")
        qw.matmul(xd.data_ptr(), rows, y.data_ptr(), stream)
        qw.sync(stream)
        _check(oracle, t, blocks[name], n, k, x, y.cpu().numpy())
        qw.close()
    with pytest.raises(vxk.VxkError):
        g.qweight("absent")
    g.close()


@pytest.mark.parametrize("t,n,k,rows", [
    (Q4_K, 1280, 1280, 512),   # the encoder's q of 128 streams x 4 frames, 8 chunks in one launch
    (Q6_K, 1280, 5120, 200),   # the encoder's w2, a ragged last chunk
    (Q4_K, 1024, 2048, 130),   # three chunks, the last of 2 rows
    (Q8_0, 256, 512, 130),     # Q8_0 (int8 mma.sync): 64 rows per launch
])
def test_many_rows_in_one_call(vxk, oracle, t, n, k, rows):
    rng = np.random.default_rng(300 + rows + t)
    w = oracle.random_qblocks(t, n, k, rng)
    x = rng.normal(0, 1, (rows, k)).astype(np.float32)
    (got,) = _run(vxk, w, t, n, k, x, max_batch=rows)
    _check(oracle, t, w, n, k, x, got)


