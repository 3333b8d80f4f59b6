"""GPU parity of the greedy head (tied logits + argmax, the tail of the
decoder step: emit_logits_argmax, src/voxtral.cpp:2966-2972) through the
C ABI against the oracle's restatement: logits within 1e-3 (fp32
accumulation against float64), argmax equal to the oracle's wherever the top
two logits are further apart than the logit tolerance, and the first index
on exact ties (ggml_argmax)."""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

F16, BF16 = 1, 30
LOGIT_TOL = 1e-3


def _weights(rng, vocab, dim, dtype, oracle):
    w = (rng.standard_normal((vocab, dim)) * 0.05).astype(np.float32)
    if dtype == F16:
        return w.astype(np.float16).view(np.uint16)
    return oracle.f32_to_bf16_bits(w)


def _run(vxk, w_bits, x, dtype, with_logits=True):
    import torch

    vocab, dim = w_bits.shape
    rows = x.shape[0]
    head = vxk.Head(dim=dim, vocab=vocab, dtype=dtype)
    dw = torch.from_numpy(w_bits.view(np.int16)).cuda()
    dx = torch.from_numpy(x).cuda()
    am = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    lg = torch.full((rows, vocab), float("nan"), device="cuda") if with_logits else None
    stream = torch.cuda.current_stream().cuda_stream
    head.logits_argmax(dw.data_ptr(), dx.data_ptr(), rows, am.data_ptr(), lg.data_ptr() if lg is not None else 0,
                       stream)
    head.sync(stream)
    out = (am.cpu().numpy(), lg.cpu().numpy() if lg is not None else None)
    head.close()
    return out


def _check_argmax(am, logits_ref, want):
    for r in range(len(am)):
        top2 = np.sort(logits_ref[r])[-2:]
        if top2[1] - top2[0] > LOGIT_TOL:
            assert am[r] == want[r], (r, am[r], want[r])
        else:  # a near-tie: the chosen logit must be one of the maxima
            assert logits_ref[r, am[r]] >= top2[1] - LOGIT_TOL


@pytest.mark.parametrize("dtype", [F16, BF16])
def test_head_matches_oracle(vxk, oracle, dtype):
    rng = np.random.default_rng(11 + dtype)
    vocab, dim, rows = 5003, 512, 37      # a partial last tile and a partial row block
    w = _weights(rng, vocab, dim, dtype, oracle)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    am, lg = _run(vxk, w, x, dtype)
    ref, want = oracle.logits_argmax(w, dtype, x)
    assert np.max(np.abs(lg - ref)) <= LOGIT_TOL
    _check_argmax(am, ref, want)


def test_head_more_rows_than_one_pass(vxk, oracle):
    rng = np.random.default_rng(3)
    vocab, dim, rows = 3000, 256, 130     # three passes of 64, 64, 2 rows
    w = _weights(rng, vocab, dim, F16, oracle)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    am, lg = _run(vxk, w, x, F16)
    ref, want = oracle.logits_argmax(w, F16, x)
    assert np.max(np.abs(lg - ref)) <= LOGIT_TOL
    _check_argmax(am, ref, want)


def test_head_first_index_on_exact_ties(vxk, oracle):
    rng = np.random.default_rng(5)
    vocab, dim, rows = 9000, 128, 4
    w = (rng.standard_normal((vocab, dim)) * 0.01).astype(np.float16)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    # rows 8000 and 8500 (other tiles) copy row 31, which is aligned with x[0]
    w[31] = np.sign(x[0]).astype(np.float16) * np.float16(0.5)
    w[8000] = w[31]
    w[8500] = w[31]
    # for x[1] the tie sits on two later rows only
    w[4000] = np.sign(x[1]).astype(np.float16) * np.float16(0.5)
    w[7000] = w[4000]
    am, _ = _run(vxk, w.view(np.uint16), x, F16, with_logits=False)
    _, want = oracle.logits_argmax(w.view(np.uint16), F16, x)
    assert am[0] == 31 == want[0]
    assert am[1] == 4000 == want[1]


def test_head_full_vocabulary(vxk, oracle):
    """The model's shape: 131072 x 3072 f16 embeddings, 64 rows."""
    rng = np.random.default_rng(7)
    vocab, dim, rows = 131072, 3072, 64
    w = (rng.standard_normal((vocab, dim), dtype=np.float32) * 0.02).astype(np.float16)
    x = rng.standard_normal((rows, dim)).astype(np.float32)
    am, lg = _run(vxk, w.view(np.uint16), x, F16)
    xr = x.astype(np.float16).astype(np.float64)
    ref = np.empty((rows, vocab))
    for v0 in range(0, vocab, 8192):  # float64 reference in slices of the vocabulary
        ref[:, v0:v0 + 8192] = xr @ w[v0:v0 + 8192].astype(np.float64).T
    want = np.argmax(ref, axis=1)
    assert np.max(np.abs(lg - ref)) <= LOGIT_TOL
    _check_argmax(am, ref, want)


def _run_q(vxk, oracle, t, w_blocks, vocab, dim, x, keep_logits=True):
    import torch

    rows = x.shape[0]
    qw = vxk.QWeight(w_blocks, type=t, n_rows=vocab, n_cols=dim, max_batch=64)
    head = vxk.Head(dim=dim, vocab=vocab, dtype=F16)
    stream = torch.cuda.current_stream().cuda_stream
    xd = torch.from_numpy(x).cuda()
    am = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
    lg = torch.full((rows, vocab), float("nan"), device="cuda")
    head.logits_argmax_q(qw, xd.data_ptr(), rows, am.data_ptr(), lg.data_ptr() if keep_logits else 0, stream)
    qw.sync(stream)
    head.sync(stream)
    out = am.cpu().numpy(), lg.cpu().numpy()
    head.close()
    qw.close()
    return out


@pytest.mark.parametrize("t", [14, 12, 8])   # Q6_K (Q4_K_M's tok_embeddings), Q4_K, Q8_0
@pytest.mark.parametrize("rows", [1, 40])
def test_quantized_head_matches_oracle(vxk, oracle, t, rows):
    """Greedy head over quantized tied embeddings (vxk_head_logits_argmax_q):
    logits within the quantized product's fp32 bound of the oracle
    (oracle.qmatmul, ggml's arithmetic), argmax equal to the oracle's wherever
    the top two logits are further apart than twice the bound; the same ids
    when the head keeps the logits in its own scratch."""
    rng = np.random.default_rng(400 + t + rows)
    vocab, dim = 4096, 3072
    w = oracle.random_qblocks(t, vocab, dim, rng)
    x = rng.normal(0, 1, (rows, dim)).astype(np.float32)
    am, lg = _run_q(vxk, oracle, t, w, vocab, dim, x)
    ref, mag, terms = oracle.qmatmul(t, w, vocab, dim, x)
    bound = (2 * terms + 8) * 2.0**-24 * mag + 1e-30
    assert np.all(np.abs(lg.astype(np.float64) - ref) <= bound)
    for r in range(rows):
        order = np.argsort(-ref[r], kind="stable")
        if ref[r, order[0]] - ref[r, order[1]] > 2 * bound[r].max():
            assert am[r] == order[0]
        else:
            assert ref[r, am[r]] >= ref[r, order[0]] - 2 * bound[r].max()
    am2, _ = _run_q(vxk, oracle, t, w, vocab, dim, x, keep_logits=False)
    np.testing.assert_array_equal(am, am2)


def test_quantized_head_first_index_on_exact_ties(vxk, oracle):
    # rows 100 and 3000 hold the same blocks and the largest logit: ggml_argmax takes 100
    rng = np.random.default_rng(9)
    vocab, dim = 4096, 512
    w = oracle.random_qblocks(8, vocab, dim, rng)
    blk = w.reshape(vocab, dim // 32, 34)
    blk[100, :, 0:2] = np.asarray([0.05] * (dim // 32), np.float16).view(np.uint8).reshape(-1, 2)
    blk[100, :, 2:] = 127
    blk[3000] = blk[100]
    x = np.ones((2, dim), np.float32)
    am, lg = _run_q(vxk, oracle, 8, w, vocab, dim, x)
    assert lg[0, 100] == lg[0, 3000] and lg[0, 100] == lg[0].max()
    assert list(am) == [100, 100]
