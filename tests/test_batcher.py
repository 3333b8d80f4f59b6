"""The cross-context batcher's host logic (vxk_batcher_*), no GPU: a host
executor stands in for the decoder.  Contexts are threads that each call
vxk_batcher_step for their own stream, as voxtral.cpp's contexts call
voxtral_ctx_decoder_step from their own threads (include/voxtral.h:223)."""
from __future__ import annotations

import threading
import time

import pytest


def _fake(record, delay=0.0, status=0):
    def fn(streams, tokens, slots):
        record.append(list(streams))
        if delay:
            time.sleep(delay)
        return status, [t * 10 + s for s, t in zip(streams, tokens)]
    return fn


def _run_threads(vxk, b, n_threads, steps, results, errors):
    def worker(s):
        try:
            tok = s
            for i in range(steps):
                out = b.step(s, tok, i % 7)
                results.setdefault(s, []).append((tok, out))
                tok = out % 1000
        except Exception as e:  # noqa: BLE001
            errors.append(e)
    ts = [threading.Thread(target=worker, args=(s,)) for s in range(n_threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(60)
    assert not any(t.is_alive() for t in ts)


def test_every_request_gets_its_own_result(vxk):
    record = []
    b = vxk.Batcher(fn=_fake(record), max_rows=8, max_wait_us=2000)
    results, errors = {}, []
    _run_threads(vxk, b, 12, 20, results, errors)
    assert not errors
    for s, seq in results.items():
        assert len(seq) == 20
        for tok, out in seq:
            assert out == tok * 10 + s
    for batch in record:
        assert len(batch) <= 8 and len(set(batch)) == len(batch)   # one row per stream per batch
    st = b.stats()
    assert st["rows"] == 12 * 20 and st["batches"] == len(record)
    assert st["max_rows_seen"] > 1          # rows of several contexts shared batches
    b.close()


def test_expected_starts_full_batches_without_waiting(vxk):
    record = []
    b = vxk.Batcher(fn=_fake(record), max_rows=64, max_wait_us=5_000_000, expected=4)
    results, errors = {}, []
    t0 = time.monotonic()
    _run_threads(vxk, b, 4, 10, results, errors)
    assert not errors
    assert time.monotonic() - t0 < 4.0     # never waited for the 5 s deadline
    assert all(len(batch) == 4 for batch in record)
    b.close()


def test_partial_batch_after_the_deadline(vxk):
    record = []
    b = vxk.Batcher(fn=_fake(record), max_rows=64, max_wait_us=20_000)
    assert b.step(3, 5, 0) == 53          # alone: runs after the deadline
    assert record == [[3]]
    b.close()


def test_failed_batch_reaches_every_row(vxk):
    b = vxk.Batcher(fn=_fake([], status=9), max_rows=4, max_wait_us=1000)
    with pytest.raises(vxk.VxkError) as e:
        b.step(0, 1, 0)
    assert e.value.status == 9
    assert b.stats()["failed_batches"] == 1
    b.close()


def test_timeout_then_recovery(vxk):
    record = []
    b = vxk.Batcher(fn=_fake(record, delay=0.3), max_rows=4, max_wait_us=0, timeout_ms=50)
    with pytest.raises(vxk.VxkError) as e:
        b.step(1, 1, 0)
    assert e.value.status == vxk.TIMEOUT
    time.sleep(0.5)                         # the abandoned row's batch finishes on its own
    b2 = vxk.Batcher(fn=_fake([]), max_rows=4, max_wait_us=0, timeout_ms=5000)
    assert b2.step(1, 2, 0) == 21
    assert b.stats()["timeouts"] == 1
    b.close()
    b2.close()


def test_destroy_fails_queued_requests_and_waits_for_submitters(vxk):
    b = vxk.Batcher(fn=_fake([], delay=0.2), max_rows=1, max_wait_us=0)
    out = []

    def sub(s):
        try:
            out.append(b.step(s, 1, 0))
        except vxk.VxkError as e:
            out.append(e.status)
    ts = [threading.Thread(target=sub, args=(s,)) for s in range(3)]
    for t in ts:
        t.start()
    time.sleep(0.05)
    b.close()                               # returns only after every submitter left
    for t in ts:
        t.join(5)
    assert len(out) == 3
    assert vxk.INVALID_STATE in out         # queued behind the running batch


def test_rejects_bad_config(vxk):
    with pytest.raises(vxk.VxkError):
        vxk.Batcher(fn=_fake([]), max_rows=0)
    with pytest.raises(vxk.VxkError):
        vxk.Batcher(fn=_fake([]), timeout_ms=0)


def test_withdrawn_request_forms_no_empty_batch(vxk):
    """A request withdrawn (timed out) while the dispatcher waits for company
    leaves an empty queue: no batch is run and nothing counts as failed."""
    record = []
    b = vxk.Batcher(fn=_fake(record), max_rows=4, max_wait_us=300000, timeout_ms=50)
    with pytest.raises(vxk.VxkError) as e:
        b.step(1, 1, 0)
    assert e.value.status == vxk.TIMEOUT
    time.sleep(0.6)  # past the dispatcher's deadline for the withdrawn request
    st = b.stats()
    assert record == []
    assert (st["batches"], st["failed_batches"], st["timeouts"]) == (0, 0, 1)
    b.close()
