"""Ring planners: the product's (libvxk.so, vxk_*_plan_make) and the oracle's.

The expectations are those of the reference's model-free tests, re-expressed:
  tests/cpp/test_decoder_kv.cpp:47-115   (decoder ring)
  tests/cpp/test_encoder_kv.cpp:145-340  (encoder ring)
Both implementations must meet them, and must agree on randomised sequences.
"""
from __future__ import annotations

import random

import pytest

CAP_ENC, WIN, MAXNEW = 878, 750, 128


# ---- decoder ------------------------------------------------------------

class DecImpl:
    def __init__(self, vxk, oracle, which):
        self.which, self.vxk, self.oracle = which, vxk, oracle

    def ring(self, capacity, used=0, oldest=0, nxt=0):
        if self.which == "product":
            r = self.vxk.DecoderKvRing()
            r.capacity, r.used, r.oldest_absolute_position, r.next_absolute_position = capacity, used, oldest, nxt
        else:
            r = self.oracle.DecRing()
            r.capacity, r.used, r.oldest, r.next = capacity, used, oldest, nxt
        return r

    def plan(self, ring, start, n):
        if self.which == "product":
            st, p = self.vxk.decoder_plan(ring, start, n)
            return st == 0, p
        return self.oracle.dec_plan(ring, start, n)

    def commit(self, ring, p):
        if self.which == "product":
            self.vxk.decoder_commit(ring, p)
        else:
            self.oracle.dec_commit(ring, p)

    @staticmethod
    def state(ring):
        oldest = getattr(ring, "oldest_absolute_position", None)
        if oldest is None:
            return ring.used, ring.oldest, ring.next, ring.wraps, ring.evictions
        return ring.used, oldest, ring.next_absolute_position, ring.wraps, ring.evictions


@pytest.fixture(params=["product", "oracle"])
def dec(request, vxk, oracle):
    return DecImpl(vxk, oracle, request.param)


def logical_positions(p, cap):
    out = []
    for s in range(p.read_nseg):
        for i in range(p.read_seg[s].len):
            slot = p.read_seg[s].slot + i
            for a in range(p.oldest_after, p.next_after):
                if a % cap == slot:
                    out.append(a)
                    break
    return out


def test_decoder_initial_and_contiguous(dec):
    ring = dec.ring(8)
    ok, p = dec.plan(ring, 0, 3)
    assert ok
    assert p.write_nseg == 1 and p.write_seg[0].slot == 0 and p.write_seg[0].len == 3
    assert p.read_nseg == 1 and p.read_seg[0].slot == 0 and p.read_seg[0].len == 3
    assert (p.used_after, p.oldest_after, p.next_after) == (3, 0, 3)
    assert p.evicted == 0 and not p.wrapped
    dec.commit(ring, p)
    used, _, nxt, _, _ = dec.state(ring)
    assert used == 3 and nxt == 3


def test_decoder_straddled_write_and_logical_read(dec):
    ring = dec.ring(8, used=6, oldest=0, nxt=6)
    ok, p = dec.plan(ring, 6, 4)
    assert ok
    assert p.write_nseg == 2
    assert (p.write_seg[0].slot, p.write_seg[0].len) == (6, 2)
    assert (p.write_seg[1].slot, p.write_seg[1].len) == (0, 2)
    assert (p.used_after, p.oldest_after, p.next_after) == (8, 2, 10)
    assert p.evicted == 2 and p.wrapped
    assert p.read_nseg == 2
    assert (p.read_seg[0].slot, p.read_seg[0].len) == (2, 6)
    assert (p.read_seg[1].slot, p.read_seg[1].len) == (0, 2)
    assert logical_positions(p, 8) == list(range(2, 10))


def test_decoder_single_step_rollover_and_eviction(dec):
    ring = dec.ring(8)
    physical = [-1] * 8
    for pos in range(25):
        ok, p = dec.plan(ring, pos, 1)
        assert ok
        physical[p.write_seg[0].slot] = pos
        dec.commit(ring, p)
        used, oldest, nxt, _, _ = dec.state(ring)
        assert nxt == pos + 1
        assert used == (pos + 1 if pos < 7 else 8)
        assert oldest == (0 if pos < 8 else pos - 7)
        logical = logical_positions(p, 8)
        assert len(logical) == used
        for i, a in enumerate(logical):
            assert a == oldest + i
            assert physical[a % 8] == a
    used, oldest, nxt, wraps, evictions = dec.state(ring)
    assert wraps == 3          # writes at absolute 8, 16, 24
    assert evictions == 17     # 25 appended into capacity 8
    assert ring.bytes_moved == 0 and ring.full_buffer_moves == 0
    assert oldest == 17


def test_decoder_invalid_plans(dec):
    ring = dec.ring(8)
    assert not dec.plan(ring, 1, 1)[0]   # discontinuity
    assert not dec.plan(ring, 0, 0)[0]
    assert not dec.plan(ring, 0, 9)[0]
    ring.used = 2                         # inconsistent: oldest + used != next
    assert not dec.plan(ring, 0, 1)[0]


def test_decoder_product_matches_oracle_random(vxk, oracle):
    rng = random.Random(1234)
    for cap in (8, 16, 48, 8192):
        pr = DecImpl(vxk, oracle, "product")
        orc = DecImpl(vxk, oracle, "oracle")
        r1, r2 = pr.ring(cap), orc.ring(cap)
        pos = 0
        for _ in range(300):
            n = rng.choice([1, 1, 1, 2, 5, cap // 2, cap])
            ok1, p1 = pr.plan(r1, pos, n)
            ok2, p2 = orc.plan(r2, pos, n)
            assert ok1 == ok2
            fields = ["absolute_start", "n_new", "write_nseg", "read_nseg", "wrapped", "used_after",
                      "oldest_after", "next_after", "evicted"]
            for f in fields:
                assert getattr(p1, f) == getattr(p2, f), f
            for s in range(2):
                assert (p1.write_seg[s].slot, p1.write_seg[s].len) == (p2.write_seg[s].slot, p2.write_seg[s].len)
                assert (p1.read_seg[s].slot, p1.read_seg[s].len) == (p2.read_seg[s].slot, p2.read_seg[s].len)
            pr.commit(r1, p1)
            orc.commit(r2, p2)
            assert pr.state(r1) == orc.state(r2)
            pos += n


# ---- encoder ------------------------------------------------------------

class EncImpl:
    def __init__(self, vxk, oracle, which):
        self.which, self.vxk, self.oracle = which, vxk, oracle

    def plan(self, q, n, cap=CAP_ENC, win=WIN):
        if self.which == "product":
            st, p = self.vxk.enc_plan(q, n, cap, win)
            return st == 0, p
        return self.oracle.enc_plan(q, n, cap, win)

    def allows(self, kv, q, win=WIN):
        if self.which == "product":
            return self.vxk.enc_mask_allows(kv, q, win)
        return self.oracle.enc_mask_allows(kv, q, win)


@pytest.fixture(params=["product", "oracle"])
def enc(request, vxk, oracle):
    return EncImpl(vxk, oracle, request.param)


class RingModel:
    def __init__(self, cap):
        self.slot = [-1] * cap
        self.cap = cap

    def apply_writes(self, p):
        a = p.q_start
        for s in range(p.write_nseg):
            for i in range(p.write_seg[s].len):
                self.slot[p.write_seg[s].slot + i] = a
                a += 1


def verify(p, m, cap=CAP_ENC):
    wabs, wtot = p.q_start, 0
    for s in range(p.write_nseg):
        for i in range(p.write_seg[s].len):
            slot = p.write_seg[s].slot + i
            assert 0 <= slot < cap and slot == wabs % cap
            wabs += 1
            wtot += 1
    assert wtot == p.n_new
    rabs, rtot = p.win_start, 0
    for s in range(p.read_nseg):
        for i in range(p.read_seg[s].len):
            slot = p.read_seg[s].slot + i
            assert 0 <= slot < cap and rabs % cap == slot
            assert m.slot[slot] == rabs
            rabs += 1
            rtot += 1
    assert rtot == p.win_len and rabs == p.win_end


def simulate(enc, batches):
    m = RingModel(CAP_ENC)
    head = 0
    total_evicted = 0
    for n in batches:
        ok, p = enc.plan(head, n)
        assert ok
        assert p.win_len <= WIN - 1 + n and p.win_len <= CAP_ENC
        assert 1 <= p.read_nseg <= 2 and 1 <= p.write_nseg <= 2
        m.apply_writes(p)
        verify(p, m)
        total_evicted += p.evicted
        head += n
        logical = head - max(0, head - WIN)
        assert logical <= WIN and head - total_evicted == logical
    return head


def test_encoder_overflow_guards(enc):
    assert not enc.plan(0, 0)[0]
    assert not enc.plan(0, -3)[0]
    assert not enc.plan(0, MAXNEW + 1)[0]
    assert not enc.plan(-1, 4)[0]
    assert enc.plan(0, MAXNEW)[0]
    assert enc.plan(0, 1)[0]


def test_encoder_first_batch(enc):
    ok, p = enc.plan(0, 4)
    assert ok
    assert (p.win_start, p.win_end, p.win_len) == (0, 4, 4)
    assert not p.read_wraps and not p.write_wraps
    assert (p.read_seg[0].slot, p.read_seg[0].len) == (0, 4)
    assert (p.conv_mel_start, p.conv_mel_end, p.conv_slice_start) == (0, 8, 0)
    assert p.evicted == 0


def test_encoder_steady_state(enc):
    simulate(enc, [1] * 2000)
    simulate(enc, [4] * 1000)
    simulate(enc, [MAXNEW] * 100)
    simulate(enc, [1 + (i * 37) % MAXNEW for i in range(300)])


def test_encoder_window_boundary_positions(enc):
    heads = [0, 1, 2, WIN - 2, WIN - 1, WIN, WIN + 1, 2 * WIN - 1, 2 * WIN, 2 * WIN + 1,
             CAP_ENC - 1, CAP_ENC, CAP_ENC + 1, 3 * WIN, 5 * CAP_ENC + 3, 100000]
    for head in heads:
        for n in (1, 2, 4, 8, MAXNEW):
            m = RingModel(CAP_ENC)
            for a in range(max(0, head - WIN), head):
                m.slot[a % CAP_ENC] = a
            ok, p = enc.plan(head, n)
            assert ok
            m.apply_writes(p)
            verify(p, m)
            assert p.win_start == max(0, head - (WIN - 1))


def test_encoder_absolute_positions_after_rollover(enc):
    _, p0 = enc.plan(0, 1)
    _, p1 = enc.plan(CAP_ENC, 1)
    assert p0.write_seg[0].slot == p1.write_seg[0].slot
    assert p1.q_start == CAP_ENC
    for pos in (0, 1, 748, 749, 750, 751, 1499, 1500, 1501):
        _, p = enc.plan(pos, 1)
        assert p.write_seg[0].slot == pos % CAP_ENC


def test_encoder_wrap_segments(enc):
    head = CAP_ENC - 3
    m = RingModel(CAP_ENC)
    for a in range(max(0, head - WIN), head):
        m.slot[a % CAP_ENC] = a
    ok, p = enc.plan(head, 8)
    assert ok and p.write_wraps and p.write_nseg == 2
    assert p.write_seg[0].slot == head % CAP_ENC and p.write_seg[1].slot == 0
    assert p.write_seg[0].len + p.write_seg[1].len == 8
    m.apply_writes(p)
    verify(p, m)
    assert p.read_wraps


def test_encoder_mask_predicate(enc):
    assert enc.allows(5, 5)
    assert enc.allows(0, 5)
    assert not enc.allows(6, 5)
    assert enc.allows(10, 10 + (WIN - 1))
    assert not enc.allows(10, 10 + WIN)
    for ql in range(4):
        q = 2000 + ql
        ws = max(0, q - (WIN - 1))
        for kv in range(ws, q + 1):
            assert enc.allows(kv, q)
        assert not enc.allows(ws - 1, q)
        assert not enc.allows(q + 1, q)


def test_encoder_conv_window_alignment(enc):
    for P in (0, 1, 2, 3, 100, 749, 750, 4000, 100000):
        ok, p = enc.plan(P, 8)
        assert ok
        assert p.conv_mel_start % 2 == 0 and p.conv_mel_start >= 0
        assert p.conv_mel_end == 2 * (P + 8)
        assert p.conv_slice_start + p.conv_mel_start // 2 == P
        if P >= 2:
            assert p.conv_slice_start == 2
        else:
            assert p.conv_mel_start == 0 and p.conv_slice_start == P


def test_encoder_batch_segmentation(enc):
    m = RingModel(CAP_ENC)
    head, remaining = 0, 5000
    while remaining > 0:
        n = min(MAXNEW, remaining)
        ok, p = enc.plan(head, n)
        assert ok
        m.apply_writes(p)
        verify(p, m)
        head += n
        remaining -= n
    assert head == 5000
