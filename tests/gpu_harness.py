"""Shared driver for the GPU parity tests: runs the product through the C-ABI
(voxtral.cpp_b200/vxk.py -> libvxk.so) and mirrors every append in the CPU
oracle, so each test can compare cache bytes (bit-exact) and attention
outputs (max-abs tolerance) on the same seeded inputs."""
from __future__ import annotations

import numpy as np

ATOL = 2e-3  # attention tolerance against the fp64 oracle (fp32 accumulation on the GPU)


def rand(rng, *shape):
    return rng.normal(0.0, 0.5, size=shape).astype(np.float32)


class _Rows:
    """Stored K and V rows of one (stream, layer), indexed by absolute
    position (grown by doubling), so that a window is a plain slice."""

    def __init__(self, row_bytes):
        self.k = np.zeros((0, row_bytes), np.uint8)
        self.v = np.zeros((0, row_bytes), np.uint8)

    def put(self, pos0, kb, vb):
        end = pos0 + kb.shape[0]
        if end > self.k.shape[0]:
            n = max(end + 256, self.k.shape[0] * 5 // 4)
            for name in ("k", "v"):
                old = getattr(self, name)
                grown = np.zeros((n, old.shape[1]), np.uint8)
                grown[:old.shape[0]] = old
                setattr(self, name, grown)
        self.k[pos0:end] = kb
        self.v[pos0:end] = vb


class DecoderMirror:
    """Oracle-side copy of what the pool should hold."""

    def __init__(self, oracle, n_layers, n_q, n_kv, hd, dtype, capacity, theta=1e6):
        self.o = oracle
        self.n_layers, self.n_q, self.n_kv, self.hd = n_layers, n_q, n_kv, hd
        self.dtype, self.capacity, self.theta = dtype, capacity, theta
        self.rb = oracle.row_bytes(dtype, n_kv, hd)
        self.rows = {}    # (stream, layer) -> _Rows
        self.oldest = {}  # stream -> oldest absolute position kept
        self.next = {}
        self.scale = float(np.float32(1.0 / np.sqrt(float(hd))))

    def open(self, s):
        self.oldest[s] = 0
        self.next[s] = 0
        for layer in range(self.n_layers):
            self.rows[(s, layer)] = _Rows(self.rb)

    def append(self, s, layer, pos, k, v):
        kb, vb = self.o.kv_row(k, v, pos, self.theta, self.dtype)
        self.rows[(s, layer)].put(pos, kb[None], vb[None])

    def append_many(self, s, layer, pos0, k, v):
        """k, v: [n, n_kv, hd] fp32 of positions pos0 .. pos0 + n - 1."""
        kb, vb = self.o.kv_rows(k, v, pos0, self.theta, self.dtype)
        self.rows[(s, layer)].put(pos0, kb, vb)

    def advance(self, s, n):
        self.next[s] += n
        self.oldest[s] = max(self.oldest[s], self.next[s] - self.capacity)

    def window_start(self, s, pos, oldest_before):
        return max(oldest_before, pos - self.capacity + 1)

    def window(self, s, layer, lo, hi):
        """Stored K and V rows of positions [lo, hi)."""
        r = self.rows[(s, layer)]
        return r.k[lo:hi], r.v[lo:hi]

    def attend(self, s, layer, pos, win_start, q):
        k, v = self.window(s, layer, win_start, pos + 1)
        return self.o.attn_row(q, pos, self.theta, k, v, self.dtype, self.n_kv, self.scale)


class Driver:
    """Runs batches through a vxk.Pool with torch device buffers."""

    def __init__(self, vxk, oracle, seed=0, **cfg):
        import torch

        self.torch = torch
        self.vxk = vxk
        self.pool = vxk.Pool(**cfg)
        c = self.pool.config
        self.mirror = DecoderMirror(oracle, c.n_layers, c.n_q_heads, c.n_kv_heads, c.head_dim, c.dtype, c.capacity,
                                    c.rope_theta)
        self.rng = np.random.default_rng(seed)
        self.stream = torch.cuda.current_stream().cuda_stream

    def open(self):
        s = self.pool.open_stream()
        self.mirror.open(s)
        return s

    def fill(self, s, n, chunk=4096):
        """Append-only prefill of n positions to stream s (every layer, no
        attention), in batches of at most `chunk` rows, mirrored in the oracle."""
        torch = self.torch
        c = self.pool.config
        left = n
        while left > 0:
            m = min(chunk, left)
            rows = self.pool.plan([s], [m], self.stream)
            assert rows == m
            pos0 = self.mirror.next[s]
            for layer in range(c.n_layers):
                k = rand(self.rng, m, c.n_kv_heads, c.head_dim)
                v = rand(self.rng, m, c.n_kv_heads, c.head_dim)
                dk, dv = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
                self.pool.append_layer(layer, dk.data_ptr(), dv.data_ptr(), self.stream)
                self.mirror.append_many(s, layer, pos0, k, v)
            self.pool.sync(self.stream)
            self.pool.commit()
            self.mirror.advance(s, m)
            left -= m

    def step(self, stream_ids, n_new, fused=None, check_layers=None, check_rows=None):
        """One planned batch over every layer.  Returns (got, want) lists of
        output arrays for the checked (layer, row) pairs."""
        torch = self.torch
        c = self.pool.config
        n_rows = self.pool.plan(stream_ids, n_new, self.stream)
        single = all(n == 1 for n in n_new)
        fused = single if fused is None else fused
        # host-side bookkeeping of the rows
        rows = []
        for s, n in zip(stream_ids, n_new):
            oldest_before = self.mirror.oldest[s]
            for t in range(n):
                pos = self.mirror.next[s] + t
                rows.append((s, pos, self.mirror.window_start(s, pos, oldest_before)))
        assert len(rows) == n_rows
        got, want = [], []
        check_layers = range(c.n_layers) if check_layers is None else check_layers
        check_rows = range(n_rows) if check_rows is None else check_rows
        for layer in range(c.n_layers):
            q = rand(self.rng, n_rows, c.n_q_heads, c.head_dim)
            k = rand(self.rng, n_rows, c.n_kv_heads, c.head_dim)
            v = rand(self.rng, n_rows, c.n_kv_heads, c.head_dim)
            dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
            dout = torch.full((n_rows, c.n_q_heads, c.head_dim), float("nan"), device="cuda")
            if fused:
                self.pool.decode_layer(layer, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), dout.data_ptr(), self.stream)
            else:
                self.pool.append_layer(layer, dk.data_ptr(), dv.data_ptr(), self.stream)
                self.pool.attend_layer(layer, dq.data_ptr(), dout.data_ptr(), self.stream)
            r0 = 0
            for s, n in zip(stream_ids, n_new):
                self.mirror.append_many(s, layer, rows[r0][1], k[r0:r0 + n], v[r0:r0 + n])
                r0 += n
            if layer in check_layers:
                out = dout.cpu().numpy()
                for r in check_rows:
                    s, pos, ws = rows[r]
                    got.append(out[r])
                    want.append(self.mirror.attend(s, layer, pos, ws, q[r]))
        self.pool.sync(self.stream)
        self.pool.commit()
        for s, n in zip(stream_ids, n_new):
            self.mirror.advance(s, n)
        return got, want

    def check_cache(self, s, layers=None, positions=None):
        """Bit-exact comparison of stored rows for the stream's live window."""
        c = self.pool.config
        lo, hi = self.mirror.oldest[s], self.mirror.next[s]
        if positions is None:
            positions = (lo, hi - lo)
        p0, n = positions
        for layer in (range(c.n_layers) if layers is None else layers):
            k, v = self.pool.read_rows(layer, s, p0, n, self.stream)
            wk, wv = self.mirror.window(s, layer, p0, p0 + n)
            np.testing.assert_array_equal(k, wk, err_msg=f"K bytes, stream {s} layer {layer}")
            np.testing.assert_array_equal(v, wv, err_msg=f"V bytes, stream {s} layer {layer}")


def max_err(got, want):
    if not got:
        return 0.0
    return float(max(np.max(np.abs(g - w)) for g, w in zip(got, want)))
