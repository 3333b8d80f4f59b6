"""ctypes binding of the CPU oracle (vx_oracle.c / vx_cpu_step.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU legs.  The product (voxtral.cpp_b200/libvxk.so) never uses it.
See vx_oracle.h for which parts are pinned and which are parity unpinned.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libvxoracle.so"

F32, F16, Q8_0, BF16 = 0, 1, 8, 30


class DecRing(C.Structure):
    _fields_ = [("capacity", C.c_int64), ("used", C.c_int64), ("oldest", C.c_int64),
                ("next", C.c_int64), ("wraps", C.c_int64), ("evictions", C.c_int64),
                ("bytes_moved", C.c_int64), ("full_buffer_moves", C.c_int64)]


class Seg(C.Structure):
    _fields_ = [("slot", C.c_int32), ("len", C.c_int32)]


class DecPlan(C.Structure):
    _fields_ = [("absolute_start", C.c_int64), ("n_new", C.c_int32), ("write_nseg", C.c_int32),
                ("write_seg", Seg * 2), ("read_seg", Seg * 2), ("read_nseg", C.c_int32),
                ("wrapped", C.c_int32), ("used_after", C.c_int64), ("oldest_after", C.c_int64),
                ("next_after", C.c_int64), ("evicted", C.c_int64)]


class EncPlan(C.Structure):
    _fields_ = [("q_start", C.c_int64), ("n_new", C.c_int32), ("win_len", C.c_int32),
                ("win_start", C.c_int64), ("win_end", C.c_int64), ("read_seg", Seg * 2),
                ("read_nseg", C.c_int32), ("read_wraps", C.c_int32), ("write_seg", Seg * 2),
                ("write_nseg", C.c_int32), ("write_wraps", C.c_int32),
                ("conv_mel_start", C.c_int64), ("conv_mel_end", C.c_int64),
                ("conv_slice_start", C.c_int32), ("pad_", C.c_int32), ("evicted", C.c_int64)]


_lib = None


def build() -> Path:
    res = subprocess.run(["make", "-s", "-C", str(HERE)], capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{res.stdout}\n{res.stderr}")
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        P = C.c_void_p
        L.vxo_dec_kv_plan.restype = C.c_int
        L.vxo_dec_kv_plan.argtypes = [C.POINTER(DecRing), C.c_int64, C.c_int32, C.POINTER(DecPlan)]
        L.vxo_dec_kv_commit.argtypes = [C.POINTER(DecRing), C.POINTER(DecPlan)]
        L.vxo_enc_kv_plan.restype = C.c_int
        L.vxo_enc_kv_plan.argtypes = [C.c_int64, C.c_int32, C.c_int32, C.c_int32, C.POINTER(EncPlan)]
        L.vxo_enc_kv_mask_allows.restype = C.c_int
        L.vxo_enc_kv_mask_allows.argtypes = [C.c_int64, C.c_int64, C.c_int32]
        L.vxo_f32_to_f16.restype = C.c_uint16
        L.vxo_f32_to_f16.argtypes = [C.c_float]
        L.vxo_f16_to_f32.restype = C.c_float
        L.vxo_f16_to_f32.argtypes = [C.c_uint16]
        L.vxo_f32_to_f16_n.argtypes = [P, P, C.c_int64]
        L.vxo_f32_to_bf16_n.argtypes = [P, P, C.c_int64]
        L.vxo_quantize_row_q8_0.argtypes = [P, C.c_int64, P]
        L.vxo_dequantize_row_q8_0.argtypes = [P, C.c_int64, P]
        L.vxo_rope_cache.argtypes = [C.c_int64, C.c_int32, C.c_float, P]
        L.vxo_rope_table.argtypes = [C.c_int64, C.c_int32, C.c_float, P]
        L.vxo_rope_apply.argtypes = [P, C.c_int32, C.c_int32, C.c_int64, C.c_float, P]
        L.vxo_row_bytes.restype = C.c_int64
        L.vxo_row_bytes.argtypes = [C.c_int32, C.c_int32, C.c_int32]
        L.vxo_kv_row.argtypes = [P, P, C.c_int32, C.c_int32, C.c_int64, C.c_float, C.c_int32, P, P]
        L.vxo_kv_rows.argtypes = [P, P, C.c_int64, C.c_int32, C.c_int32, C.c_int64, C.c_float, C.c_int32, P, P]
        L.vxo_row_to_f32.argtypes = [P, C.c_int32, C.c_int32, C.c_int32, P]
        L.vxo_attn_row.argtypes = [P, C.c_int64, C.c_float, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   P, P, C.c_int32, C.c_int64, C.c_float, P]
        L.vxo_cpu_decode_step_f16.argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int64,
                                              P, P, P, P, P, P, P, P, C.c_int64, C.c_float, C.c_int32, P]
        L.vxo_cpu_decode_step.argtypes = [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                          C.c_int64, P, P, P, P, P, P, P, P, C.c_int64, C.c_float, C.c_int32, P]
        L.vxo_qrow_bytes.restype = C.c_int64
        L.vxo_qrow_bytes.argtypes = [C.c_int32, C.c_int64]
        L.vxo_quantize_row_q8_K.argtypes = [P, C.c_int64, P, P, P]
        L.vxo_dequantize_row_w.argtypes = [C.c_int32, P, C.c_int64, P]
        L.vxo_qmatmul.restype = C.c_int32
        L.vxo_qmatmul.argtypes = [C.c_int32, P, C.c_int32, C.c_int32, P, C.c_int32, P, P]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---- planners ---------------------------------------------------------------

def dec_plan(ring: DecRing, start: int, n_new: int):
    p = DecPlan()
    ok = lib().vxo_dec_kv_plan(C.byref(ring), start, n_new, C.byref(p))
    return bool(ok), p


def dec_commit(ring: DecRing, p: DecPlan):
    lib().vxo_dec_kv_commit(C.byref(ring), C.byref(p))


def enc_plan(q_start: int, n_new: int, capacity: int, window: int):
    p = EncPlan()
    ok = lib().vxo_enc_kv_plan(q_start, n_new, capacity, window, C.byref(p))
    return bool(ok), p


def enc_mask_allows(kv: int, q: int, window: int) -> bool:
    return bool(lib().vxo_enc_kv_mask_allows(kv, q, window))


# ---- numerics ---------------------------------------------------------------

def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().vxo_f32_to_f16_n(_ptr(x), _ptr(y), x.size)
    return y


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().vxo_f32_to_bf16_n(_ptr(x), _ptr(y), x.size)
    return y


def quantize_q8_0(x: np.ndarray) -> np.ndarray:
    """Rows of values (last dim multiple of 32) -> ggml block_q8_0 bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    flat = x.reshape(-1, n)
    out = np.empty((flat.shape[0], n // 32 * 34), dtype=np.uint8)
    for i in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[i])
        lib().vxo_quantize_row_q8_0(_ptr(row), n, out[i].ctypes.data)
    return out.reshape(x.shape[:-1] + (n // 32 * 34,))


def rope_cache(pos: int, n_dims: int, base: float) -> np.ndarray:
    cs = np.empty(n_dims, dtype=np.float32)
    lib().vxo_rope_cache(pos, n_dims, base, _ptr(cs))
    return cs


def rope_table(rows: int, n_dims: int, base: float) -> np.ndarray:
    t = np.empty((rows, n_dims), dtype=np.float32)
    lib().vxo_rope_table(rows, n_dims, base, _ptr(t))
    return t


def rope_apply(x: np.ndarray, pos: int, base: float) -> np.ndarray:
    """x: [n_heads, head_dim] fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().vxo_rope_apply(_ptr(x), x.shape[0], x.shape[1], pos, base, _ptr(y))
    return y


def row_bytes(dtype: int, n_kv: int, head_dim: int) -> int:
    return int(lib().vxo_row_bytes(dtype, n_kv, head_dim))


def kv_row(k: np.ndarray, v: np.ndarray, pos: int, base: float, dtype: int):
    """k, v: [n_kv, head_dim] fp32 -> stored (K rotated) row bytes in ggml layout."""
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    n_kv, hd = k.shape
    rb = row_bytes(dtype, n_kv, hd)
    ko = np.empty(rb, dtype=np.uint8)
    vo = np.empty(rb, dtype=np.uint8)
    lib().vxo_kv_row(_ptr(k), _ptr(v), n_kv, hd, pos, base, dtype, _ptr(ko), _ptr(vo))
    return ko, vo


def kv_rows(k: np.ndarray, v: np.ndarray, pos0: int, base: float, dtype: int):
    """k, v: [n, n_kv, head_dim] fp32 of tokens at positions pos0 .. pos0 + n - 1
    -> stored row bytes [n, row bytes] (K rotated), like kv_row on each."""
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    n, n_kv, hd = k.shape
    rb = row_bytes(dtype, n_kv, hd)
    ko = np.empty((n, rb), dtype=np.uint8)
    vo = np.empty((n, rb), dtype=np.uint8)
    lib().vxo_kv_rows(_ptr(k), _ptr(v), n, n_kv, hd, pos0, base, dtype, _ptr(ko), _ptr(vo))
    return ko, vo


def row_to_f32(row: np.ndarray, dtype: int, n_kv: int, head_dim: int) -> np.ndarray:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    out = np.empty(n_kv * head_dim, dtype=np.float32)
    lib().vxo_row_to_f32(_ptr(row), dtype, n_kv, head_dim, _ptr(out))
    return out


def attn_row(q: np.ndarray, q_pos: int, base: float, k_rows: np.ndarray, v_rows: np.ndarray,
             dtype: int, n_kv: int, scale: float, rope_q: bool = True) -> np.ndarray:
    """q: [n_q, hd] fp32 (pre-RoPE when rope_q); k_rows/v_rows: [n_keys, row_bytes] uint8."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k_rows = np.ascontiguousarray(k_rows, dtype=np.uint8)
    v_rows = np.ascontiguousarray(v_rows, dtype=np.uint8)
    n_q, hd = q.shape
    out = np.empty_like(q)
    lib().vxo_attn_row(_ptr(q), q_pos, base, 1 if rope_q else 0, n_q, n_kv, hd, _ptr(k_rows), _ptr(v_rows),
                       dtype, k_rows.shape[0], scale, _ptr(out))
    return out


def cpu_decode_step(dtype, k_cache, v_cache, q, k, v, pos, win, rope, scale, n_threads):
    """Timed multi-core CPU step for an f16 or q8_0 cache (vx_cpu_step.c):
    caches uint8 [stream][layer][kv][cap][row bytes]."""
    n_streams, n_layers, n_q, hd = q.shape
    n_kv = k.shape[2]
    cap = k_cache.shape[-2]
    out = np.empty_like(q)
    lib().vxo_cpu_decode_step(dtype, n_streams, n_layers, n_q, n_kv, hd, cap, _ptr(k_cache), _ptr(v_cache),
                              _ptr(q), _ptr(k), _ptr(v), _ptr(pos), _ptr(win), _ptr(rope), rope.shape[0],
                              scale, n_threads, _ptr(out))
    return out


def cpu_decode_step_f16(k_cache, v_cache, q, k, v, pos, win, rope, scale, n_threads):
    """Timed multi-core CPU step (vx_cpu_step.c); arrays as documented there."""
    n_streams, n_layers, n_q, hd = q.shape
    n_kv = k.shape[2]
    cap = k_cache.shape[-2]
    out = np.empty_like(q)
    lib().vxo_cpu_decode_step_f16(n_streams, n_layers, n_q, n_kv, hd, cap, _ptr(k_cache), _ptr(v_cache),
                                  _ptr(q), _ptr(k), _ptr(v), _ptr(pos), _ptr(win), _ptr(rope), rope.shape[0],
                                  scale, n_threads, _ptr(out))
    return out


def logits_argmax(w_bits: np.ndarray, dtype: int, x: np.ndarray):
    """Greedy head restated: emit_logits_argmax (src/voxtral.cpp:2966-2972),
    ggml_mul_mat(tok_embeddings, last_hidden) then ggml_argmax, for a tied
    embedding matrix stored as f16 (dtype 1) or bf16 (dtype 30).

    w_bits [vocab][dim] uint16 patterns, x [rows][dim] fp32.  Like ggml's
    f16 / bf16 dot products, each x row is first rounded to W's type; the
    products are summed here in float64 (the exact-math target).  Returns
    (logits float64 [rows][vocab], argmax int64 [rows]) with ties resolved to
    the first index, as ggml_argmax does.
    """
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == 30:
        wf = (w_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        xr = (f32_to_bf16_bits(x).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    else:
        wf = w_bits.view(np.float16).astype(np.float64)
        xr = x.astype(np.float16).astype(np.float64)
    logits = xr @ wf.T
    return logits, np.argmax(logits, axis=1)


Q4_K, Q6_K = 12, 14
QBLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def qrow_bytes(wtype: int, k: int) -> int:
    return int(lib().vxo_qrow_bytes(wtype, k))


def quantize_q8_K(x: np.ndarray):
    """ggml quantize_row_q8_K_ref on one row: (d fp32 [k/256], q int8 [k],
    bsums int16 [k/16])."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    k = x.size
    d = np.empty(k // 256, np.float32)
    q = np.empty(k, np.int8)
    bs = np.empty(k // 16, np.int16)
    lib().vxo_quantize_row_q8_K(_ptr(x), k, _ptr(d), _ptr(q), _ptr(bs))
    return d, q, bs


def dequantize_w(wtype: int, blocks: np.ndarray, k: int) -> np.ndarray:
    """One row of GGUF blocks (uint8) of type Q8_0 / Q4_K / Q6_K -> fp32."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1)
    y = np.empty(k, np.float32)
    lib().vxo_dequantize_row_w(wtype, _ptr(blocks), k, _ptr(y))
    return y


def qmatmul(wtype: int, w_blocks: np.ndarray, n: int, k: int, x: np.ndarray):
    """ggml_mul_mat(W, x) for a quantized W restated (vx_qmm.c).

    w_blocks: uint8 [n][row bytes] GGUF blocks; x: fp32 [rows][k].  Returns
    (y float64 [rows][n], mag float64 [rows][n], terms per output): the
    parity bound for an fp32 result is (terms + 4) * 2^-24 * mag.
    """
    w_blocks = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows = x.shape[0]
    assert x.shape[1] == k and k <= 16384 and w_blocks.size == n * qrow_bytes(wtype, k)
    y = np.empty((rows, n), np.float64)
    mag = np.empty((rows, n), np.float64)
    terms = lib().vxo_qmatmul(wtype, _ptr(w_blocks), n, k, _ptr(x), rows, _ptr(y), _ptr(mag))
    if terms < 0:
        raise ValueError(f"unsupported weight type {wtype}")
    return y, mag, int(terms)


def random_qblocks(wtype: int, n: int, k: int, rng: np.random.Generator, zero_mean: bool = False) -> np.ndarray:
    """Valid random GGUF blocks for an n x k weight (test input): random
    quants and sub-block scales, block scales drawn so that the dequantized
    weights are O(0.05).  Q4_K's random mins bias its weights positive;
    zero_mean=True draws Q4_K blocks with dmin = 7.5 d and each min equal to
    its scale (weights symmetric about 0, mean |w| ~ 1/sqrt(k)), which keeps
    the activations of a stack of such layers O(1)."""
    per, size = QBLOCK[wtype]
    nb = k // per
    blk = rng.integers(0, 256, size=(n, nb, size), dtype=np.uint8)
    def f16(a):
        return np.asarray(a, np.float16).view(np.uint16).view(np.uint8).reshape(a.shape + (2,))
    if wtype == Q8_0:
        blk[:, :, 0:2] = f16(rng.uniform(2e-4, 8e-4, (n, nb)))
        blk[:, :, 2:] = rng.integers(-127, 128, size=(n, nb, 32)).astype(np.int8).view(np.uint8)
    elif wtype == Q4_K and zero_mean:
        d = np.asarray(rng.uniform(0.5, 1.5, (n, nb)) / (126.0 * np.sqrt(k)), np.float16)
        blk[:, :, 0:2] = f16(d)
        blk[:, :, 2:4] = f16(d.astype(np.float32) * 7.5)
        sc = rng.integers(0, 64, size=(n, nb, 8)).astype(np.uint8)
        s = blk[:, :, 4:16]
        s[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
        s[..., 4:8] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
        s[..., 8:12] = (sc[..., 4:8] & 0xF) | ((sc[..., 4:8] & 0xF) << 4)
        blk[:, :, 4:16] = s
    elif wtype == Q4_K:
        blk[:, :, 0:2] = f16(rng.uniform(5e-4, 2e-3, (n, nb)))
        blk[:, :, 2:4] = f16(rng.uniform(1e-3, 4e-3, (n, nb)))
    else:
        blk[:, :, 192:208] = rng.integers(-128, 128, size=(n, nb, 16)).astype(np.int8).view(np.uint8)
        blk[:, :, 208:210] = f16(rng.uniform(2e-5, 6e-5, (n, nb)))
    return blk.reshape(n, nb * size)


def quantize_blocks(wtype: int, x: np.ndarray) -> np.ndarray:
    """Encodes fp32 rows x [n][k] as valid GGUF blocks of Q8_0 / Q4_K / Q6_K
    (test input: weights with a chosen distribution).  Q8_0 is ggml's rule;
    for the K-quants this is a plain absmax / min-max encoder of the block
    format (not ggml's search for the best scales): Q6_K scale per 16 values
    max|x| / 31, Q4_K scale and offset per 32 values from the min and max,
    the block's d / dmin = largest sub-block scale / 127 (Q6_K) or 63 (Q4_K)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n, k = x.shape
    if wtype == Q8_0:
        return np.stack([quantize_q8_0(x[i]) for i in range(n)]).reshape(n, -1)
    nb = k // 256
    xb = x.reshape(n, nb, 256).astype(np.float64)
    f16 = lambda a: np.asarray(a, np.float16)  # noqa: E731
    if wtype == Q6_K:
        sub = xb.reshape(n, nb, 16, 16)
        s = np.abs(sub).max(axis=3) / 31.0                      # [n, nb, 16]
        d = f16(s.max(axis=2) / 127.0)                          # [n, nb]
        df = d.astype(np.float64)
        sc = np.where(df[..., None] > 0, np.rint(s / np.where(df[..., None] > 0, df[..., None], 1)), 0)
        sc = np.clip(sc, -128, 127).astype(np.int8)
        step = df[..., None] * sc.astype(np.float64)            # [n, nb, 16]
        q = np.where(step[..., None] > 0, np.rint(sub / np.where(step[..., None] > 0, step[..., None], 1)), 0)
        q6 = (np.clip(q, -32, 31) + 32).astype(np.uint8).reshape(n, nb, 2, 4, 32)   # [half, g, l]
        low, high = q6 & 0xF, q6 >> 4
        ql = np.empty((n, nb, 2, 64), np.uint8)
        ql[..., 0:32] = low[:, :, :, 0] | (low[:, :, :, 2] << 4)
        ql[..., 32:64] = low[:, :, :, 1] | (low[:, :, :, 3] << 4)
        qh = (high[:, :, :, 0] | (high[:, :, :, 1] << 2) | (high[:, :, :, 2] << 4) | (high[:, :, :, 3] << 6))
        out = np.empty((n, nb, 210), np.uint8)
        out[..., 0:128] = ql.reshape(n, nb, 128)
        out[..., 128:192] = qh.astype(np.uint8).reshape(n, nb, 64)
        out[..., 192:208] = sc.view(np.uint8)
        out[..., 208:210] = d.view(np.uint16).view(np.uint8).reshape(n, nb, 2)
        return out.reshape(n, nb * 210)
    if wtype == Q4_K:
        sub = xb.reshape(n, nb, 8, 32)
        mn = np.minimum(sub.min(axis=3), 0.0)
        mx = sub.max(axis=3)
        scale = (mx - mn) / 15.0
        off = -mn
        d = f16(scale.max(axis=2) / 63.0)
        dmin = f16(off.max(axis=2) / 63.0)
        df, mf = d.astype(np.float64)[..., None], dmin.astype(np.float64)[..., None]
        sc = np.clip(np.where(df > 0, np.rint(scale / np.where(df > 0, df, 1)), 0), 0, 63).astype(np.uint8)
        m = np.clip(np.where(mf > 0, np.rint(off / np.where(mf > 0, mf, 1)), 0), 0, 63).astype(np.uint8)
        step = df * sc
        q = np.where(step[..., None] > 0,
                     np.rint((sub + (mf * m)[..., None]) / np.where(step[..., None] > 0, step[..., None], 1)), 0)
        q = np.clip(q, 0, 15).astype(np.uint8).reshape(n, nb, 4, 2, 32)
        qs = (q[:, :, :, 0] | (q[:, :, :, 1] << 4)).reshape(n, nb, 128)
        s = np.empty((n, nb, 12), np.uint8)
        s[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
        s[..., 4:8] = m[..., 0:4] | ((m[..., 4:8] >> 4) << 6)
        s[..., 8:12] = (sc[..., 4:8] & 0xF) | ((m[..., 4:8] & 0xF) << 4)
        out = np.empty((n, nb, 144), np.uint8)
        out[..., 0:2] = d.view(np.uint16).view(np.uint8).reshape(n, nb, 2)
        out[..., 2:4] = dmin.view(np.uint16).view(np.uint8).reshape(n, nb, 2)
        out[..., 4:16] = s
        out[..., 16:144] = qs
        return out.reshape(n, nb * 144)
    raise ValueError(f"unsupported weight type {wtype}")


def normal_qblocks(wtype: int, n: int, k: int, rng: np.random.Generator, sigma: float | None = None) -> np.ndarray:
    """GGUF blocks of an n x k weight drawn from N(0, sigma^2), sigma = 1/sqrt(k)
    by default (a projection that keeps activations O(1)), then quantized."""
    sigma = 1.0 / np.sqrt(k) if sigma is None else sigma
    return quantize_blocks(wtype, rng.normal(0.0, sigma, (n, k)).astype(np.float32))
