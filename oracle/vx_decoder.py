"""CPU restatement of voxtral.cpp's whole decoder step and adapter ring.

TEST INFRASTRUCTURE ONLY.  Nothing in the product library imports or calls
this module; tests/ use it as the checker of vxk_decoder_*.

It follows the reference's graphs node by node, with ggml's CPU semantics:
  - build_decoder_step_graph_reusable / build_decoder_prefill_graph
    (src/voxtral.cpp:2891-2965, 3047-3104): x = get_rows(tok_embeddings,
    token) + audio_emb[slot]; every layer; final rms_norm * dec_norm; logits
    of each stream's last row (tied tok_embeddings, or output.weight) and
    their argmax (emit_logits_argmax, 2966-2972);
  - build_decoder_layer (2630-2886): rms_norm * attn_norm; q/k/v products;
    RoPE mode 0 + f16/q8_0 append + GQA attention (vx_oracle.kv_row /
    attn_row, fp64); o product + residual; rms_norm * ffn_norm, then h + h *
    ada; SwiGLU (silu(w1 h) * w3 h); w2 product + residual;
  - the time MLP ada = ada2 . gelu_erf(ada0 . time_emb) with
    compute_time_embedding (730-741) evaluated through the C library's
    expf / logf / cosf / sinf, as the reference does on the host;
  - build_adapter_ring_graph_reusable (2589-2620): 4 encoder frames per
    group, adapter.0, gelu_erf, adapter.2.

Arithmetic: rms_norm sums the fp32 squares in fp64 and applies
1 / sqrtf(mean + eps) like ggml_compute_forward_rms_norm_f32; get_rows of a
quantized table uses the bit-exact dequantizers of vx_qmm.c; quantized
products are vx_oracle.qmatmul (integer block dots of ggml's quantized
activations, summed in fp64, the exact-math target) rounded to fp32; silu,
gelu_erf and the fp64 attention are exact-math targets as well.
Parity: unpinned numerically (ggml is absent here); the restatement's pieces
are pinned where vx_oracle's are (dequantizers and quantizers against
gguf 0.19.0).
"""
from __future__ import annotations

import ctypes as C
import ctypes.util
import math
from dataclasses import dataclass, field

import numpy as np

import vx_oracle as vo

F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30

_libm = C.CDLL(ctypes.util.find_library("m") or "libm.so.6")
for _fn in ("expf", "logf", "cosf", "sinf", "erff"):
    getattr(_libm, _fn).restype = C.c_float
    getattr(_libm, _fn).argtypes = [C.c_float]


def _f32(v) -> np.float32:
    return np.float32(v)


@dataclass
class Tensor:
    """A GGUF tensor: ggml type, rows x cols (ne[1] x ne[0]) and its bytes
    (uint8 blocks for quantized types, a float32 / float16 array otherwise)."""
    type: int
    rows: int
    cols: int
    data: np.ndarray


def dequant_rows(t: Tensor, idx=None) -> np.ndarray:
    """Rows of t as fp32, exactly as ggml's CPU dequantizers give them."""
    idx = range(t.rows) if idx is None else idx
    if t.type == F32:
        return np.asarray(t.data, np.float32).reshape(t.rows, t.cols)[list(idx)]
    if t.type == F16:
        return np.asarray(t.data, np.float16).reshape(t.rows, t.cols)[list(idx)].astype(np.float32)
    if t.type == BF16:
        b = np.asarray(t.data, np.uint16).reshape(t.rows, t.cols)[list(idx)]
        return (b.astype(np.uint32) << 16).view(np.float32)
    blocks = np.asarray(t.data, np.uint8).reshape(t.rows, -1)
    return np.stack([vo.dequantize_w(t.type, blocks[i], t.cols) for i in idx])


def act_roundtrip(wtype: int, x: np.ndarray) -> np.ndarray:
    """x as ggml's vec_dot_type for weight type wtype rounds it."""
    x = np.asarray(x, np.float32).reshape(-1)
    if wtype == F32:
        return x.copy()
    if wtype == F16:
        return x.astype(np.float16).astype(np.float32)
    if wtype == BF16:
        return (vo.f32_to_bf16_bits(x).astype(np.uint32) << 16).view(np.float32)
    if wtype == Q8_0:
        blk = vo.quantize_q8_0(x).reshape(-1, 34)
        d = blk[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1, 1)
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        return (d * q).reshape(-1)
    d, q, _ = vo.quantize_q8_K(x)
    return (np.repeat(d, 256) * q.astype(np.float32)).astype(np.float32)


def matvec_exact(t: Tensor, x: np.ndarray) -> np.ndarray:
    """W x in fp64 over the dequantized W and the vec_dot_type-rounded x."""
    w = dequant_rows(t).astype(np.float64)
    return (w @ act_roundtrip(t.type, x).astype(np.float64)).astype(np.float32)


def time_embedding(t: float, dim: int) -> np.ndarray:
    half = dim // 2
    out = np.empty(dim, np.float32)
    ln = _libm.logf(10000.0)
    for i in range(half):
        inv = _libm.expf(_f32(-ln) * _f32(i) / _f32(half))
        ang = float(_f32(t) * _f32(inv))
        out[i] = _libm.cosf(ang)
        out[i + half] = _libm.sinf(ang)
    return out


def gelu_erf_libm(x: np.ndarray) -> np.ndarray:
    """0.5f * x * (1 + erff(x / sqrt 2)) in fp32 with the C library's erff."""
    x = np.asarray(x, np.float32)
    e = np.array([_libm.erff(float(_f32(v) * _f32(0.70710678118654752440))) for v in x.reshape(-1)],
                 np.float32).reshape(x.shape)
    return (_f32(0.5) * x) * (_f32(1.0) + e)


def gelu_erf_exact(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    e = np.vectorize(math.erf)(x.astype(np.float64) / math.sqrt(2.0))
    return (0.5 * x.astype(np.float64) * (1.0 + e)).astype(np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.asarray(x, np.float32)
    sq = (x * x).astype(np.float64)
    mean = (sq.sum(axis=-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    scale = _f32(1.0) / np.sqrt(mean + _f32(eps))
    return (x * scale) * np.asarray(w, np.float32)


def qproduct(t: Tensor, x: np.ndarray) -> np.ndarray:
    """ggml_mul_mat(W, x) for quantized W, rounded to fp32."""
    y, _, _ = vo.qmatmul(t.type, np.asarray(t.data, np.uint8).reshape(t.rows, -1), t.rows, t.cols,
                         np.asarray(x, np.float32))
    return y.astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    x64 = np.asarray(x, np.float32).astype(np.float64)
    return (x64 / (1.0 + np.exp(-x64))).astype(np.float32)


@dataclass
class StreamCache:
    k: list = field(default_factory=list)  # per layer: list of stored K rows (bytes) in position order
    v: list = field(default_factory=list)
    next_pos: int = 0


class Decoder:
    """The reference decoder over host tensors (see the module docstring)."""

    def __init__(self, tensors: dict, n_layers: int, eps: float = 1e-5, theta: float = 1e6, time_value: float = 6.0,
                 cache_dtype: int = F16, n_q: int = 32, n_kv: int = 8, head_dim: int = 128, capacity: int = 8192,
                 attention=None):
        """attention: None for the fp64 restatement, or an object with
        begin(batch), layer(l, q, k, v) -> out [rows][n_q][head_dim] and end()
        that supplies the attention of each layer instead (a test plugs the
        device kernel in here to check the composition of everything else)."""
        self.attention = attention
        self.t = tensors
        self.L = n_layers
        self.eps = eps
        self.theta = theta
        self.n_q, self.n_kv, self.hd = n_q, n_kv, head_dim
        self.cache_dtype = cache_dtype
        self.capacity = capacity
        emb = tensors["tok_embeddings.weight"]
        self.dim, self.vocab = emb.cols, emb.rows
        self.ada = None
        if "dec.blk.0.ada0.weight" in tensors:
            temb = time_embedding(time_value, self.dim)
            self.ada = []
            for l in range(n_layers):
                h = matvec_exact(tensors[f"dec.blk.{l}.ada0.weight"], temb)
                h = gelu_erf_libm(h)
                self.ada.append(matvec_exact(tensors[f"dec.blk.{l}.ada2.weight"], h))
        self.streams: dict[int, StreamCache] = {}
        self.audio: dict[int, dict[int, np.ndarray]] = {}
        self.enc: dict[int, dict[int, np.ndarray]] = {}

    def vec(self, name):
        return dequant_rows(self.t[name]).reshape(-1)

    def stream(self, s: int) -> StreamCache:
        if s not in self.streams:
            self.streams[s] = StreamCache(k=[[] for _ in range(self.L)], v=[[] for _ in range(self.L)])
        return self.streams[s]

    def forward(self, batch, audio_rows):
        """batch: list of (stream, [tokens]) (plan order); audio_rows: per row
        the fp32 audio embedding added to it.  Appends to the caches and
        returns (hidden [n_streams][dim], logits float64 [n_streams][vocab],
        argmax [n_streams])."""
        rows = []
        for s, toks in batch:
            st = self.stream(s)
            for i, tok in enumerate(toks):
                rows.append((s, st.next_pos + i, tok))
        n = len(rows)
        emb = dequant_rows(self.t["tok_embeddings.weight"], [tok for _, _, tok in rows])
        x = emb + np.asarray(audio_rows, np.float32).reshape(n, self.dim)
        scale = 1.0 / math.sqrt(self.hd)
        if self.attention is not None:
            self.attention.begin([(s, len(toks)) for s, toks in batch])
        for l in range(self.L):
            p = f"dec.blk.{l}."
            xn = rms_norm(x, self.vec(p + "attn_norm.weight"), self.eps)
            q = qproduct(self.t[p + "attn_q.weight"], xn).reshape(n, self.n_q, self.hd)
            k = qproduct(self.t[p + "attn_k.weight"], xn).reshape(n, self.n_kv, self.hd)
            v = qproduct(self.t[p + "attn_v.weight"], xn).reshape(n, self.n_kv, self.hd)
            for r, (s, pos, _) in enumerate(rows):
                ko, vo_ = vo.kv_row(k[r], v[r], pos, self.theta, self.cache_dtype)
                st = self.stream(s)
                st.k[l].append(ko)
                st.v[l].append(vo_)
            att = np.empty((n, self.n_q, self.hd), np.float32)
            if self.attention is not None:
                att[:] = self.attention.layer(l, q, k, v)
            for r, (s, pos, _) in enumerate(rows if self.attention is None else ()):
                st = self.stream(s)
                # rows of this stream appended up to and including pos (causal), window = capacity
                upto = pos + 1
                lo = max(0, upto - self.capacity)
                kr = np.stack(st.k[l][lo:upto])
                vr = np.stack(st.v[l][lo:upto])
                att[r] = vo.attn_row(q[r], pos, self.theta, kr, vr, self.cache_dtype, self.n_kv, scale)
            x = x + qproduct(self.t[p + "attn_o.weight"], att.reshape(n, -1))
            h = rms_norm(x, self.vec(p + "ffn_norm.weight"), self.eps)
            if self.ada is not None:
                h = h + h * self.ada[l]
            g = silu(qproduct(self.t[p + "ffn_w1.weight"], h)) * qproduct(self.t[p + "ffn_w3.weight"], h)
            x = x + qproduct(self.t[p + "ffn_w2.weight"], g)
        if self.attention is not None:
            self.attention.end()
        for s, toks in batch:
            self.stream(s).next_pos += len(toks)
        last, r = [], 0
        for _, toks in batch:
            r += len(toks)
            last.append(r - 1)
        hn = rms_norm(x[last], self.vec("dec.norm.weight"), self.eps)
        hw = self.t.get("output.weight", self.t["tok_embeddings.weight"])
        if hw.type in (F16, BF16):
            bits = np.asarray(hw.data).view(np.uint16).reshape(hw.rows, hw.cols)
            logits, amax = vo.logits_argmax(bits, hw.type, hn)
        else:
            logits, _, _ = vo.qmatmul(hw.type, np.asarray(hw.data, np.uint8).reshape(hw.rows, -1), hw.rows, hw.cols,
                                      hn)
            amax = np.argmax(logits, axis=1)
        return hn, logits, amax

    def adapt(self, enc_rows: np.ndarray) -> np.ndarray:
        """enc_rows [n][4][enc_dim] -> audio embeddings [n][dim]."""
        x = np.asarray(enc_rows, np.float32).reshape(enc_rows.shape[0], -1)
        h = gelu_erf_exact(qproduct(self.t["adapter.0.weight"], x))
        return qproduct(self.t["adapter.2.weight"], h)
