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


def conv1d_causal_f16(x: np.ndarray, w: Tensor, b: np.ndarray, stride: int, pad_left: int, outputs) -> np.ndarray:
    """ggml_conv_1d after ggml_pad_ext (causal_conv1d_graph, src/voxtral.cpp:1767-1814)
    at the output positions `outputs`: im2col rounds x to f16 and the f16 dot
    product takes the weights as f16; sums in fp64, then + bias in fp32.
    x [in_ch][len] fp32, w: Tensor of ne [3, in, out] (rows = out, data [out][in][3])."""
    xin = np.asarray(x, np.float32).astype(np.float16).astype(np.float64)
    in_ch, length = xin.shape
    wf = np.asarray(w.data).reshape(-1, in_ch, 3).astype(np.float32).astype(np.float16).astype(np.float64)
    out = np.empty((len(outputs), wf.shape[0]), np.float32)
    for n, t in enumerate(outputs):
        cols = np.zeros((in_ch, 3))
        for k in range(3):
            j = stride * t + k - pad_left
            if 0 <= j < length:
                cols[:, k] = xin[:, j]
        out[n] = (np.einsum("oik,ik->o", wf, cols).astype(np.float32) + np.asarray(b, np.float32))
    return out


class Encoder:
    """The reference streaming encoder stack (build_encoder_steady_graph,
    src/voxtral.cpp:2386-2511) over host tensors: conv stem, layers with
    biases and RMS norms, final norm.  attention: None for the fp64
    restatement (vx_oracle.attn_row over the window), or an object like
    Decoder's that supplies each layer's attention."""

    def __init__(self, tensors: dict, n_layers: int, n_heads: int, head_dim: int = 64, eps: float = 1e-5,
                 theta: float = 1e6, cache_dtype: int = BF16, window: int = 750, attention=None):
        self.t, self.L, self.H, self.hd = tensors, n_layers, n_heads, head_dim
        self.eps, self.theta, self.dtype, self.window = eps, theta, cache_dtype, window
        self.attention = attention
        self.dim = tensors["enc.norm.weight"].cols
        self.hist: dict = {}

    def vec(self, name):
        return dequant_rows(self.t[name]).reshape(-1)

    def stem(self, mel_window: np.ndarray, n_new: int) -> np.ndarray:
        win = 2 * n_new + 4
        assert mel_window.shape[1] == win
        c0 = conv1d_causal_f16(mel_window, self.t["enc.conv0.weight"], self.vec("enc.conv0.bias"), 1, 2, range(win))
        y = gelu_erf_exact(c0).T  # [dim][win]
        c1 = conv1d_causal_f16(y, self.t["enc.conv1.weight"], self.vec("enc.conv1.bias"), 2, 1,
                               range(2, 2 + n_new))
        return gelu_erf_exact(c1)

    def forward(self, batch, x0=None):
        """batch: list of (stream, q_start, n_new, mel_window [n_mel][2 n + 4]).
        x0: None, or the stem output to start from (rows of dim).  Returns the
        final-normed rows [sum n_new][dim]."""
        x = np.concatenate([self.stem(m, n) for _, _, n, m in batch]) if x0 is None else np.asarray(x0, np.float32)
        rows = [(s, q0 + j) for s, q0, n, _ in batch for j in range(n)]
        n = len(rows)
        scale = float(np.float32(1.0 / math.sqrt(self.hd)))
        if self.attention is not None:
            self.attention.begin([(s, nn) for s, _, nn, _ in batch])
        for l in range(self.L):
            p = f"enc.blk.{l}."
            xn = rms_norm(x, self.vec(p + "attn_norm.weight"), self.eps)

            def proj(name, inp):
                y = qproduct(self.t[p + name + ".weight"], inp)
                if p + name + ".bias" in self.t:
                    y = y + self.vec(p + name + ".bias")
                return y
            q = proj("attn_q", xn).reshape(n, self.H, self.hd)
            k = proj("attn_k", xn).reshape(n, self.H, self.hd)
            v = proj("attn_v", xn).reshape(n, self.H, self.hd)
            for r, (s, pos) in enumerate(rows):
                self.hist[(s, l, pos)] = vo.kv_row(k[r], v[r], pos, self.theta, self.dtype)
            if self.attention is not None:
                att = self.attention.layer(l, q, k, v)
            else:
                att = np.empty((n, self.H, self.hd), np.float32)
                for r, (s, pos) in enumerate(rows):
                    lo = max(0, pos - self.window + 1)
                    kk = np.stack([self.hist[(s, l, a)][0] for a in range(lo, pos + 1)])
                    vv = np.stack([self.hist[(s, l, a)][1] for a in range(lo, pos + 1)])
                    att[r] = vo.attn_row(q[r], pos, self.theta, kk, vv, self.dtype, self.H, scale)
            x = x + proj("attn_o", att.reshape(n, -1))
            h = rms_norm(x, self.vec(p + "ffn_norm.weight"), self.eps)
            g = silu(qproduct(self.t[p + "ffn_w1.weight"], h)) * qproduct(self.t[p + "ffn_w3.weight"], h)
            x = x + proj("ffn_w2", g)
        if self.attention is not None:
            self.attention.end()
        return rms_norm(x, self.vec("enc.norm.weight"), self.eps)
