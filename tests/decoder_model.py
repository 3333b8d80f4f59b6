"""Seeded synthetic decoder models written as GGUF files (test input).

The tensor names, shapes and keys are those voxtral.cpp's loader reads
(src/voxtral.cpp:1097-1110, 1225-1252); the weights are N(0, 1/cols) values
encoded as blocks of the requested ggml types (vx_oracle.normal_qblocks), so
the activations of the stack stay O(1) like a trained model's; norms near 1.  A Q4_K_M
file stores attn_v / ffn_w2 / tok_embeddings as Q6_K and the other
matrices as Q4_K (src/voxtral-quantize.cpp:146-158); `types` picks others.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

import vx_decoder as vd
import vx_oracle as vo

Q4_K_M = dict(q=vd.Q4_K, k=vd.Q4_K, v=vd.Q6_K, o=vd.Q4_K, w1=vd.Q4_K, w3=vd.Q4_K, w2=vd.Q6_K, emb=vd.Q6_K,
              ada0=vd.Q4_K, ada2=vd.F16, ad0=vd.Q4_K, ad2=vd.Q4_K)
Q8_0_ALL = dict(q=vd.Q8_0, k=vd.Q8_0, v=vd.Q8_0, o=vd.Q8_0, w1=vd.Q8_0, w3=vd.Q8_0, w2=vd.Q8_0, emb=vd.Q8_0,
                ada0=vd.Q8_0, ada2=vd.Q8_0, ad0=vd.Q8_0, ad2=vd.Q8_0)


def _matrix(rng, t, rows, cols):
    if t in (vd.Q8_0, vd.Q4_K, vd.Q6_K):
        return vd.Tensor(t, rows, cols, vo.normal_qblocks(t, rows, cols, rng))
    vals = rng.normal(0.0, 1.0 / np.sqrt(cols), (rows, cols)).astype(np.float32)
    if t == vd.F16:
        return vd.Tensor(t, rows, cols, vals.astype(np.float16))
    if t == vd.F32:
        return vd.Tensor(t, rows, cols, vals)
    raise ValueError(t)


def build(path: Path, seed: int, n_layers: int = 2, dim: int = 1024, hidden: int = 1024, vocab: int = 2048,
          ada_dim: int = 32, enc_dim: int = 256, types: dict = Q4_K_M, untied_f16_head: bool = False):
    """Writes the GGUF file and returns {name: vd.Tensor}."""
    import gguf

    rng = np.random.default_rng(seed)
    qdim, kvdim = 32 * 128, 8 * 128
    t: dict[str, vd.Tensor] = {}
    t["tok_embeddings.weight"] = _matrix(rng, types["emb"], vocab, dim)
    if untied_f16_head:
        t["output.weight"] = _matrix(rng, vd.F16, vocab, dim)
    for l in range(n_layers):
        p = f"dec.blk.{l}."
        t[p + "attn_q.weight"] = _matrix(rng, types["q"], qdim, dim)
        t[p + "attn_k.weight"] = _matrix(rng, types["k"], kvdim, dim)
        t[p + "attn_v.weight"] = _matrix(rng, types["v"], kvdim, dim)
        t[p + "attn_o.weight"] = _matrix(rng, types["o"], dim, qdim)
        t[p + "ffn_w1.weight"] = _matrix(rng, types["w1"], hidden, dim)
        t[p + "ffn_w3.weight"] = _matrix(rng, types["w3"], hidden, dim)
        t[p + "ffn_w2.weight"] = _matrix(rng, types["w2"], dim, hidden)
        t[p + "ada0.weight"] = _matrix(rng, types["ada0"], ada_dim, dim)
        t[p + "ada2.weight"] = _matrix(rng, types["ada2"], dim, ada_dim)
        t[p + "attn_norm.weight"] = vd.Tensor(vd.F32, 1, dim, rng.uniform(0.8, 1.2, dim).astype(np.float32))
        t[p + "ffn_norm.weight"] = vd.Tensor(vd.F32, 1, dim, rng.uniform(0.8, 1.2, dim).astype(np.float32))
    t["dec.norm.weight"] = vd.Tensor(vd.F32, 1, dim, rng.uniform(0.8, 1.2, dim).astype(np.float32))
    t["adapter.0.weight"] = _matrix(rng, types["ad0"], dim, 4 * enc_dim)
    t["adapter.2.weight"] = _matrix(rng, types["ad2"], dim, dim)

    w = gguf.GGUFWriter(str(path), "voxtral_realtime")
    w.add_int32("voxtral.decoder.dim", dim)
    w.add_int32("voxtral.decoder.n_layers", n_layers)
    w.add_int32("voxtral.decoder.n_heads", 32)
    w.add_int32("voxtral.decoder.head_dim", 128)
    w.add_int32("voxtral.decoder.hidden_dim", hidden)
    w.add_int32("voxtral.decoder.n_kv_heads", 8)
    w.add_float32("voxtral.decoder.norm_eps", 1e-5)
    w.add_float32("voxtral.decoder.rope_theta", 1e6)
    w.add_bool("voxtral.ada_rms_norm_t_cond", True)
    w.add_int32("voxtral.vocab_size", vocab)
    gtype = {vd.Q8_0: gguf.GGMLQuantizationType.Q8_0, vd.Q4_K: gguf.GGMLQuantizationType.Q4_K,
             vd.Q6_K: gguf.GGMLQuantizationType.Q6_K}
    for name, ten in t.items():
        if ten.type in gtype:
            w.add_tensor(name, np.asarray(ten.data, np.uint8).reshape(ten.rows, -1), raw_dtype=gtype[ten.type])
        elif ten.rows == 1:
            w.add_tensor(name, np.asarray(ten.data).reshape(-1))
        else:
            w.add_tensor(name, np.asarray(ten.data).reshape(ten.rows, ten.cols))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return t


def build_encoder(path: Path, seed: int, n_layers: int = 2, dim: int = 512, n_heads: int = 8, hidden: int = 1024,
                  n_mel: int = 128, types: dict = Q4_K_M):
    """A seeded streaming encoder (tensor names and keys of src/voxtral.cpp:1085-1095,
    1190-1222) written as a GGUF file; returns {name: vd.Tensor}."""
    import gguf

    rng = np.random.default_rng(seed)
    qdim = n_heads * 64
    t: dict[str, vd.Tensor] = {}

    def conv(name, out_ch, in_ch):
        w = rng.normal(0.0, 1.0 / np.sqrt(3 * in_ch), (out_ch, in_ch, 3)).astype(np.float16)
        t[name] = vd.Tensor(vd.F16, out_ch, in_ch * 3, w)

    def vec(name, n, lo=-0.1, hi=0.1):
        t[name] = vd.Tensor(vd.F32, 1, n, rng.uniform(lo, hi, n).astype(np.float32))

    conv("enc.conv0.weight", dim, n_mel)
    vec("enc.conv0.bias", dim)
    conv("enc.conv1.weight", dim, dim)
    vec("enc.conv1.bias", dim)
    for l in range(n_layers):
        p = f"enc.blk.{l}."
        t[p + "attn_q.weight"] = _matrix(rng, types["q"], qdim, dim)
        t[p + "attn_k.weight"] = _matrix(rng, types["k"], qdim, dim)
        t[p + "attn_v.weight"] = _matrix(rng, types["v"], qdim, dim)
        t[p + "attn_o.weight"] = _matrix(rng, types["o"], dim, qdim)
        t[p + "ffn_w1.weight"] = _matrix(rng, types["w1"], hidden, dim)
        t[p + "ffn_w3.weight"] = _matrix(rng, types["w3"], hidden, dim)
        t[p + "ffn_w2.weight"] = _matrix(rng, types["w2"], dim, hidden)
        vec(p + "attn_q.bias", qdim)
        vec(p + "attn_v.bias", qdim)
        vec(p + "attn_o.bias", dim)
        vec(p + "ffn_w2.bias", dim)
        vec(p + "attn_norm.weight", dim, 0.8, 1.2)
        vec(p + "ffn_norm.weight", dim, 0.8, 1.2)
    vec("enc.norm.weight", dim, 0.8, 1.2)

    w = gguf.GGUFWriter(str(path), "voxtral_realtime")
    for key, val in (("dim", dim), ("n_layers", n_layers), ("n_heads", n_heads), ("head_dim", 64),
                     ("hidden_dim", hidden), ("n_kv_heads", n_heads)):
        w.add_int32(f"voxtral.encoder.{key}", val)
    w.add_float32("voxtral.encoder.norm_eps", 1e-5)
    w.add_float32("voxtral.encoder.rope_theta", 1e6)
    gtype = {vd.Q8_0: gguf.GGMLQuantizationType.Q8_0, vd.Q4_K: gguf.GGMLQuantizationType.Q4_K,
             vd.Q6_K: gguf.GGMLQuantizationType.Q6_K}
    for name, ten in t.items():
        if ten.type in gtype:
            w.add_tensor(name, np.asarray(ten.data, np.uint8).reshape(ten.rows, -1), raw_dtype=gtype[ten.type])
        else:
            w.add_tensor(name, np.asarray(ten.data))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return t


def mel_window(mel: np.ndarray, q0: int, n: int) -> np.ndarray:
    """The conv stem's input for encoder rows q0 .. q0 + n - 1 of one stream:
    mel frames 2 (q0 - 2) .. 2 (q0 + n) - 1, channel-major, zeros before frame 0."""
    win = 2 * n + 4
    out = np.zeros((mel.shape[0], win), np.float32)
    f0 = 2 * (q0 - 2)
    for i in range(win):
        if f0 + i >= 0:
            out[:, i] = mel[:, f0 + i]
    return out
