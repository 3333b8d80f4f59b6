"""GGUF model files (vxk_gguf_*), CPU side.

The reader is checked against gguf 0.19.0, an independent implementation of
the published format: files written by gguf.GGUFWriter (metadata of every
value type, F32 / F16 / Q8_0 / Q4_K / Q6_K tensors, a non-default alignment)
must give the same keys, values, tensor names, types, shapes, data offsets
and bytes as gguf.GGUFReader; truncated and foreign files are refused with
an error instead of being read past their end.
"""
from __future__ import annotations

import numpy as np
import pytest

import vx_oracle as vo

gguf = pytest.importorskip("gguf")


def _write(path, alignment=None):
    rng = np.random.default_rng(3)
    w = gguf.GGUFWriter(str(path), "voxtral_realtime")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_uint32("voxtral.decoder.n_layers", 26)
    w.add_int32("voxtral.decoder.n_heads", 32)
    w.add_float32("voxtral.decoder.rope_theta", 1.0e6)
    w.add_bool("voxtral.encoder.causal", True)
    w.add_string("voxtral.note", "héllo")
    w.add_uint64("voxtral.big", 1 << 40)
    w.add_int8("voxtral.i8", -5)
    w.add_float64("voxtral.f64", 0.125)
    w.add_array("voxtral.tokenizer.special_token_ranks", [1, 2, 3, 70000])
    w.add_array("voxtral.strings", ["a", "bc", ""])
    tensors = {}
    f32 = rng.standard_normal((5, 3)).astype(np.float32)
    w.add_tensor("enc.norm.weight", f32)
    tensors["enc.norm.weight"] = (0, f32.tobytes())
    f16 = rng.standard_normal((64,)).astype(np.float16)
    w.add_tensor("dec.bias", f16)
    tensors["dec.bias"] = (1, f16.tobytes())
    for name, t, gt in (("dec.blk.0.attn_q.weight", 12, gguf.GGMLQuantizationType.Q4_K),
                        ("dec.blk.0.attn_v.weight", 14, gguf.GGMLQuantizationType.Q6_K),
                        ("adapter.0.weight", 8, gguf.GGMLQuantizationType.Q8_0)):
        blocks = vo.random_qblocks(t, 128, 512, rng)
        w.add_tensor(name, blocks, raw_dtype=gt)
        tensors[name] = (t, blocks.tobytes())
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return tensors


@pytest.mark.parametrize("alignment", [None, 64])
def test_reader_matches_gguf(vxk, tmp_path, alignment):
    path = tmp_path / "m.gguf"
    written = _write(path, alignment)
    ref = gguf.GGUFReader(str(path))
    g = vxk.Gguf(path)
    assert g.version == 3
    assert g.get("voxtral.decoder.n_layers") == 26
    assert g.get("voxtral.decoder.n_heads") == 32
    assert g.get("voxtral.decoder.rope_theta") == np.float32(1.0e6)
    assert g.get("voxtral.encoder.causal") is True
    assert g.get("voxtral.note") == "héllo"
    assert g.get("voxtral.big") == 1 << 40
    assert g.get("voxtral.i8") == -5
    assert g.get("voxtral.f64") == 0.125
    assert g.get("general.architecture") == "voxtral_realtime"
    np.testing.assert_array_equal(g.get("voxtral.tokenizer.special_token_ranks"), [1, 2, 3, 70000])
    assert g.get("voxtral.strings") == ["a", "bc", ""]
    # GGUFReader also lists the header as pseudo-fields "GGUF.*"
    assert set(g.keys()) == {k for k in ref.fields.keys() if not k.startswith("GGUF.")}
    with pytest.raises(KeyError):
        g.get("voxtral.absent")
    mine = {t["name"]: t for t in g.tensors()}
    assert [t["name"] for t in g.tensors()] == [t.name for t in ref.tensors]
    for rt in ref.tensors:
        t = mine[rt.name]
        assert t["type"] == int(rt.tensor_type)
        assert t["ne"] == [int(x) for x in rt.shape]
        assert t["offset"] == int(rt.data_offset)
        assert t["n_bytes"] == int(rt.n_bytes)
        assert g.tensor_bytes(rt.name).tobytes() == written[rt.name][1]
        if alignment:
            assert (t["offset"] - mine[ref.tensors[0].name]["offset"]) % alignment == 0
    assert g.find_tensor("absent") == -1
    g.close()


def test_refuses_truncated_and_foreign_files(vxk, tmp_path):
    path = tmp_path / "m.gguf"
    _write(path)
    data = path.read_bytes()
    for n in (3, 23, 64, len(data) // 2, len(data) - 1):
        bad = tmp_path / f"t{n}.gguf"
        bad.write_bytes(data[:n])
        with pytest.raises(vxk.VxkError):
            vxk.Gguf(bad)
    foreign = tmp_path / "f.bin"
    foreign.write_bytes(b"NOTGGUF" + bytes(100))
    with pytest.raises(vxk.VxkError):
        vxk.Gguf(foreign)
    with pytest.raises(vxk.VxkError):
        vxk.Gguf(tmp_path / "missing.gguf")


def test_refuses_a_tensor_offset_that_would_wrap(vxk, tmp_path):
    """A relative data offset near 2^64 (aligned) must be refused, not wrapped
    around into the header bytes."""
    path = tmp_path / "m.gguf"
    _write(path)
    r = gguf.GGUFReader(str(path))
    t = r.tensors[-1]
    at = int(t.field.offset) + sum(int(p.nbytes) for p in t.field.parts[:-1])
    data = bytearray(path.read_bytes())
    assert int.from_bytes(data[at:at + 8], "little") == int(t.data_offset) - int(r.data_offset)
    data[at:at + 8] = ((1 << 64) - 32).to_bytes(8, "little")
    bad = tmp_path / "wrap.gguf"
    bad.write_bytes(bytes(data))
    with pytest.raises(vxk.VxkError) as e:
        vxk.Gguf(bad)
    assert "runs past the file" in str(e.value)
