"""The C-ABI library loads and exports exactly the entry points include/vxk.h
declares (the drop-in boundary), and host-only calls behave without a GPU."""
from __future__ import annotations

import ctypes as C
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "vxk.h"
LIB = ROOT / "voxtral.cpp_b200" / "libvxk.so"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"VXK_API\s+[^;(]*?\b(vxk_\w+)\s*\(", text, flags=re.S))


def exported_symbols() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB)], capture_output=True, text=True, check=True).stdout
    syms = set()
    for line in out.splitlines():
        parts = line.split()
        if len(parts) >= 3 and parts[1] in ("T", "W"):
            syms.add(parts[2].split("@")[0])
    return syms


def test_header_declares_entry_points():
    decl = declared_symbols()
    assert len(decl) >= 40
    for name in ("vxk_decode_layer", "vxk_batch_plan", "vxk_pool_compact", "vxk_enc_layer",
                 "vxk_decoder_kv_plan_make", "vxk_enc_kv_plan_make"):
        assert name in decl


def test_library_exports_exactly_the_header(vxk):
    decl = declared_symbols()
    exp = exported_symbols()
    assert decl <= exp, f"missing: {sorted(decl - exp)}"
    extra = {s for s in exp - decl if s.startswith("vxk_")}
    assert not extra, f"undeclared exports: {sorted(extra)}"
    # nothing but the vxk_ C ABI leaks out of the shared object
    assert all(s.startswith("vxk_") for s in exp), sorted(s for s in exp if not s.startswith("vxk_"))[:10]


def test_binding_covers_every_symbol(vxk):
    assert set(vxk.SIGNATURES) == declared_symbols()


def test_status_strings_and_version(vxk):
    lib = vxk.load()
    assert lib.vxk_status_string(0) == b"ok"
    assert lib.vxk_status_string(9) == b"backend_error"
    assert lib.vxk_status_string(12) == b"timeout"
    assert lib.vxk_status_string(77) == b"unknown"
    assert lib.vxk_api_version() == 1


def test_default_configs(vxk):
    lib = vxk.load()
    c = lib.vxk_pool_default_config()
    assert (c.n_layers, c.n_q_heads, c.n_kv_heads, c.head_dim, c.block_tokens, c.capacity) == (26, 32, 8, 128, 16, 8192)
    assert c.dtype == vxk.DTYPE_F16 and c.rope_theta == pytest.approx(1e6)
    assert c.struct_size == C.sizeof(vxk.PoolConfig)
    e = lib.vxk_enc_default_config()
    assert (e.n_layers, e.n_heads, e.head_dim, e.window, e.capacity) == (32, 32, 64, 750, 878)
    assert e.struct_size == C.sizeof(vxk.EncConfig)
    h = lib.vxk_head_default_config()
    assert (h.dim, h.vocab, h.dtype) == (3072, 131072, vxk.DTYPE_F16)
    assert h.struct_size == C.sizeof(vxk.HeadConfig)


def test_head_create_rejects_bad_config_without_gpu(vxk):
    lib = vxk.load()
    h = C.c_void_p()
    for field, value in (("dim", 100), ("vocab", 0), ("dtype", 8), ("struct_size", 8)):
        c = lib.vxk_head_default_config()
        setattr(c, field, value)
        assert lib.vxk_head_create(C.byref(c), C.byref(h)) == vxk.INVALID_ARGUMENT, field
        assert not h.value
    assert lib.vxk_head_logits_argmax(None, None, None, 1, None, None, None) == vxk.INVALID_ARGUMENT
    lib.vxk_head_destroy(None)


def test_pool_create_rejects_bad_config_without_gpu(vxk):
    lib = vxk.load()
    c = lib.vxk_pool_default_config()
    c.head_dim = 64
    h = C.c_void_p()
    assert lib.vxk_pool_create(C.byref(c), C.byref(h)) == vxk.INVALID_ARGUMENT
    assert not h.value
    buf = C.create_string_buffer(256)
    lib.vxk_pool_last_error(None, buf, 256)
    assert b"head_dim" in buf.value
    c = lib.vxk_pool_default_config()
    c.capacity = 100   # not a multiple of the page size
    assert lib.vxk_pool_create(C.byref(c), C.byref(h)) == vxk.INVALID_ARGUMENT
    c = lib.vxk_pool_default_config()
    c.struct_size = 8
    assert lib.vxk_pool_create(C.byref(c), C.byref(h)) == vxk.INVALID_ARGUMENT


def test_null_handles_are_rejected(vxk):
    lib = vxk.load()
    assert lib.vxk_batch_commit(None) == vxk.INVALID_ARGUMENT
    assert lib.vxk_decode_layer(None, 0, None, None, None, None, None) == vxk.INVALID_ARGUMENT
    assert lib.vxk_enc_layer(None, 0, None, None, None, None, None) == vxk.INVALID_ARGUMENT
    assert lib.vxk_pool_probe_wait_timeout(None, 10, None) == vxk.INVALID_ARGUMENT
    lib.vxk_pool_destroy(None)
    lib.vxk_enc_destroy(None)


def test_product_does_not_link_the_oracle():
    out = subprocess.run(["nm", "-D", str(LIB)], capture_output=True, text=True, check=True).stdout
    assert "vxo_" not in out
    ldd = subprocess.run(["ldd", str(LIB)], capture_output=True, text=True).stdout
    assert "vxoracle" not in ldd
