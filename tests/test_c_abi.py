"""The boundary from C and C++: include/vxk.h compiles on its own as C11 and as
C++17 (the reference compiles its public headers the same way,
tests/headers/public_header_smoke.c/.cpp), a C program linked against
libvxk.so runs the host-only entry points with the reference's own ring
planner expectations (tests/c/abi_host.c), and every struct of the ctypes
mirror (voxtral.cpp_b200/vxk.py) has the size and field offsets a C compiler
gives the header's struct.  No GPU is needed."""
from __future__ import annotations

import ctypes as C
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
INCLUDE = ROOT / "include"
LIBDIR = ROOT / "voxtral.cpp_b200"
CDIR = Path(__file__).resolve().parent / "c"

CC = shutil.which("gcc")
CXX = shutil.which("g++")

# ctypes mirror class -> C typedef of include/vxk.h
STRUCTS = {
    "DecoderKvRing": "vxk_decoder_kv_ring",
    "KvSeg": "vxk_kv_seg",
    "DecoderKvPlan": "vxk_decoder_kv_plan",
    "EncKvPlan": "vxk_enc_kv_plan",
    "PoolConfig": "vxk_pool_config",
    "PoolStats": "vxk_pool_stats",
    "EncConfig": "vxk_enc_config",
    "HeadConfig": "vxk_head_config",
    "QWeightConfig": "vxk_qweight_config",
    "GgufTensor": "vxk_gguf_tensor",
    "DecoderConfig": "vxk_decoder_config",
    "DecoderInfo": "vxk_decoder_info",
    "EncoderInfo": "vxk_encoder_info",
    "BatcherConfig": "vxk_batcher_config",
    "BatcherStats": "vxk_batcher_stats",
}


def _run(cmd, **kw):
    res = subprocess.run(cmd, capture_output=True, text=True, **kw)
    assert res.returncode == 0, f"{' '.join(map(str, cmd))}\n{res.stdout}\n{res.stderr}"
    return res.stdout


def _link(vxk):
    vxk.load()
    return ["-L", str(LIBDIR), "-l:libvxk.so", f"-Wl,-rpath,{LIBDIR}"]


@pytest.mark.skipif(CC is None, reason="no C compiler")
def test_header_compiles_as_c11(tmp_path):
    _run([CC, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(INCLUDE), "-c",
          str(CDIR / "header_smoke.c"), "-o", str(tmp_path / "smoke_c.o")])


@pytest.mark.skipif(CXX is None, reason="no C++ compiler")
def test_header_compiles_as_cpp17_with_c_linkage(tmp_path, vxk):
    exe = tmp_path / "smoke_cpp"
    _run([CXX, "-std=c++17", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(INCLUDE),
          str(CDIR / "header_smoke.cpp"), "-o", str(exe), *_link(vxk)])
    _run([str(exe)])


@pytest.mark.skipif(CC is None, reason="no C compiler")
def test_c_program_runs_host_calls(tmp_path, vxk):
    exe = tmp_path / "abi_host"
    _run([CC, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic", "-I", str(INCLUDE),
          str(CDIR / "abi_host.c"), "-o", str(exe), *_link(vxk)])
    out = _run([str(exe)], timeout=120)
    assert out.strip().startswith("ok "), out


@pytest.mark.skipif(CC is None, reason="no C compiler")
def test_ctypes_layouts_match_the_c_compiler(tmp_path, vxk):
    lines = ["#include <stddef.h>", "#include <stdio.h>", "#include <vxk.h>", "int main(void) {"]
    expect = {}
    for py_name, c_name in STRUCTS.items():
        cls = getattr(vxk, py_name)
        lines.append(f'    printf("{c_name} %zu\\n", sizeof({c_name}));')
        expect[c_name] = C.sizeof(cls)
        for field in cls._fields_:
            fname = field[0]
            lines.append(f'    printf("{c_name}.{fname} %zu\\n", offsetof({c_name}, {fname}));')
            expect[f"{c_name}.{fname}"] = getattr(cls, fname).offset
    lines += ["    return 0;", "}"]
    src = tmp_path / "layouts.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layouts"
    _run([CC, "-std=c11", "-Wall", "-Werror", "-I", str(INCLUDE), str(src), "-o", str(exe)])
    got = {}
    for line in _run([str(exe)]).splitlines():
        key, val = line.split()
        got[key] = int(val)
    assert got == expect
