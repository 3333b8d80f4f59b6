"""Every kernel of libvxk.so compiles for sm_100a without register spills.

The kernels are written to keep their working set in registers; several run
at their launch bounds' register limit (the tcgen05 quantized product runs 16
warps at 128 registers a thread).  A build of that product that spilled 68
bytes to local memory gave wrong results when its launches ran back to back
behind programmatic dependent launch, while every launch on its own was
right, so a spill is treated as a build error here.  ptxas's own report
(-Xptxas -v) is read; no GPU is needed.
"""
from __future__ import annotations

import concurrent.futures
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
CSRC = ROOT / "voxtral.cpp_b200" / "csrc"
NVCC = next((p for p in ("/usr/local/cuda/bin/nvcc", shutil.which("nvcc")) if p and Path(p).exists()), None)


def _ptxas_report(src: Path, out_dir: Path) -> str:
    cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
           "-I", str(ROOT / "include"), "-I", str(CSRC), "-c", str(src), "-o", str(out_dir / (src.name + ".o")),
           "-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return res.stderr


@pytest.mark.skipif(NVCC is None, reason="nvcc not found")
def test_no_kernel_spills_registers(tmp_path):
    sources = sorted(CSRC.glob("*.cu"))
    assert sources
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(sources)) as ex:
        reports = dict(zip(sources, ex.map(lambda s: _ptxas_report(s, tmp_path), sources)))
    checked = 0
    spilled = []
    for src, text in reports.items():
        entry = None
        for line in text.splitlines():
            m = re.search(r"Compiling entry function '([^']+)'", line)
            if m:
                entry = m.group(1)
                continue
            m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
            if m and entry:
                checked += 1
                if int(m.group(1)) or int(m.group(2)):
                    spilled.append(f"{src.name}: {entry}: {line.strip()}")
                entry = None
    assert checked >= len(sources), "ptxas reported no kernels"
    assert not spilled, "\n".join(spilled)
