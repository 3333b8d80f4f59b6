"""Builds libvxk.so (the sm_100a kernel layer) in-tree.

nvcc cross-compiles for sm_100a without a GPU.  Objects go to _build/, the
shared library next to this file so it travels with the source tree.  Only the
vxk_* C-ABI symbols are exported (csrc/vxk.map); the CUDA runtime is linked
statically.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libvxk.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
          "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _compile(src: Path, verbose_ptxas: bool) -> Path:
    obj = BUILD / (src.name + ".o")
    hdrs = list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    newest = max([src.stat().st_mtime] + [h.stat().st_mtime for h in hdrs])
    if obj.exists() and obj.stat().st_mtime >= newest and not verbose_ptxas:
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu" and verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas and res.stderr:
        sys.stderr.write(res.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs),
               "-Xlinker", f"--version-script={CSRC / 'vxk.map'}", "-cudart", "static"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
