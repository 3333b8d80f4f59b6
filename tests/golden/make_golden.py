"""Generates the committed golden fixtures used to pin the oracle.

Run from the repository root:  python tests/golden/make_golden.py

Independent references used here (not the oracle):
  * q8_0: gguf 0.19.0 ``gguf.quants.Q8_0.quantize_blocks`` -- a third-party numpy
    restatement of ggml's quantize_row_q8_0_ref ("bit-exact same results as
    reference implementation in ggml-quants.c").
  * f16: numpy's float32 -> float16 cast (IEEE round-to-nearest-even).
  * bf16: explicit round-to-nearest-even on the float32 bit pattern in numpy.
The inputs are seeded; edge cases (ties, zeros, subnormals, saturation) are
appended by hand.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def q8_inputs() -> np.ndarray:
    rng = np.random.default_rng(20261201)
    rows = [rng.normal(0.0, 0.5, size=(64, 32)).astype(np.float32)]
    rows.append(rng.uniform(-3, 3, size=(16, 32)).astype(np.float32))
    special = np.zeros((8, 32), dtype=np.float32)
    special[1, :] = 1.0                                   # all equal
    special[2, :] = np.linspace(-127, 127, 32)            # exact integers, amax 127
    special[3, 0] = 127.0                                 # ties at x*id = k + 0.5
    special[3, 1:] = np.arange(1, 32) + 0.5
    special[4, :] = -np.arange(32, dtype=np.float32) / 31.0
    special[5, :] = 1e-8                                  # tiny values, d subnormal in f16
    special[6, ::2] = 65000.0                             # large (d near f16 range)
    special[6, 1::2] = -0.5
    special[7, :] = rng.normal(0, 1e-3, size=32)
    rows.append(special)
    return np.concatenate(rows, axis=0)


def make_q8() -> None:
    from gguf.quants import Q8_0  # third-party reference, only needed to regenerate

    x = q8_inputs()
    blocks = Q8_0.quantize_blocks(x.copy())
    np.savez_compressed(OUT / "q8_0_blocks.npz", x=x, blocks=blocks.astype(np.uint8))


def make_f16_bf16() -> None:
    rng = np.random.default_rng(7)
    vals = [rng.normal(0, 0.5, 4096), rng.normal(0, 100, 1024), rng.uniform(-1, 1, 1024) * 1e-5]
    # halfway cases between adjacent f16 values and around overflow / subnormal edges
    h = np.arange(0, 0x7BFF, 97, dtype=np.uint16).view(np.float16).astype(np.float32)
    h_next = (np.arange(0, 0x7BFF, 97, dtype=np.uint16) + 1).view(np.float16).astype(np.float32)
    vals.append((h + h_next) / 2)
    vals.append(np.array([65504.0, 65519.0, 65520.0, 70000.0, -65520.0, 2.0 ** -24, 2.0 ** -25,
                          1.5 * 2.0 ** -25, 2.0 ** -26, 0.0, -0.0, 6.1035156e-05, 6.0975552e-05]))
    x = np.concatenate([np.asarray(v, dtype=np.float32) for v in vals])
    f16 = x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    bf = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    np.savez_compressed(OUT / "f16_bf16.npz", x=x, f16=f16, bf16=bf)


if __name__ == "__main__":
    make_q8()
    make_f16_bf16()
    print("fixtures written to", OUT)
