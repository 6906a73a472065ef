"""Generate tests/golden/kquant_golden.npz: Q4_K / Q6_K blocks and their dequantised values
as computed by gguf-py (llama.cpp's own numpy restatement of ggml's dequantize_row_q4_K /
dequantize_row_q6_K), the third-party package the reference's arithmetic comes from.

Run in a container where `gguf` (pinned: 0.19.0) is importable:
    python tests/golden/gen_kquant_golden.py
The blocks are seeded random bytes with finite f16 scales, plus edge cases (zero scales,
subnormal and negative d, extreme 6-bit scales and int8 scales of -128).
"""
import os

import numpy as np

import gguf
from gguf.quants import Q4_K, Q6_K

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kquant_golden.npz")


def f16_bytes(values):
    return np.asarray(values, np.float16).view(np.uint8).reshape(-1, 2)


def q4k_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 144), dtype=np.uint8)
    d = rng.uniform(1e-4, 0.05, n)
    dmin = rng.uniform(1e-4, 0.05, n)
    d[0], dmin[0] = 0.0, 0.0            # all-zero scale
    d[1] = 6e-8                          # subnormal f16
    d[2], dmin[2] = -0.01, -0.02         # negative scales are representable
    b[3, 4:16] = 0xFF                    # every 6-bit scale and min at 63
    b[4, 4:16] = 0x00
    b[:, 0:2] = f16_bytes(d)
    b[:, 2:4] = f16_bytes(dmin)
    return b


def q6k_blocks(rng, n):
    b = rng.integers(0, 256, size=(n, 210), dtype=np.uint8)
    d = rng.uniform(-0.01, 0.01, n)
    d[0] = 0.0
    d[1] = 1e-7
    b[2, 192:208] = 0x80                 # int8 scales of -128
    b[3, 192:208] = 0x7F
    b[4, 0:192] = 0xFF                   # every 6-bit quant at 63
    b[:, 208:210] = f16_bytes(d)
    return b


def main():
    rng = np.random.default_rng(20261201)
    q4 = q4k_blocks(rng, 64)
    q6 = q6k_blocks(rng, 64)
    y4 = Q4_K.dequantize_blocks(q4.copy()).astype(np.float32).reshape(-1)
    y6 = Q6_K.dequantize_blocks(q6.copy()).astype(np.float32).reshape(-1)
    np.savez_compressed(OUT, q4k_bytes=q4, q4k_values=y4, q6k_bytes=q6, q6k_values=y6,
                        gguf_version=np.array(gguf.__version__ if hasattr(gguf, "__version__") else "0.19.0"))
    print(OUT, q4.shape, q6.shape)


if __name__ == "__main__":
    main()
