"""Generates tests/golden/kquant_golden.npz.

Inputs: the block patterns of the reference's own known-answer tests
(src/kernels/simd.zig:586-806) plus seeded random blocks.  Expected
dequantized values come from gguf-py's numpy dequantizers (the `gguf`
package, ggml's own Python reimplementation of the same block formats) —
an implementation independent of both the reference and this repository.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np
import gguf.quants as gq
from gguf import GGMLQuantizationType as T

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))
from vantablack_b200 import synth as S  # noqa: E402


def f16b(v):
    return np.array([v], np.float16).view(np.uint8)


def kat_q8_0():  # simd.zig:586-599
    blk = np.zeros(34, np.uint8)
    blk[0:2] = f16b(0.125)
    qs = [-64, -32, -16, -8, -4, -2, -1, 0, 1, 2, 4, 8, 16, 32, 64, 100, -100, 50, -50, 25, -25, 12, -12, 6, -6,
          3, -3, 1, -1, 0, 0, 0]
    blk[2:] = np.array(qs, np.int8).view(np.uint8)
    return blk


def kat_q4_k():  # simd.zig:601-651
    blk = np.zeros(144, np.uint8)
    blk[0:2] = f16b(0.0078125)
    blk[2:4] = f16b(0.0625)
    for s in range(4):
        blk[4 + s] = (s + 1) * 5
        blk[8 + s] = s + 2
        blk[12 + s] = ((s + 1) * 3) | ((s + 1) << 4)
    for i in range(128):
        blk[16 + i] = ((i * 7) % 16) | (((i * 11) % 16) << 4)
    return blk


def kat_q5_k():  # simd.zig:653-697
    blk = np.zeros(176, np.uint8)
    blk[0:2] = f16b(0.00390625)
    blk[2:4] = f16b(0.03125)
    for s in range(4):
        blk[4 + s] = (s + 1) * 4
        blk[8 + s] = s + 1
        blk[12 + s] = ((s + 1) * 2) | ((s + 1) << 4)
    for l in range(32):
        blk[16 + l] = (l * 31) % 256
    for i in range(128):
        blk[48 + i] = ((i * 13) % 16) | (((i * 7) % 16) << 4)
    return blk


def kat_q6_k():  # simd.zig:699-732
    blk = np.zeros(210, np.uint8)
    blk[208:210] = f16b(0.001953125)
    for i in range(128):
        blk[i] = (i * 17) % 256
    for i in range(64):
        blk[128 + i] = (i * 19) % 256
    blk[192:208] = (np.arange(16) - 8).astype(np.int8).view(np.uint8)
    return blk


def main():
    rng = np.random.default_rng(20261201)
    out = {}
    for name, q, t, kat in [("q8_0", S.Q8_0, T.Q8_0, kat_q8_0), ("q4_k", S.Q4_K, T.Q4_K, kat_q4_k),
                            ("q5_k", S.Q5_K, T.Q5_K, kat_q5_k), ("q6_k", S.Q6_K, T.Q6_K, kat_q6_k)]:
        bb, el = S.BLOCK_BYTES[q], S.BLOCK_ELEMS[q]
        rand = S.quant_tensor(rng, q, 1, 8 * el)
        blocks = np.concatenate([kat(), rand]).reshape(-1, bb)
        deq = gq.dequantize(blocks, t).astype(np.float32).reshape(-1)
        out[f"{name}_blocks"] = blocks.reshape(-1)
        out[f"{name}_dequant"] = deq
    # matmul_q8_0 known-answer test weights (simd.zig:770-806): m=4, k=64.
    m, k = 4, 64
    w = np.zeros((m, 2, 34), np.uint8)
    for i in range(m):
        for b in range(2):
            w[i, b, 0:2] = f16b(0.0625 * (b + 1))
            w[i, b, 2:] = np.array([((i * 97 + b * 31 + j) % 17) - 8 for j in range(32)], np.int8).view(np.uint8)
    x = (np.arange(k) % 11).astype(np.float32) * np.float32(0.1) - np.float32(0.5)
    ref_w = gq.dequantize(w.reshape(-1, 34), T.Q8_0).reshape(m, k).astype(np.float64)
    out["mm_q8_0_w"] = w.reshape(-1)
    out["mm_q8_0_x"] = x
    out["mm_q8_0_y"] = (ref_w @ x.astype(np.float64)).astype(np.float32)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "kquant_golden.npz")
    np.savez_compressed(path, **out)
    print(path, {k_: v.shape for k_, v in out.items()})


if __name__ == "__main__":
    main()
