"""Seeded synthetic GGUF-format weights and activations.

The bytes are generated once on the host (numpy PCG64) and uploaded
unchanged, so the CUDA backend and the CPU oracle read identical inputs.
Distributions (per block format):

* Q4_K (144 B / 256 weights): f16 d, dmin = f16(|N(0,1)| * 2^-7); the 12
  packed scale bytes and 128 nibble bytes uniform u8.
* Q5_K (176 B / 256): as Q4_K, with d, dmin = f16(|N(0,1)| * 2^-8) and the
  32 high-bit bytes uniform u8.
* Q6_K (210 B / 256): 128 B low nibbles and 64 B high 2-bit fields uniform
  u8; 16 i8 sub-block scales uniform in [-32, 31]; f16 d = f16(|N(0,1)| * 2^-9).
* Q8_0 (34 B / 32): f16 d = f16(|N(0,1)| * 2^-8); 32 i8 uniform in [-127, 127].
* TQ2_0 (66 B / 256, id 32 as in the reference's parser): 64 bytes of 2-bit
  fields, each field uniform in {0, 1, 2} (ternary -1/0/+1); f16 d =
  f16(|N(0,1)| * 2^-6).
* activations f32 ~ N(0, 1); norm weights 1 + 0.02 * N(0, 1).

Block layouts follow the ggml formats restated in the reference at
src/kernels/simd.zig:145-434.
"""
from __future__ import annotations

import numpy as np

F32, Q8_0, Q4_K, Q5_K, Q6_K, TQ2_0 = 0, 8, 12, 13, 14, 32

BLOCK_BYTES = {Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210, TQ2_0: 66}
BLOCK_ELEMS = {Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256, TQ2_0: 256}
NAMES = {Q8_0: "q8_0", Q4_K: "q4_k", Q5_K: "q5_k", Q6_K: "q6_k", TQ2_0: "tq2_0", F32: "f32"}


def row_bytes(quant: int, k: int) -> int:
    if quant == F32:
        return 4 * k
    if k % BLOCK_ELEMS[quant]:
        raise ValueError(f"k={k} is not a multiple of the {NAMES[quant]} block size")
    return (k // BLOCK_ELEMS[quant]) * BLOCK_BYTES[quant]


def _f16_bytes(rng: np.random.Generator, n: int, scale: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(n)) * scale).astype(np.float16).view(np.uint8).reshape(n, 2)


def quant_tensor(rng: np.random.Generator, quant: int, m: int, k: int) -> np.ndarray:
    """m rows of k weights in `quant` format, flat uint8 (row-major)."""
    nb = m * (k // BLOCK_ELEMS[quant])
    bb = BLOCK_BYTES[quant]
    blocks = np.frombuffer(rng.bytes(nb * bb), np.uint8).reshape(nb, bb).copy()
    if quant == Q4_K:
        blocks[:, 0:2] = _f16_bytes(rng, nb, 2.0 ** -7)
        blocks[:, 2:4] = _f16_bytes(rng, nb, 2.0 ** -7)
    elif quant == Q5_K:
        blocks[:, 0:2] = _f16_bytes(rng, nb, 2.0 ** -8)
        blocks[:, 2:4] = _f16_bytes(rng, nb, 2.0 ** -8)
    elif quant == Q6_K:
        blocks[:, 192:208] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8).view(np.uint8)
        blocks[:, 208:210] = _f16_bytes(rng, nb, 2.0 ** -9)
    elif quant == Q8_0:
        blocks[:, 0:2] = _f16_bytes(rng, nb, 2.0 ** -8)
        blocks[:, 2:34] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    elif quant == TQ2_0:
        f = rng.integers(0, 3, size=(nb, 64, 4), dtype=np.uint8)
        blocks[:, 0:64] = f[..., 0] | (f[..., 1] << 2) | (f[..., 2] << 4) | (f[..., 3] << 6)
        blocks[:, 64:66] = _f16_bytes(rng, nb, 2.0 ** -6)
    else:
        raise ValueError(f"unsupported quant {quant}")
    return blocks.reshape(-1)


def activations(rng: np.random.Generator, *shape: int) -> np.ndarray:
    return rng.standard_normal(shape, dtype=np.float32)


def norm_weight(rng: np.random.Generator, n: int) -> np.ndarray:
    return (1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32)


def mlx_tensor(rng, m: int, k: int, bits: int, group: int, bf16: bool):
    """Seeded MLX affine tensor (mlx.zig layout): uniform random u32 words
    (k / (32 / bits) per row), scales |N(0,1)| * 2^-6 and biases N(0,1) * 2^-4,
    stored as f16 or as bf16 (the top half of the f32).  Returns
    (weight bytes, scale bytes, bias bytes)."""
    words = rng.integers(0, 2**32, size=m * (k // (32 // bits)), dtype=np.uint64).astype("<u4")
    ng = m * (k // group)
    sc = np.abs(rng.standard_normal(ng)) * 2.0**-6
    bi = rng.standard_normal(ng) * 2.0**-4
    def enc(v):
        if bf16:
            return (v.astype(np.float32).view(np.uint32) >> 16).astype("<u2")
        return v.astype(np.float16).view("<u2")
    return (np.frombuffer(words.tobytes(), np.uint8).copy(), np.frombuffer(enc(sc).tobytes(), np.uint8).copy(),
            np.frombuffer(enc(bi).tobytes(), np.uint8).copy())
