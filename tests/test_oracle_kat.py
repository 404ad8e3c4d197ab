"""Pins the CPU oracle to the reference's own known-answer tests
(src/kernels/simd.zig:500-806, src/kernels/math.zig:205-254) and to
gguf-py's independent dequantizers (tests/golden/kquant_golden.npz)."""
import os

import numpy as np
import pytest

import oracle as O
from vantablack_b200 import synth as S

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "kquant_golden.npz"))


def test_dot_i8_div16():  # simd.zig:502-513
    a = (np.arange(32) - 16).astype(np.int8)
    b = (np.arange(32) * 3 - 47).astype(np.int8)
    assert O.dot_i8(a, b) == int((a.astype(np.int32) * b.astype(np.int32)).sum())


def test_dot_i8_tail():  # simd.zig:515-525
    a = (np.arange(19) - 9).astype(np.int8)
    b = (np.arange(19) + 1).astype(np.int8)
    assert O.dot_i8(a, b) == int((a.astype(np.int32) * b.astype(np.int32)).sum())


def test_dot_i8_saturation():  # simd.zig:527-531
    a = np.full(32, -128, np.int8)
    assert O.dot_i8(a, a) == 524288


def test_dot_f32():  # simd.zig:533-543
    a = np.arange(1, 20, dtype=np.float32)
    b = a * 2
    exp = np.float32(0)
    for i in range(19):
        exp = np.float32(exp + a[i] * b[i])
    assert abs(O.dot_f32(a, b) - exp) <= 1e-4


@pytest.mark.parametrize("name,q", [("q8_0", S.Q8_0), ("q4_k", S.Q4_K), ("q5_k", S.Q5_K), ("q6_k", S.Q6_K)])
def test_dequant_bit_exact_vs_gguf(name, q):
    blocks = GOLD[f"{name}_blocks"]
    exp = GOLD[f"{name}_dequant"]
    got = O.dequant(q, blocks, exp.size)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


def test_q8_0_dequant_kat():  # simd.zig:586-599
    blk = GOLD["q8_0_blocks"][:34]
    qs = blk[2:].view(np.int8).astype(np.float32)
    assert np.allclose(O.dequant(S.Q8_0, blk, 32), np.float32(0.125) * qs, atol=1e-4)


def test_q4_k_kat_spots_and_matmul():  # simd.zig:601-651
    blk = GOLD["q4_k_blocks"][:144]
    dq = O.dequant(S.Q4_K, blk, 256)
    d, dmin = np.float32(0.0078125), np.float32(0.0625)
    e0 = d * np.float32(blk[4] & 63) * np.float32(blk[16] & 15) - dmin * np.float32(blk[8] & 63)
    e32 = d * np.float32(blk[5] & 63) * np.float32(blk[16] >> 4) - dmin * np.float32(blk[9] & 63)
    assert abs(dq[0] - e0) <= 1e-4 and abs(dq[32] - e32) <= 1e-4
    x = (np.arange(256) % 7).astype(np.float32) * np.float32(0.1)
    got = O.matmul_single(S.Q4_K, blk, x, 1, 256)[0]
    assert abs(got - float(np.dot(dq.astype(np.float64), x))) <= 1e-3


def test_q5_k_kat():  # simd.zig:653-697
    blk = GOLD["q5_k_blocks"][:176]
    dq = O.dequant(S.Q5_K, blk, 256)
    d, dmin = np.float32(0.00390625), np.float32(0.03125)
    w5 = (blk[48] & 15) + (16 if blk[16] & 1 else 0)
    e0 = d * np.float32(blk[4] & 63) * np.float32(w5) - dmin * np.float32(blk[8] & 63)
    assert abs(dq[0] - e0) <= 1e-4
    x = (np.arange(256) % 9).astype(np.float32) * np.float32(0.1) - np.float32(0.4)
    got = O.matmul_single(S.Q5_K, blk, x, 1, 256)[0]
    assert abs(got - float(np.dot(dq.astype(np.float64), x))) <= 1e-3


def test_q6_k_kat():  # simd.zig:699-732
    blk = GOLD["q6_k_blocks"][:210]
    dq = O.dequant(S.Q6_K, blk, 256)
    q1 = int((blk[0] & 15) | ((blk[128] & 3) << 4)) - 32
    e0 = np.float32(0.001953125) * np.float32(np.int8(blk[192].astype(np.int8))) * np.float32(q1)
    assert abs(dq[0] - e0) <= 1e-4
    x = (np.arange(256) % 11).astype(np.float32) * np.float32(0.05) - np.float32(0.25)
    got = O.matmul_single(S.Q6_K, blk, x, 1, 256)[0]
    assert abs(got - float(np.dot(dq.astype(np.float64), x))) <= 1e-3


def _tq2_kat_block():
    """simd.zig:735-746: scale 0.25; byte i packs (i%3, (i+1)%3, (i+2)%3, i%3)."""
    blk = np.zeros(66, np.uint8)
    blk[64:66] = np.array([0.25], np.float16).view(np.uint8)
    for i in range(64):
        blk[i] = (i % 3) | (((i + 1) % 3) << 2) | (((i + 2) % 3) << 4) | ((i % 3) << 6)
    return blk


def test_tq2_0_kat():  # simd.zig:734-768 ("TQ2_0 dequant + matmul self-consistent")
    blk = _tq2_kat_block()
    dq = O.dequant(S.TQ2_0, blk, 256)
    for g, idx in enumerate((0, 64, 128, 192)):  # spot checks at g*64 + l, l = idx - 64g
        l = idx - g * 64
        raw = (int(blk[g * 16 + (l % 16)]) >> (2 * g)) & 3
        assert abs(dq[idx] - 0.25 * (raw - 1)) <= 1e-5
    x = (np.arange(256) % 5).astype(np.float32) * np.float32(0.2) - np.float32(0.1)
    got = O.matmul_single(S.TQ2_0, blk, x, 1, 256)[0]
    assert abs(got - float((dq.astype(np.float64) * x).sum())) <= 1e-3
    # the reference's layout: weights l, l+16, l+32, l+48 of a group share one field
    assert np.array_equal(dq[0:16], dq[16:32]) and np.array_equal(dq[64:80], dq[112:128])


def test_tq2_0_threaded_matmul_equals_single():
    rng = np.random.default_rng(35)
    m, k = 37, 1024
    w = S.quant_tensor(rng, S.TQ2_0, m, k)
    x = S.activations(rng, k)
    assert np.array_equal(O.matmul(S.TQ2_0, w, x, m, k), O.matmul_single(S.TQ2_0, w, x, m, k))


def test_matmul_q8_0_kat():  # simd.zig:770-806
    got = O.matmul(S.Q8_0, GOLD["mm_q8_0_w"], GOLD["mm_q8_0_x"], 4, 64)
    assert np.allclose(got, GOLD["mm_q8_0_y"], atol=1e-3)


def test_math_kats():  # math.zig:205-254
    x = np.arange(1, 9, dtype=np.float32)
    ref = x / np.sqrt((x * x).sum() / 8)
    assert np.allclose(O.rms_norm(x, np.ones(8, np.float32), 0.0), ref, atol=1e-4)
    r = O.rope(np.array([1, 2, 3, 4], np.float32), 0, 10000.0)
    assert abs(r[0] - 1) < 1e-5 and abs(r[1] - 2) < 1e-5
    assert abs(O.softmax(np.array([0.5, 1.5, -0.5, 2.0], np.float32)).sum() - 1) < 1e-5
    g = O.geglu(np.array([-2.0, -0.5, 0.0, 0.5, 1.0, 2.0], np.float32), np.ones(6, np.float32))
    assert np.allclose(g, [-0.045402, -0.154286, 0.0, 0.345714, 0.841192, 1.954598], atol=1e-4)
    gg = np.array([0.5, -1.0, 2.0, 0.0], np.float32)
    u = np.array([1.0, 2.0, 0.5, 4.0], np.float32)
    assert np.allclose(O.swiglu(gg, u), gg / (1 + np.exp(-gg)) * u, atol=1e-5)
    assert O.argmax(np.array([0.1, 0.5, 1.5, 0.3], np.float32)) == 2


@pytest.mark.parametrize("q", [S.Q8_0, S.Q4_K, S.Q5_K, S.Q6_K])
def test_threaded_matmul_equals_single(q):
    rng = np.random.default_rng(q)
    m, k = 37, 512
    w = S.quant_tensor(rng, q, m, k)
    x = S.activations(rng, k)
    O.set_threads(4)
    a = O.matmul(q, w, x, m, k)
    O.set_threads(1)
    assert np.array_equal(a, O.matmul_single(q, w, x, m, k))
    W = O.dequant(q, w, m * k).reshape(m, k).astype(np.float64)
    assert np.abs(a - W @ x).max() <= 1e-4 * np.abs(W @ x).max()


def test_batched_matmul_matches_dot_f32():
    rng = np.random.default_rng(5)
    m, k, B = 9, 512, 3
    w = S.quant_tensor(rng, S.Q6_K, m, k)
    acts = S.activations(rng, B, k)
    out = O.matmul_batched(S.Q6_K, w, acts, m, k, B)
    W = O.dequant(S.Q6_K, w, m * k).reshape(m, k)
    for b in range(B):
        for i in range(m):
            assert out[b, i] == np.float32(O.dot_f32(W[i], acts[b]))


def test_q8_0_quantizer_rule():
    rng = np.random.default_rng(3)
    x = S.activations(rng, 256)
    x[32:64] = 0.0  # all-zero block: d = 0, q = 0
    qs, d = O.quantize_q8_0(x)
    xb = x.reshape(-1, 32)
    dd = (np.abs(xb).max(1) / np.float32(127)).astype(np.float32)
    assert np.array_equal(d, dd)
    with np.errstate(divide="ignore"):
        inv = np.where(dd != 0, np.float32(1) / dd, np.float32(0)).astype(np.float32)
    v = (xb * inv[:, None]).astype(np.float32)
    q = np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))  # round half away from zero
    assert np.array_equal(qs.reshape(-1, 32), q.astype(np.int8))
    assert np.abs(qs).max() <= 127


def test_sampler_greedy_kat():  # sampler.zig:113-119
    assert O.sample([0.1, 0.5, 2.0, 0.3, 1.2], 0.0, 0, 0.0, 0.7)[0] == 2


def test_sampler_deterministic_kat():  # sampler.zig:121-130 (same draw, same token)
    a = O.sample([1.0, 2.0, 3.0, 4.0, 5.0], 1.0, 0, 0.0, 0.42)[0]
    b = O.sample([1.0, 2.0, 3.0, 4.0, 5.0], 1.0, 0, 0.0, 0.42)[0]
    assert a == b


def test_sampler_top_k1_is_greedy_kat():  # sampler.zig:132-138, for any draw
    for u in (1e-7, 0.3, 0.999999):  # u = 0 would stop at index 0 (u <= acc = 0), as in the reference
        assert O.sample([0.1, 0.5, 2.0, 0.3, 1.2], 1.0, 1, 0.0, u)[0] == 2


def test_sampler_pipeline_by_hand():
    """Temperature, top-k ties, nucleus cut and the CDF walk against a float64
    restatement of sampler.zig:49-97 on a case whose boundaries are far from u."""
    logits = np.array([1.0, 3.0, 3.0, 0.5, 2.0, -1.0], np.float32)
    tok, p = O.sample(logits, 0.5, 4, 0.8, 0.7)
    z = logits.astype(np.float64) / 0.5
    thr = np.sort(z)[::-1][3]
    z[z < thr] = -np.inf
    q = np.exp(z - z.max()); q /= q.sum()
    order = sorted(range(6), key=lambda i: (-q[i], i))
    c = np.cumsum(q[order]); cut = int(np.argmax(c >= 0.8)) + 1
    for i in order[cut:]:
        q[i] = 0
    q /= q.sum()
    assert np.allclose(p, q, atol=1e-6)
    assert tok == int(np.argmax(np.cumsum(q) >= 0.7))


def _mlx_q4_nibbles_0_15():
    w0 = sum(i << (4 * i) for i in range(8))
    w1 = sum((i + 8) << (4 * i) for i in range(8))
    return np.frombuffer(np.array([w0, w1], "<u4").tobytes(), np.uint8)


def test_mlx_dequant_q4_kat():  # mlx.zig:339-367: scale 1, bias 0 recovers the nibbles
    w = _mlx_q4_nibbles_0_15()
    one, zero = np.array([0x00, 0x3C], np.uint8), np.array([0, 0], np.uint8)
    assert np.array_equal(O.mlx_dequant(w, one, zero, 1, 16, 4, 16, False)[0], np.arange(16, dtype=np.float32))


def test_mlx_matmul_q4_kat():  # mlx.zig:369-405
    w = _mlx_q4_nibbles_0_15()
    s, b = np.array([0x00, 0x38], np.uint8), np.array([0x00, 0x34], np.uint8)  # f16 0.5, 0.25
    assert abs(O.mlx_matmul(w, s, b, np.ones(16, np.float32), 1, 16, 4, 16, False)[0] - 64.0) <= 1e-4
    alt = np.where(np.arange(16) % 2 == 0, 1.0, -1.0).astype(np.float32)
    assert abs(O.mlx_matmul(w, s, b, alt, 1, 16, 4, 16, False)[0] + 4.0) <= 1e-4


def test_mlx_matmul_q8_kat():  # mlx.zig:407-434
    w = np.frombuffer(np.array([0x03020100, 0x07060504], "<u4").tobytes(), np.uint8)
    one, zero = np.array([0x00, 0x3C], np.uint8), np.array([0, 0], np.uint8)
    assert abs(O.mlx_matmul(w, one, zero, np.ones(8, np.float32), 1, 8, 8, 8, False)[0] - 28.0) <= 1e-4


def test_mlx_dispatch_q4_q8_agree_kat():  # mlx.zig:436-459
    one, zero = np.array([0x00, 0x3C], np.uint8), np.array([0, 0], np.uint8)
    w4 = np.frombuffer(np.array([sum(i << (4 * i) for i in range(8))], "<u4").tobytes(), np.uint8)
    w8 = np.arange(8, dtype=np.uint8)
    x = np.ones(8, np.float32)
    assert O.mlx_matmul(w4, one, zero, x, 1, 8, 4, 8, False)[0] == O.mlx_matmul(w8, one, zero, x, 1, 8, 8, 8, False)[0] == 28.0


def test_mlx_matmul_runtime_fixture():  # forward.zig:853-960: every nibble 3, f16 scale 0.5, bias 0.25, x = e0
    m, k = 4, 64
    w = np.full(m * k // 2, 0x33, np.uint8)
    s = np.tile(np.array([0x00, 0x38], np.uint8), m)
    b = np.tile(np.array([0x00, 0x34], np.uint8), m)
    x = np.zeros(k, np.float32); x[0] = 1.0
    assert np.array_equal(O.mlx_matmul(w, s, b, x, m, k, 4, 64, False), np.full(m, 1.75, np.float32))
    # bf16 variant (forward.zig:968-1040): scale bf16 0.5 = 0x3F00, bias bf16 -1.0 = 0xBF80 -> 3 * 0.5 - 1
    s16 = np.tile(np.array([0x00, 0x3F], np.uint8), m)
    b16 = np.tile(np.array([0x80, 0xBF], np.uint8), m)
    assert np.array_equal(O.mlx_matmul(w, s16, b16, x, m, k, 4, 64, True), np.full(m, 0.5, np.float32))


def test_mlx_unsupported_bits():
    with pytest.raises(ValueError):
        O.mlx_matmul(np.zeros(16, np.uint8), np.zeros(2, np.uint8), np.zeros(2, np.uint8), np.zeros(8, np.float32),
                     1, 8, 7, 8, False)


@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
@pytest.mark.parametrize("bf16", [False, True])
def test_mlx_oracle_vs_numpy(bits, bf16):
    """The C restatement of mlx.zig against an independent numpy unpacking of
    the same layout (u32 words, 32 // bits values low bits first, per-group
    f16/bf16 scale and bias): dequant bit-exact, matmul within 1e-5."""
    from vantablack_b200 import synth as S
    el = 32 // bits
    group = 64 if 64 % el == 0 else 32 * el  # a multiple of 32 / bits values
    rng = np.random.default_rng(bits * 2 + bf16)
    m, k = 7, 4 * group
    w, sc, bi = S.mlx_tensor(rng, m, k, bits, group, bf16)
    words = np.frombuffer(w.tobytes(), "<u4").reshape(m, k // el)
    shifts = (np.arange(el, dtype=np.uint32) * bits)
    q = ((words[:, :, None] >> shifts) & ((1 << bits) - 1)).reshape(m, k).astype(np.float32)
    def dec(b):
        h = np.frombuffer(b.tobytes(), "<u2").reshape(m, k // group)
        return (h.astype(np.uint32) << 16).view(np.float32) if bf16 else h.view(np.float16).astype(np.float32)
    s = np.repeat(dec(sc), group, axis=1)
    b = np.repeat(dec(bi), group, axis=1)
    want = q * s + b  # f32 multiply then add, as dequantRow does
    got = O.mlx_dequant(w, sc, bi, m, k, bits, group, bf16)
    assert np.array_equal(got.view(np.uint32), want.astype(np.float32).view(np.uint32))
    x = rng.standard_normal(k).astype(np.float32)
    y = O.mlx_matmul(w, sc, bi, x, m, k, bits, group, bf16)
    ref = want.astype(np.float64) @ x.astype(np.float64)
    assert np.abs(y - ref).max() <= 1e-5 * np.abs(ref).max()


def test_sampler_random_vs_float64():
    """Sampler.sample on random logits against a float64 restatement: the kept
    set and the token agree wherever rounding cannot decide them."""
    rng = np.random.default_rng(17)
    checked = 0
    for trial in range(40):
        n = int(rng.integers(50, 3000))
        lg = (rng.standard_normal(n) * rng.uniform(0.5, 4)).astype(np.float32)
        t = float(rng.uniform(0.3, 1.5))
        k = int(rng.integers(0, n)) if trial % 3 else 0
        p = float(rng.uniform(0.2, 0.99)) if trial % 2 else 0.0
        u = float(rng.random())
        tok, probs = O.sample(lg, t, k, p, u)
        z = lg.astype(np.float64) * np.float32(1 / np.float32(t))
        if 0 < k < n:
            z[z < np.sort(z)[::-1][k - 1]] = -np.inf
        q = np.exp(z - z.max()); q /= q.sum()
        if 0 < p < 1:
            order = sorted(range(n), key=lambda i: (-q[i], i))
            c = np.cumsum(q[order])
            if np.abs(c - p).min() < 1e-4:
                continue
            cut = int(np.argmax(c >= p)) + 1
            q[np.asarray(order[cut:], dtype=int)] = 0
            q /= q.sum()
        cdf = np.cumsum(q)
        if np.abs(cdf - u).min() < 1e-4:
            continue
        assert np.array_equal(probs > 0, q > 0)
        assert tok == int(np.argmax(cdf >= u))
        checked += 1
    assert checked >= 25
