"""GPU parity of the decode GEMV, dequantizer and Q8_0 x Q8_0 path against
the CPU oracle, through the C ABI.  Tolerances (north star): dequantized
values and int32 block dots bit-exact; fp32 GEMV outputs
max|y - y_ref| / max|y_ref| <= 1e-4."""
import numpy as np
import pytest
import torch

import oracle as O
from vantablack_b200 import synth as S

pytestmark = pytest.mark.gpu
TOL = 1e-4
O.set_threads(8)


def ops():
    from vantablack_b200 import ops as _ops
    return _ops


def rel_err(got, ref):
    return float(np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("q", [S.Q8_0, S.Q4_K, S.Q5_K, S.Q6_K, S.TQ2_0])
def test_dequant_bit_exact(q):
    rng = np.random.default_rng(100 + q)
    m, k = 33, 2048
    w = S.quant_tensor(rng, q, m, k)
    got = ops().dequant(q, torch.from_numpy(w).cuda(), m * k).cpu().numpy()
    exp = O.dequant(q, w, m * k)
    assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))


GEMV_SHAPES = [
    (S.Q4_K, 5632, 2048),   # TinyLlama ffn_up (the headline GEMV shape)
    (S.Q4_K, 1024, 4096), (S.Q4_K, 14336, 4096),
    (S.Q6_K, 4096, 4096), (S.Q6_K, 4096, 14336), (S.Q6_K, 2048, 5632),  # ragged Q6_K rows (4620 B)
    (S.Q8_0, 4096, 4096), (S.Q8_0, 14336, 4096), (S.Q8_0, 4096, 14336),
    (S.Q5_K, 4096, 4096), (S.Q5_K, 1000, 2304),
    (S.Q4_K, 1, 256), (S.Q6_K, 3, 256), (S.Q8_0, 5, 32), (S.Q4_K, 7, 2560),  # tiny / ragged tails
    (S.Q4_K, 4111, 4608), (S.Q4_K, 96, 24576),  # ragged last 32-row tile at size; long-K fallback
    (S.Q4_K, 6144, 4096), (S.Q4_K, 1000, 2048),  # 16-row tiles (large and small launch variants)
    (S.Q6_K, 1000, 6144), (S.Q6_K, 17, 2048),  # Q6_K tensor-core path: ragged last 16-row tile
    (S.TQ2_0, 4096, 4096), (S.TQ2_0, 14336, 4096), (S.TQ2_0, 1000, 2304), (S.TQ2_0, 3, 256),  # 594 B rows: ragged
]


@pytest.mark.parametrize("q,m,k", GEMV_SHAPES)
def test_gemv_matches_oracle(q, m, k):
    rng = np.random.default_rng(m * 7 + k + q)
    w = S.quant_tensor(rng, q, m, k)
    x = S.activations(rng, k)
    y = ops().gemv(q, torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(), m, k).cpu().numpy()
    ops().check_device_error()
    ref = O.matmul(q, w, x, m, k)
    assert rel_err(y, ref) <= TOL


def test_gemv_pdl_chain_matches():
    """Back-to-back PDL launches where each GEMV reads the previous output."""
    rng = np.random.default_rng(11)
    k = 2048
    ws = [S.quant_tensor(rng, S.Q4_K, k, k) for _ in range(3)]
    x = S.activations(rng, k)
    dws = [torch.from_numpy(w).cuda() for w in ws]
    cur = torch.from_numpy(x).cuda()
    for dw in dws:
        cur = ops().gemv(S.Q4_K, dw, cur, k, k, pdl=True)
    got = cur.cpu().numpy()
    ref = x
    for w in ws:
        ref = O.matmul(S.Q4_K, w, ref, k, k)
    assert rel_err(got, ref) <= 1e-3  # three chained roundings


def test_q8_0_quantizer_and_block_dots_bit_exact():
    rng = np.random.default_rng(21)
    m, k = 257, 4096
    w = S.quant_tensor(rng, S.Q8_0, m, k)
    x = S.activations(rng, k)
    x[64:96] = 0.0
    qs, d = ops().quantize_q8_0(torch.from_numpy(x).cuda())
    eqs, ed = O.quantize_q8_0(x)
    assert np.array_equal(qs.cpu().numpy(), eqs)
    assert np.array_equal(d.cpu().numpy().view(np.uint32), ed.view(np.uint32))
    dots = ops().q8_0_block_dots(torch.from_numpy(w).cuda(), qs, m, k).cpu().numpy()
    assert np.array_equal(dots, O.q8_0_block_dots(w, eqs, m, k))


@pytest.mark.parametrize("m,k", [(4096, 4096), (14336, 4096), (333, 1024)])
def test_gemv_q8_0_q8_0_matches_oracle(m, k):
    rng = np.random.default_rng(m + k)
    w = S.quant_tensor(rng, S.Q8_0, m, k)
    x = S.activations(rng, k)
    y = ops().gemv_q8_0_q8_0(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(), m, k).cpu().numpy()
    assert rel_err(y, O.matmul_q8_0_q8_0(w, x, m, k)) <= TOL


@pytest.mark.parametrize("q", [S.Q4_K, S.TQ2_0])
def test_embed_rows_bit_exact(q):
    rng = np.random.default_rng(4)
    vocab, dim = 100, 2048
    t = S.quant_tensor(rng, q, vocab, dim)
    ids = np.array([0, 99, 3, 3, 57], np.int32)
    got = ops().embed(q, torch.from_numpy(t).cuda(), torch.from_numpy(ids).cuda(), dim).cpu().numpy()
    rb = S.row_bytes(q, dim)
    for i, r in enumerate(ids):
        exp = O.dequant(q, t[r * rb:(r + 1) * rb], dim)
        assert np.array_equal(got[i].view(np.uint32), exp.view(np.uint32))


def test_tq2_0_reference_kat_on_gpu():
    """The reference's TQ2_0 known-answer block (simd.zig:734-768) through the
    GPU dequantizer and GEMV."""
    blk = np.zeros(66, np.uint8)
    blk[64:66] = np.array([0.25], np.float16).view(np.uint8)
    for i in range(64):
        blk[i] = (i % 3) | (((i + 1) % 3) << 2) | (((i + 2) % 3) << 4) | ((i % 3) << 6)
    dq = ops().dequant(S.TQ2_0, torch.from_numpy(blk).cuda(), 256).cpu().numpy()
    assert np.array_equal(dq.view(np.uint32), O.dequant(S.TQ2_0, blk, 256).view(np.uint32))
    x = (np.arange(256) % 5).astype(np.float32) * np.float32(0.2) - np.float32(0.1)
    y = ops().gemv(S.TQ2_0, torch.from_numpy(blk).cuda(), torch.from_numpy(x).cuda(), 1, 256).cpu().numpy()
    assert abs(float(y[0]) - float((dq.astype(np.float64) * x).sum())) <= 1e-3


def test_context_bridge_matmul():
    """The Metal-bridge-shaped API: upload, one-shot matmul at an offset, copy back."""
    import ctypes
    from vantablack_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(8)
    m, k = 300, 4096
    w = S.quant_tensor(rng, S.Q6_K, m, k)
    blob = np.concatenate([np.zeros(64, np.uint8), w])  # tensor at offset 64 inside a weight blob
    x = S.activations(rng, k)
    ctx = lib.vtb_cuda_init(0)
    assert ctx
    wb = lib.vtb_cuda_upload(ctx, blob.ctypes.data, blob.nbytes)
    xb = lib.vtb_cuda_upload(ctx, x.ctypes.data, x.nbytes)
    yb = lib.vtb_cuda_alloc(ctx, m * 4, None)
    assert wb and xb and yb
    _lib.check(lib.vtb_cuda_matmul_q6_k(ctx, yb, wb, 64, xb, m, k), "matmul")
    y = np.empty(m, np.float32)
    _lib.check(lib.vtb_cuda_copy_d2h(ctx, y.ctypes.data, yb, 0, m * 4), "d2h")
    assert rel_err(y, O.matmul(S.Q6_K, w, x, m, k)) <= TOL
    assert lib.vtb_cuda_matmul_q6_k(ctx, yb, wb, 64, xb, m + 1, k) == -1  # beyond the buffer
    for b in (wb, xb, yb):
        lib.vtb_cuda_release(b)
    lib.vtb_cuda_destroy(ctx)


def test_context_bridge_chained_matmuls():
    """Context matmuls queued back to back: each output buffer feeds the next
    matmul and the last one overwrites the chain's input buffer.  Each result
    must match the oracle applied to the device's own previous output."""
    from vantablack_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(9)
    n = 2048
    steps = [(S.Q4_K, lib.vtb_cuda_matmul_q4_k), (S.Q6_K, lib.vtb_cuda_matmul_q6_k), (S.Q5_K, lib.vtb_cuda_matmul_q5_k)]
    ws = [S.quant_tensor(rng, q, n, n) for q, _ in steps]
    x = S.activations(rng, n)
    ctx = lib.vtb_cuda_init(0)
    wb = [lib.vtb_cuda_upload(ctx, w.ctypes.data, w.nbytes) for w in ws]
    bufs = [lib.vtb_cuda_upload(ctx, x.ctypes.data, x.nbytes), lib.vtb_cuda_alloc(ctx, n * 4, None),
            lib.vtb_cuda_alloc(ctx, n * 4, None)]
    chain = [(0, 1), (1, 2), (2, 0)]  # (input buffer, output buffer) per step
    for (q, fn), b, (i, o) in zip(steps, wb, chain):
        _lib.check(fn(ctx, bufs[o], b, 0, bufs[i], n, n), "matmul")
    got = [np.empty(n, np.float32) for _ in range(3)]
    for y, o in zip(got, (1, 2, 0)):  # asynchronous read-back, visible after one wait
        _lib.check(lib.vtb_cuda_copy_d2h_async(ctx, y.ctypes.data, bufs[o], 0, n * 4), "d2h_async")
    _lib.check(lib.vtb_cuda_wait_idle(ctx), "wait_idle")
    inputs = [x, got[0], got[1]]
    for (q, _), w, xin, y in zip(steps, ws, inputs, got):
        assert rel_err(y, O.matmul(q, w, xin, n, n)) <= TOL, S.NAMES[q]
    for b in wb + bufs:
        lib.vtb_cuda_release(b)
    lib.vtb_cuda_destroy(ctx)


@pytest.mark.parametrize("q", [S.Q4_K, S.Q6_K, S.Q8_0, S.Q5_K, S.TQ2_0])
@pytest.mark.parametrize("kind", ["huge", "tiny", "outliers", "zeros"])
def test_gemv_activation_ranges(q, kind):
    """Activation magnitudes far from N(0,1): per-sub-block scaling must hold
    the 1e-4 bound (huge/tiny values, one outlier per block, zero blocks)."""
    rng = np.random.default_rng(77)
    m, k = 512, 4096
    w = S.quant_tensor(rng, q, m, k)
    x = S.activations(rng, k)
    if kind == "huge":
        x *= np.float32(3e4)
    elif kind == "tiny":
        x *= np.float32(1e-6)
    elif kind == "outliers":
        x[::32] *= np.float32(1000.0)
    else:
        x[: k // 2] = 0.0
    y = ops().gemv(q, torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(), m, k).cpu().numpy()
    assert rel_err(y, O.matmul(q, w, x, m, k)) <= TOL


def test_segment_graph_matches_one_shot():
    """Segments (vtb_metal_segment_* counterpart, bridge.h:72-183): a chain of
    matmuls of every K-quant plus a device copy, with host input and read-back
    inside the segment, equals the same one-shot calls bit for bit; committing
    the same list again replays the cached graph with new host data; a bad
    argument is reported by commit."""
    import torch
    from vantablack_b200 import _lib
    lib = _lib.load()
    rng = np.random.default_rng(21)
    n = 2048
    quants = [(S.Q4_K, "q4_k"), (S.Q6_K, "q6_k"), (S.Q5_K, "q5_k"), (S.Q8_0, "q8_0")]
    ws = [S.quant_tensor(rng, q, n, n) for q, _ in quants]
    ctx = lib.vtb_cuda_init(0)
    wb = [lib.vtb_cuda_upload(ctx, w.ctypes.data, w.nbytes) for w in ws]
    bufs = [lib.vtb_cuda_alloc(ctx, n * 4, None) for _ in range(5)]
    hx = torch.empty(n, dtype=torch.float32).pin_memory()
    hy = torch.empty(len(quants) + 2, n, dtype=torch.float32).pin_memory()

    def one_shot(x):
        _lib.check(lib.vtb_cuda_copy_h2d(ctx, bufs[0], 0, x.ctypes.data, n * 4), "h2d")
        for i, (q, name) in enumerate(quants):
            _lib.check(getattr(lib, f"vtb_cuda_matmul_{name}")(ctx, bufs[i + 1], wb[i], 0, bufs[i], n, n), "mm")
        out = [np.empty(n, np.float32) for _ in range(len(quants))]
        for i, y in enumerate(out):
            _lib.check(lib.vtb_cuda_copy_d2h(ctx, y.ctypes.data, bufs[i + 1], 0, n * 4), "d2h")
        return out

    def segment(x):
        hx.copy_(torch.from_numpy(x))
        seg = lib.vtb_cuda_segment_begin(ctx)
        assert seg
        lib.vtb_cuda_segment_copy_h2d(seg, bufs[0], 0, hx.data_ptr(), n * 4)
        # read back before a later copy of the same segment overwrites bufs[0]
        lib.vtb_cuda_segment_copy_d2h(seg, hy[len(quants) + 1].data_ptr(), bufs[0], 0, n * 4)
        for i, (q, name) in enumerate(quants):
            getattr(lib, f"vtb_cuda_segment_matmul_{name}")(seg, bufs[i + 1], wb[i], 0, bufs[i], n, n)
            lib.vtb_cuda_segment_copy_d2h(seg, hy[i].data_ptr(), bufs[i + 1], 0, n * 4)
        lib.vtb_cuda_segment_copy(seg, bufs[0], 0, bufs[2], 0, n)  # overwrites the chain's input
        lib.vtb_cuda_segment_copy_d2h(seg, hy[len(quants)].data_ptr(), bufs[0], 0, n * 4)
        _lib.check(lib.vtb_cuda_segment_commit(seg), "commit")
        _lib.check(lib.vtb_cuda_wait_idle(ctx), "wait")
        return [hy[i].numpy().copy() for i in range(len(quants) + 2)]

    for trial in range(3):  # the second and third commits replay the cached graph
        x = S.activations(rng, n)
        ref = one_shot(x)
        got = segment(x)
        for a, b in zip(ref, got):
            assert np.array_equal(a, b)
        assert np.array_equal(got[len(quants)], ref[1])
        assert np.array_equal(got[len(quants) + 1], x)
        assert rel_err(ref[0], O.matmul(S.Q4_K, ws[0], x, n, n)) <= TOL
    seg = lib.vtb_cuda_segment_begin(ctx)
    lib.vtb_cuda_segment_matmul_q4_k(seg, bufs[1], wb[0], 0, bufs[0], n + 1, n)  # beyond the weights
    assert lib.vtb_cuda_segment_commit(seg) == -1
    assert lib.vtb_cuda_segment_commit(seg) == -1  # nothing open any more
    _lib.check(lib.vtb_cuda_check_device_error(), "device error word")
    for b in wb + bufs:
        lib.vtb_cuda_release(b)
    lib.vtb_cuda_destroy(ctx)
