"""MLX affine-quantized GEMV and dequant (src/kernels/mlx.zig; Metal
matmul_mlx_q4, src/metal/bridge.m:245-291) against the oracle's restatement
on the same seeded tensors.  Bar: dequant bit-exact; GEMV max|d| / max|ref|
<= 1e-4 (fp32 accumulation in another order)."""
import ctypes

import numpy as np
import pytest
import torch

import oracle as O
from vantablack_b200 import _lib, ops, synth as S

pytestmark = pytest.mark.gpu
TOL = 1e-4


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


def dev(a: np.ndarray, off: int = 0) -> torch.Tensor:
    """Upload bytes so that the returned tensor starts `off` bytes past a
    256-byte boundary (safetensors tensors sit at arbitrary offsets)."""
    t = torch.zeros(a.size + off, dtype=torch.uint8, device="cuda")
    t[off:] = torch.from_numpy(a).cuda()
    return t[off:]


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("bits", [2, 3, 4, 5, 6, 8])
def test_mlx_gemv_and_dequant(bits, bf16):
    rng = np.random.default_rng(bits * 10 + bf16)
    el = 32 // bits
    group = 64 if 64 % el == 0 else {3: 320, 5: 192, 6: 320}[bits]  # a multiple of 32 / bits
    m, k = 1000, 40 * group if bits in (3, 5, 6) else 4096
    w, sc, bi = S.mlx_tensor(rng, m, k, bits, group, bf16)
    x = S.activations(rng, k)
    y = ops.gemv_mlx(dev(w), dev(sc), dev(bi), torch.from_numpy(x).cuda(), m, k, bits, group, bf16).cpu().numpy()
    assert rel(y, O.mlx_matmul(w, sc, bi, x, m, k, bits, group, bf16)) <= TOL
    rows = 37
    d = ops.dequant_mlx(dev(w), dev(sc), dev(bi), rows, k, bits, group, bf16).cpu().numpy()
    assert np.array_equal(d.view(np.uint32), O.mlx_dequant(w, sc, bi, rows, k, bits, group, bf16).view(np.uint32))
    ops.check_device_error()


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("offs", [(0, 0, 0), (1, 3, 1), (3, 2, 5)])
def test_mlx_q4_groups_and_unaligned(group, offs):
    """4-bit at the group sizes MLX ships, with the weight, scales and biases
    at byte offsets that are not 4-byte aligned."""
    rng = np.random.default_rng(group + sum(offs))
    m, k = 14336 if group == 64 else 2048, 4096
    w, sc, bi = S.mlx_tensor(rng, m, k, 4, group, True)
    x = S.activations(rng, k)
    y = ops.gemv_mlx(dev(w, offs[0]), dev(sc, offs[1]), dev(bi, offs[2]), torch.from_numpy(x).cuda(), m, k, 4,
                     group, True).cpu().numpy()
    assert rel(y, O.mlx_matmul(w, sc, bi, x, m, k, 4, group, True)) <= TOL
    d = ops.dequant_mlx(dev(w, offs[0]), dev(sc, offs[1]), dev(bi, offs[2]), 5, k, 4, group, True).cpu().numpy()
    assert np.array_equal(d, O.mlx_dequant(w, sc, bi, 5, k, 4, group, True))


def test_mlx_runtime_fixture_on_gpu():
    """forward.zig:853-1040: every nibble 3, scale 0.5, bias 0.25 (f16) or
    -1.0 (bf16), x = e0 -> 1.75 / 0.5 on every row, as the CPU baseline gives."""
    m, k = 4, 64
    w = np.full(m * k // 2, 0x33, np.uint8)
    x = np.zeros(k, np.float32); x[0] = 1.0
    for s, b, bf16, want in ((b"\x00\x38", b"\x00\x34", False, 1.75), (b"\x00\x3f", b"\x80\xbf", True, 0.5)):
        sc = np.frombuffer(s * m, np.uint8).copy()
        bi = np.frombuffer(b * m, np.uint8).copy()
        y = ops.gemv_mlx(dev(w), dev(sc), dev(bi), torch.from_numpy(x).cuda(), m, k, 4, 64, bf16).cpu().numpy()
        assert np.array_equal(y, np.full(m, want, np.float32))


def test_mlx_bridge_one_shot():
    """vtb_cuda_matmul_mlx_q4: weight, scales and biases in one uploaded blob at
    odd offsets (one safetensors shard), as vtb_metal_matmul_mlx_q4 takes them."""
    lib = _lib.load()
    rng = np.random.default_rng(21)
    m, k, group = 512, 2048, 64
    w, sc, bi = S.mlx_tensor(rng, m, k, 4, group, False)
    blob = np.concatenate([np.zeros(3, np.uint8), w, np.zeros(1, np.uint8), sc, bi])
    w_off, s_off = 3, 3 + w.size + 1
    b_off = s_off + sc.size
    x = S.activations(rng, k)
    ctx = lib.vtb_cuda_init(0)
    wb = lib.vtb_cuda_upload(ctx, blob.ctypes.data, blob.nbytes)
    xb = lib.vtb_cuda_upload(ctx, x.ctypes.data, x.nbytes)
    yb = lib.vtb_cuda_alloc(ctx, m * 4, None)
    _lib.check(lib.vtb_cuda_matmul_mlx_q4(ctx, yb, wb, w_off, wb, s_off, wb, b_off, xb, 0, m, k, group, 0), "mlx")
    y = np.empty(m, np.float32)
    _lib.check(lib.vtb_cuda_copy_d2h(ctx, y.ctypes.data, yb, 0, m * 4), "d2h")
    assert rel(y, O.mlx_matmul(w, sc, bi, x, m, k, 4, group, False)) <= TOL
    assert lib.vtb_cuda_matmul_mlx_q4(ctx, yb, wb, w_off, wb, s_off, wb, b_off, xb, 0, m + 1, k, group, 0) == -1
    for b in (wb, xb, yb):
        lib.vtb_cuda_release(b)
    lib.vtb_cuda_destroy(ctx)


def test_mlx_q4_wide_rows():
    """k = 14336 (Llama-3-8B ffn_down): 57 KB of staged activations per CTA."""
    rng = np.random.default_rng(5)
    m, k, group = 4096, 14336, 64
    w, sc, bi = S.mlx_tensor(rng, m, k, 4, group, False)
    x = S.activations(rng, k)
    y = ops.gemv_mlx(dev(w), dev(sc), dev(bi), torch.from_numpy(x).cuda(), m, k, 4, group, False).cpu().numpy()
    assert rel(y, O.mlx_matmul(w, sc, bi, x, m, k, 4, group, False)) <= TOL
