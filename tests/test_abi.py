"""The C-ABI library loads without a GPU and exports every symbol that
include/vtb_cuda.h declares; host-side argument checks reject bad calls
before any launch."""
import ctypes

import pytest

from vantablack_b200 import _lib, build


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_exports_every_header_symbol(lib):
    syms = _lib.header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(lib, s), f"libvtbcuda.so does not export {s}"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"


def test_no_torch_in_abi():
    import re
    text = open(_lib.HEADER).read()
    assert not re.search(r"\btorch\b|\bat::|\bc10::|\bat::Tensor\b|\bPyObject\b", text)


def test_introspection(lib):
    assert b"sm_100a" in lib.vtb_cuda_version_string()
    assert lib.vtb_cuda_row_bytes(12, 2048) == 1152
    assert lib.vtb_cuda_row_bytes(14, 5632) == 4620
    assert lib.vtb_cuda_row_bytes(8, 4096) == 4352
    assert lib.vtb_cuda_row_bytes(12, 100) == -1
    assert lib.vtb_cuda_status_string(-9) == b"device-side bounded wait timed out"


def test_argument_checks_without_launch(lib):
    buf = ctypes.create_string_buffer(64)
    p = (ctypes.addressof(buf) + 15) & ~15
    # unsupported quant, k not a whole number of blocks, misaligned weights, null x
    assert lib.vtb_cuda_gemv(3, p, p, p, 4, 256, None, 0) == -8
    assert lib.vtb_cuda_gemv(12, p, p, p, 4, 100, None, 0) == -1
    assert lib.vtb_cuda_gemv(12, p + 1, p, p, 4, 256, None, 0) == -1
    assert lib.vtb_cuda_gemv(12, p, None, p, 4, 256, None, 0) == -1
    assert lib.vtb_cuda_gemv(12, p, p, p, 0, 256, None, 0) == -1
    assert b"aligned" in lib.vtb_cuda_last_error() or lib.vtb_cuda_last_error()
    assert lib.vtb_cuda_dequant(14, p, p, 100, None) == -1
    assert lib.vtb_cuda_quantize_q8_0(p, 33, p, p, None) == -1


def test_capabilities_slot_without_a_device(lib):
    """vtb_cuda_capabilities fills the vtable's Capabilities (backend.zig:43-55)."""
    class Caps(ctypes.Structure):
        _fields_ = [("supports_fused_qkv", ctypes.c_int32), ("supports_kquant_gpu", ctypes.c_int32),
                    ("supports_mlx_q4", ctypes.c_int32), ("unified_memory", ctypes.c_int32),
                    ("name", ctypes.c_char_p)]
    c = Caps()
    assert lib.vtb_cuda_capabilities(None, ctypes.byref(c)) == 0
    assert (c.supports_fused_qkv, c.supports_kquant_gpu, c.supports_mlx_q4, c.unified_memory) == (1, 1, 0, 0)
    assert b"b200" in c.name
    assert lib.vtb_cuda_capabilities(None, None) == -1


def test_sampler_argument_checks_without_launch(lib):
    """vtb_cuda_sample / vtb_cuda_state_sample reject bad configurations on the host."""
    buf = ctypes.create_string_buffer(64)
    p = ctypes.addressof(buf)
    u = (ctypes.c_float * 1)(0.5)
    cfg = _lib.SamplerConfig(-1.0, 0, 0.0, 0)  # negative temperature
    assert lib.vtb_cuda_sample(p, 1, 8, 8, ctypes.byref(cfg), u, p, None) == -1
    cfg = _lib.SamplerConfig(float("nan"), 0, 0.0, 0)
    assert lib.vtb_cuda_sample(p, 1, 8, 8, ctypes.byref(cfg), u, p, None) == -1
    cfg = _lib.SamplerConfig(1.0, 0, 0.9, 0)
    assert lib.vtb_cuda_sample(p, 0, 8, 8, ctypes.byref(cfg), u, p, None) == -1    # no rows
    assert lib.vtb_cuda_sample(p, 257, 8, 8, ctypes.byref(cfg), u, p, None) == -1  # above 256 rows
    assert lib.vtb_cuda_sample(p, 1, 8, 4, ctypes.byref(cfg), u, p, None) == -1    # stride below n
    assert lib.vtb_cuda_sample(p, 1, 8, 8, ctypes.byref(cfg), None, p, None) == -1  # no draws
    assert lib.vtb_cuda_sample(p, 1, 8, 8, None, u, p, None) == -1
    assert lib.vtb_cuda_state_sample(None, 1, ctypes.byref(cfg), u, p) == -1


def test_mlx_argument_checks_without_launch(lib):
    """MLX entry points reject unsupported widths and group sizes on the host."""
    buf = ctypes.create_string_buffer(256)
    p = (ctypes.addressof(buf) + 15) & ~15
    assert lib.vtb_cuda_gemv_mlx(p, p, p, p, p, 4, 64, 7, 64, 0, None) == -8      # 7 bits
    assert lib.vtb_cuda_gemv_mlx(p, p, p, p, p, 4, 64, 4, 48, 0, None) == -1      # group does not divide k
    assert lib.vtb_cuda_gemv_mlx(p, p, p, p, p, 4, 60, 3, 15, 0, None) == -1      # group not a multiple of 10
    assert lib.vtb_cuda_gemv_mlx(p, p, p, p + 4, p, 4, 64, 4, 64, 0, None) == -1  # x not 16-byte aligned
    assert lib.vtb_cuda_gemv_mlx(None, p, p, p, p, 4, 64, 4, 64, 0, None) == -1
    assert lib.vtb_cuda_dequant_mlx(p, p, p, None, 4, 64, 4, 64, 0, None) == -1
    assert lib.vtb_cuda_matmul_mlx_q4(None, None, None, 0, None, 0, None, 0, None, 0, 4, 64, 64, 0) == -1
