"""The allocation-free Q8_0 x Q8_0 GEMV (vtb_cuda_gemv_q8_0_q8_0_noalloc).

It exists for hosts that cannot allocate device memory on their decode path
(a fixed budget reserved at start-up, or a warm serving loop that forbids
allocation): its activation scratch is a fixed array inside the library.
This file is collected last on purpose.  Through the C ABI it checks that
two calls in a row -- the second with a different shape and data over the
scratch the first one left behind, with and without programmatic dependent
launch -- give bit-identical output to the allocating entry point (both run
the same quantizer and GEMV kernels on the same data), that a warm call
allocates no device memory and leaves the device error word clear, and that
a k above the fixed maximum is refused.
"""
import numpy as np
import pytest
import torch

from vantablack_b200 import _lib, ops
from vantablack_b200 import synth as S

pytestmark = pytest.mark.gpu


def _reference(lib, w, x, m, k, stream):
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    xq = torch.empty(k, dtype=torch.int8, device="cuda")
    dx = torch.empty(k // 32, dtype=torch.float32, device="cuda")
    _lib.check(lib.vtb_cuda_gemv_q8_0_q8_0(w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, xq.data_ptr(),
                                           dx.data_ptr(), stream, 0), "gemv_q8_0_q8_0")
    return y


def _noalloc(lib, w, x, y, m, k, stream, pdl):
    _lib.check(lib.vtb_cuda_gemv_q8_0_q8_0_noalloc(w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, stream, pdl),
               "gemv_q8_0_q8_0_noalloc")


@pytest.mark.parametrize("pdl", [0, 1])
def test_noalloc_bit_identical_to_allocating_entry_point_twice(pdl):
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(123 + pdl)
    for m, k in ((4096, 4096), (777, 14336)):  # second call: different shape and data over the same scratch
        w = torch.from_numpy(S.quant_tensor(rng, S.Q8_0, m, k)).cuda()
        x = torch.from_numpy(S.activations(rng, k)).cuda()
        y = torch.full((m,), float("nan"), dtype=torch.float32, device="cuda")
        _noalloc(lib, w, x, y, m, k, stream, pdl)
        ref = _reference(lib, w, x, m, k, stream)
        got, exp = y.cpu().numpy(), ref.cpu().numpy()
        assert np.array_equal(got, exp), float(np.abs(got - exp).max())
    ops.check_device_error()


def test_noalloc_warm_call_allocates_nothing():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(7)
    m, k = 2048, 8192
    w = torch.from_numpy(S.quant_tensor(rng, S.Q8_0, m, k)).cuda()
    x = torch.from_numpy(S.activations(rng, k)).cuda()
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    _noalloc(lib, w, x, y, m, k, stream, 0)  # warm: resolves the scratch address, loads the kernels
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch_alloc0 = torch.cuda.memory_allocated()
    for _ in range(3):
        _noalloc(lib, w, x, y, m, k, stream, 1)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert torch.cuda.memory_allocated() == torch_alloc0
    ops.check_device_error()


def test_noalloc_rejects_k_above_the_fixed_scratch():
    lib = _lib.load()
    k = 65536 + 32
    w = torch.zeros(34 * (k // 32), dtype=torch.uint8, device="cuda")
    x = torch.zeros(k, dtype=torch.float32, device="cuda")
    y = torch.empty(1, dtype=torch.float32, device="cuda")
    rc = lib.vtb_cuda_gemv_q8_0_q8_0_noalloc(w.data_ptr(), x.data_ptr(), y.data_ptr(), 1, k,
                                             torch.cuda.current_stream().cuda_stream, 0)
    assert rc == -1
    assert b"VTB_CUDA_NOALLOC_MAX_K" in lib.vtb_cuda_last_error()
