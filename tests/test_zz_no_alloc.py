"""The allocation-free Q8_0 x Q8_0 GEMV (vtb_cuda_gemv_q8_0_q8_0_noalloc).

It exists for hosts that cannot allocate device memory on their decode path
(a fixed budget reserved at start-up, or a warm serving loop that forbids
allocation): its activation scratch is a fixed array inside the library.
This file is collected last on purpose.  It checks, through the C ABI, that
two calls in a row -- the second with different inputs over the scratch the
first one left behind -- give the same output as the allocating entry point,
within the GEMV tolerance, and that a k above the fixed maximum is refused.
"""
import numpy as np
import pytest
import torch

from vantablack_b200 import _lib
from vantablack_b200 import synth as S

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _reference(lib, w, x, m, k, stream):
    y = torch.empty(m, dtype=torch.float32, device="cuda")
    xq = torch.empty(k, dtype=torch.int8, device="cuda")
    dx = torch.empty(k // 32, dtype=torch.float32, device="cuda")
    _lib.check(lib.vtb_cuda_gemv_q8_0_q8_0(w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, xq.data_ptr(),
                                           dx.data_ptr(), stream, 0), "gemv_q8_0_q8_0")
    return y


def test_noalloc_matches_allocating_entry_point_twice():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(123)
    for m, k in ((4096, 4096), (777, 14336)):  # second call: different shape and data over the same scratch
        w = torch.from_numpy(S.quant_tensor(rng, S.Q8_0, m, k)).cuda()
        x = torch.from_numpy(S.activations(rng, k)).cuda()
        y = torch.empty(m, dtype=torch.float32, device="cuda")
        _lib.check(lib.vtb_cuda_gemv_q8_0_q8_0_noalloc(w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, stream, 0),
                   "gemv_q8_0_q8_0_noalloc")
        ref = _reference(lib, w, x, m, k, stream)
        got, exp = y.cpu().numpy(), ref.cpu().numpy()
        assert float(np.abs(got - exp).max() / np.abs(exp).max()) <= TOL


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
