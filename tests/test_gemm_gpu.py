"""Prefill GEMM (tcgen05 tensor cores) against the oracle's matmulBatched
(prefill.zig:325-378).  Tolerances: bf16 mode max|d|/max|ref| <= 2e-2
(north star), precise (hi/lo split) mode <= 1e-4."""
import numpy as np
import pytest
import torch

import oracle as O
from vantablack_b200 import synth as S

pytestmark = pytest.mark.gpu
O.set_threads(16)


def ops():
    from vantablack_b200 import ops as _ops
    return _ops


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


@pytest.mark.parametrize("q,m,k,B", [
    (S.Q4_K, 14336, 4096, 87),   # config 3: ffn_up/gate, B = 87
    (S.Q6_K, 4096, 14336, 87),   # config 3: ffn_down
    (S.Q4_K, 512, 4096, 512), (S.Q6_K, 256, 14336, 512), (S.Q4_K, 384, 4096, 2048),
    (S.Q5_K, 300, 2048, 17), (S.Q8_0, 200, 1024, 33), (S.Q6_K, 130, 5632, 1), (S.Q4_K, 1, 256, 300),
])
@pytest.mark.parametrize("precise", [False, True])
def test_gemm_matches_oracle(q, m, k, B, precise):
    rng = np.random.default_rng(m + k + B + q)
    w = S.quant_tensor(rng, q, m, k)
    acts = S.activations(rng, B, k)
    out = ops().gemm(q, torch.from_numpy(w).cuda(), torch.from_numpy(acts).cuda(), m, k, precise=precise)
    got = out.cpu().numpy()
    ops().check_device_error()
    ref = O.matmul_batched(q, w, acts, m, k, B)
    assert rel(got, ref) <= (1e-4 if precise else 2e-2)


def test_gemm_full_size_b2048_against_gemv():
    """Config 3 at B = 2048 (14336 x 4096 Q4_K): sampled tokens against the
    fp32-class GEMV on the GPU (the CPU oracle would take minutes)."""
    rng = np.random.default_rng(9)
    m, k, B = 14336, 4096, 2048
    w = torch.from_numpy(S.quant_tensor(rng, S.Q4_K, m, k)).cuda()
    acts = torch.from_numpy(S.activations(rng, B, k)).cuda()
    out = ops().gemm(S.Q4_K, w, acts, m, k, precise=True)
    for b in (0, 1, 777, 2047):
        y = ops().gemv(S.Q4_K, w, acts[b].contiguous(), m, k)
        assert rel(out[b].cpu().numpy(), y.cpu().numpy().astype(np.float64)) <= 1e-4
