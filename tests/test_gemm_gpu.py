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
    (S.Q4_K, 14336, 4096, 87),   # Llama-3-8B ffn_up/gate, B = 87
    (S.Q6_K, 4096, 14336, 87),   # Llama-3-8B ffn_down, B = 87
    (S.Q4_K, 512, 4096, 512), (S.Q6_K, 256, 14336, 512), (S.Q4_K, 384, 4096, 2048),
    (S.Q5_K, 300, 2048, 17), (S.Q8_0, 200, 1024, 33), (S.Q6_K, 130, 5632, 1), (S.Q4_K, 1, 256, 300),
    (S.TQ2_0, 300, 2304, 40), (S.TQ2_0, 256, 4096, 512),
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


def _row_sample(q, w, m, k, rows):
    """The weight bytes of the given rows, concatenated (whole rows of blocks)."""
    rb = S.row_bytes(q, k)
    return np.concatenate([w[r * rb:(r + 1) * rb] for r in rows])


@pytest.mark.parametrize("q,m,k,B", [
    (S.Q4_K, 14336, 4096, 512), (S.Q4_K, 14336, 4096, 2048),   # ffn_up/gate at full size
    (S.Q6_K, 4096, 14336, 512), (S.Q6_K, 4096, 14336, 2048),   # ffn_down at full size
])
@pytest.mark.parametrize("precise", [False, True])
def test_gemm_full_size_sampled_rows_vs_oracle(q, m, k, B, precise):
    """Full-size prefill GEMMs at B = 512 and 2048: every token of 12 sampled
    weight rows (first, last, tile and split boundaries, random) against the
    oracle's matmulBatched on the same rows."""
    rng = np.random.default_rng(q * 7 + B)
    w = S.quant_tensor(rng, q, m, k)
    acts = S.activations(rng, B, k)
    out = ops().gemm(q, torch.from_numpy(w).cuda(), torch.from_numpy(acts).cuda(), m, k, precise=precise)
    ops().check_device_error()
    rows = sorted({0, 1, 127, 128, 255, m // 2, m - 129, m - 128, m - 1, *rng.integers(0, m, 3).tolist()})
    ref = O.matmul_batched(q, _row_sample(q, w, m, k, rows), acts, len(rows), k, B)
    got = out[:, rows].cpu().numpy()
    assert rel(got, ref) <= (1e-4 if precise else 2e-2)
