"""One process, several GPUs: the launchers' per-device state (shared-memory
opt-in, SM count, occupancy) must be set up on every device a caller uses.
Runs the tensor-core GEMVs and the GEMM on each visible device in turn and
checks each result against the CPU oracle.  Skipped with fewer than 2 GPUs."""
import numpy as np
import pytest
import torch

import oracle as O
from vantablack_b200 import synth as S

pytestmark = pytest.mark.gpu


def rel_err(got, ref):
    return float(np.abs(got.astype(np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_kernels_on_every_device():
    from vantablack_b200 import ops
    rng = np.random.default_rng(21)
    m, k, b = 1024, 4096, 16
    cases = [(q, S.quant_tensor(rng, q, m, k)) for q in (S.Q4_K, S.Q6_K)]
    x = S.activations(rng, k)
    acts = S.activations(rng, b, k)
    for dev in range(torch.cuda.device_count()):
        with torch.cuda.device(dev):
            for q, w in cases:
                wt = torch.from_numpy(w).cuda()
                y = ops.gemv(q, wt, torch.from_numpy(x).cuda(), m, k).cpu().numpy()
                assert rel_err(y, O.matmul(q, w, x, m, k)) <= 1e-4, (dev, S.NAMES[q])
                o = ops.gemm(q, wt, torch.from_numpy(acts).cuda(), m, k, precise=True).cpu().numpy()
                ref = np.stack([O.matmul(q, w, acts[i], m, k) for i in range(b)])
                assert rel_err(o, ref) <= 1e-4, (dev, S.NAMES[q], "gemm")
            ops.check_device_error()
