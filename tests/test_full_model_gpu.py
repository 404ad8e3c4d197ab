"""BASELINE config 4 at full size: TinyLlama-1.1B architecture, random init,
128-token prompt (batched prefill) + 256 greedy decode steps; token ids must
equal the CPU oracle's (forward.zig / prefill.zig restatement)."""
import numpy as np
import pytest

import oracle as O
from vantablack_b200.model import TINYLLAMA, HostWeights

pytestmark = pytest.mark.gpu


def test_tinyllama_prompt128_decode256_greedy_identical():
    from vantablack_b200.model import Context, CudaModel, CudaState
    O.set_threads(16)
    w = HostWeights(TINYLLAMA, seed=4)
    prompt = np.random.default_rng(44).integers(3, TINYLLAMA.vocab_size, 128)
    ids_ref, lg_ref = O.Model(w).generate_greedy(prompt, 256, use_prefill=True)
    ctx = Context(0)
    st = CudaState(CudaModel(ctx, w), 1, max_rows=128)
    ids, lg = st.generate_greedy(prompt, 256, use_prefill=True)
    first_diff = next((i for i, (a, b) in enumerate(zip(ids, ids_ref)) if a != b), None)
    assert first_diff is None, f"first differing decode step: {first_diff}"
    assert float(np.abs(lg - lg_ref).max() / np.abs(lg_ref).max()) <= 1e-3
