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


def test_llama3_8b_greedy_identical():
    """BASELINE config 5 architecture (Llama-3-8B, Q4_K_M-style, random init)
    on one GPU.  Default: 256-token prefill + 32 greedy steps; with
    VTB_FULL_8B=1 the configured 2048-token prefill + 512 steps (slow on the
    CPU oracle)."""
    import os
    from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState
    full = os.environ.get("VTB_FULL_8B") == "1"
    n_prompt, n_gen = (2048, 512) if full else (256, 32)
    O.set_threads(os.cpu_count() or 16)
    w = HostWeights(LLAMA3_8B, seed=5)
    prompt = np.random.default_rng(55).integers(3, LLAMA3_8B.vocab_size, n_prompt)
    ctx = Context(0)
    st = CudaState(CudaModel(ctx, w), 1, max_rows=n_prompt)
    ids, lg = st.generate_greedy(prompt, n_gen, use_prefill=True)
    ids_ref, lg_ref = O.Model(w).generate_greedy(prompt, n_gen, use_prefill=True)
    first_diff = next((i for i, (a, b) in enumerate(zip(ids, ids_ref)) if a != b), None)
    assert first_diff is None, f"first differing decode step: {first_diff}"
    assert float(np.abs(lg - lg_ref).max() / np.abs(lg_ref).max()) <= 1e-3


def test_llama3_8b_full_config_vs_golden():
    """BASELINE config 5 at full size — 2048-token prefill + 512 greedy steps —
    against the oracle's token ids and final logits stored in
    tests/golden/llama3_8b_p2048_g512.npz (tests/golden/make_llama3_8b_full.py)."""
    import os
    from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "llama3_8b_p2048_g512.npz")
    if not os.path.exists(path):
        pytest.skip("golden fixture not generated")
    g = np.load(path)
    n_prompt, n_gen = int(g["n_prompt"]), int(g["n_gen"])
    w = HostWeights(LLAMA3_8B, seed=int(g["seed_w"]))
    prompt = np.random.default_rng(int(g["seed_p"])).integers(3, LLAMA3_8B.vocab_size, n_prompt)
    st = CudaState(CudaModel(Context(0), w), 1, max_rows=n_prompt)
    lg, _ = st.prefill(prompt)
    ids_ref = [int(v) for v in g["ids"]]
    for step in range(n_gen):
        # the oracle's 16 largest logits of this step, read back at the same indices
        ti, tv = g["top_idx"][step], g["top_val"][step]
        err = float(np.abs(lg[ti] - tv).max() / np.abs(tv).max())
        assert err <= 1e-3, f"step {step}: top-16 logits differ by {err:.2e}"
        nxt = int(np.argmax(lg))
        assert nxt == ids_ref[step], f"step {step}: token {nxt} != oracle {ids_ref[step]}"
        lgs, _ = st.step([nxt])
        lg = lgs[0]
    lg_ref = g["logits"]
    assert float(np.abs(lg - lg_ref).max() / np.abs(lg_ref).max()) <= 1e-3


def test_llama3_8b_batch32_subset():
    """Batch-32 decode of the 8B architecture: all 32 sequences for the first
    steps, two of them checked against independent oracle runs."""
    import os
    from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState
    O.set_threads(os.cpu_count() or 16)
    w = HostWeights(LLAMA3_8B, seed=6)
    rng = np.random.default_rng(66)
    toks = rng.integers(3, LLAMA3_8B.vocab_size, 32)
    st = CudaState(CudaModel(Context(0), w), 32, max_rows=32)
    refs = {0: O.Model(w), 17: O.Model(w)}
    ref_tok = {s: int(toks[s]) for s in refs}
    for step in range(6):
        _, am = st.step(toks, want_logits=False)
        for s, ref in refs.items():
            nxt = O.argmax(ref.step(ref_tok[s]))
            assert int(am[s]) == nxt, f"sequence {s} step {step}"
            ref_tok[s] = nxt
        toks = am
