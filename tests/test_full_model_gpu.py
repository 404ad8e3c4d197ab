"""Full-size model workloads.  TinyLlama-1.1B architecture, random init,
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
    """Llama-3-8B architecture (Q4_K_M-style, random init)
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
    """Llama-3-8B at full size — 2048-token prefill + 512 greedy steps —
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


def test_llama3_8b_batch32_vs_golden():
    """Batch-32 decode of the Llama-3-8B architecture (32 independent sequences
    decoded as one batch: the split-K GEMM path) against the oracle fixture
    tests/golden/llama3_8b_b32.npz (tests/golden/make_llama3_8b_b32.py), on
    the fixture's per-sequence input streams: all 32 sequences for the first
    16 steps and sequences 0 and 17 for 512 steps, the greedy choice (argmax)
    identical and each step's top-16 logits within 1e-3."""
    import os
    from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "llama3_8b_b32.npz")
    if not os.path.exists(path):
        pytest.skip("golden fixture not generated")
    g = np.load(path)
    w = HostWeights(LLAMA3_8B, seed=int(g["seed_w"]))
    streams = g["tokens"].astype(np.int32)  # [32, 512] input token per sequence and step
    n_short, n_long = g["short_ids"].shape[1], g["long_ids"].shape[1]
    long_seqs = [int(s) for s in g["long_seqs"]]
    st = CudaState(CudaModel(Context(0), w), 32, max_rows=32)
    for step in range(n_long):
        lg, am = st.step(streams[:, step])
        seqs = range(32) if step < n_short else long_seqs
        for s in seqs:
            if step < n_short:
                ti, tv, ref = g["short_top_idx"][s, step], g["short_top_val"][s, step], int(g["short_ids"][s, step])
            else:
                j = long_seqs.index(s)
                ti, tv, ref = g["long_top_idx"][j, step], g["long_top_val"][j, step], int(g["long_ids"][j, step])
            err = float(np.abs(lg[s][ti] - tv).max() / np.abs(tv).max())
            assert err <= 1e-3, f"sequence {s} step {step}: top-16 logits differ by {err:.2e}"
            assert int(am[s]) == ref, f"sequence {s} step {step}: token {int(am[s])} != oracle {ref}"
