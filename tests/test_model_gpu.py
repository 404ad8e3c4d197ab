"""GPU forward loop (the backend vtable + CUDA graph step + batched prefill)
against the CPU oracle's restatement of forward.zig / prefill.zig on the
same seeded weights.  Bar: identical greedy token ids; logits within
max|d| / max|ref| <= 1e-3 (several fp32 GEMVs and attention in sequence)."""
import numpy as np
import pytest

import oracle as O
from vantablack_b200 import synth as S
from vantablack_b200.model import LlamaConfig, HostWeights

pytestmark = pytest.mark.gpu
O.set_threads(8)

SMALL = LlamaConfig(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab_size=512,
                    max_seq=600, rope_base=10000.0)
LTOL = 1e-3


def rel(a, b):
    return float(np.abs(a.astype(np.float64) - b).max() / np.abs(b).max())


@pytest.fixture(scope="module")
def small():
    from vantablack_b200.model import Context, CudaModel
    w = HostWeights(SMALL, seed=1)
    ctx = Context(0)
    return w, ctx, CudaModel(ctx, w)


def test_decode_steps_match_oracle(small):
    from vantablack_b200.model import CudaState
    w, ctx, m = small
    ref = O.Model(w)
    st = CudaState(m, 1)
    toks = np.random.default_rng(2).integers(3, SMALL.vocab_size, 300)
    for i, t in enumerate(toks):  # crosses the 256-position attention split boundary
        lg, am = st.step([int(t)])
        rl = ref.step(int(t))
        assert rel(lg[0], rl) <= LTOL, f"step {i}"
        assert int(am[0]) == O.argmax(rl)
    assert st.pos() == len(toks) == ref.pos


def test_vtable_slots_equal_graph_step(small):
    from vantablack_b200.model import CudaState
    w, ctx, m = small
    a, b = CudaState(m, 1), CudaState(m, 1)
    for t in (5, 17, 400, 3):
        la, _ = a.step([t], graph=True)
        lb, _ = b.step([t], graph=False)
        assert np.array_equal(la, lb)


def test_prefill_matches_oracle_and_continues(small):
    from vantablack_b200.model import CudaState
    w, ctx, m = small
    prompt = np.random.default_rng(3).integers(3, SMALL.vocab_size, 40)
    ref = O.Model(w)
    rl = ref.prefill(prompt)
    st = CudaState(m, 1, max_rows=16)  # forces three prefill chunks
    lg, am = st.prefill(prompt)
    assert rel(lg, rl) <= LTOL and am == O.argmax(rl)
    assert st.pos() == 40
    for t in (7, 9):
        l2, _ = st.step([t])
        assert rel(l2[0], ref.step(t)) <= LTOL


def test_greedy_tokens_identical(small):
    from vantablack_b200.model import CudaState
    w, ctx, m = small
    prompt = np.random.default_rng(4).integers(3, SMALL.vocab_size, 24)
    ids_ref, _ = O.Model(w).generate_greedy(prompt, 48, use_prefill=True)
    ids, _ = CudaState(m, 1).generate_greedy(prompt, 48, use_prefill=True)
    assert ids == ids_ref


def test_batch_decode_sequences_independent(small):
    from vantablack_b200.model import CudaState
    w, ctx, m = small
    st = CudaState(m, 3)
    refs = [O.Model(w) for _ in range(3)]
    rng = np.random.default_rng(6)
    for _ in range(5):
        toks = rng.integers(3, SMALL.vocab_size, 3)
        lg, am = st.step(toks)
        for s in range(3):
            rl = refs[s].step(int(toks[s]))
            assert rel(lg[s], rl) <= LTOL
            assert int(am[s]) == O.argmax(rl)


def test_errors(small):
    from vantablack_b200 import _lib
    from vantablack_b200.model import CudaState, CudaModel
    w, ctx, m = small
    st = CudaState(m, 1)
    with pytest.raises(_lib.VtbError) as e:
        st.step([SMALL.vocab_size])  # TokenOutOfRange -> invalid argument
    assert e.value.status == -1
    big = HostWeights(SMALL.with_(max_seq=4), seed=1)
    st4 = CudaState(CudaModel(ctx, big), 1)
    for t in range(4):
        st4.step([t + 3])
    with pytest.raises(_lib.VtbError) as e:
        st4.step([3])  # KvCacheFull
    assert e.value.status == -7
    with pytest.raises(_lib.VtbError):  # a projection without a CUDA kernel is refused (no CPU fallback)
        bad = HostWeights(SMALL, seed=1)
        bad.layers[0]["attn_q"] = (S.F32, np.zeros(SMALL.dim * SMALL.dim * 4, np.uint8))
        CudaModel(ctx, bad)


def test_q8_0_q5_k_and_tq2_0_models(small):
    from vantablack_b200.model import Context, CudaModel, CudaState
    w, ctx, _ = small
    for q in (S.Q8_0, S.Q5_K, S.TQ2_0):
        qs = {n: q for n in ("attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down")}
        hw = HostWeights(SMALL, seed=9, quants=dict(qs, token_embd=q, output=q))
        ids_ref, lr = O.Model(hw).generate_greedy([5, 6, 7], 8, use_prefill=False)
        ids, lg = CudaState(CudaModel(ctx, hw), 1).generate_greedy([5, 6, 7], 8, use_prefill=False)
        assert ids == ids_ref and rel(lg, lr) <= LTOL
        # batched prefill (the tcgen05 GEMM path) of the same model
        ids_p, lgp = CudaState(CudaModel(ctx, hw), 1, max_rows=16).generate_greedy(list(range(5, 21)), 4)
        ids_pr, lpr = O.Model(hw).generate_greedy(list(range(5, 21)), 4, use_prefill=True)
        assert ids_p == ids_pr and rel(lgp, lpr) <= LTOL, S.NAMES[q]


def test_q8_0_model_with_q8_0_activations(small):
    """Dynamic activation quantization (the Q8_0 x Q8_0 path on every Q8_0
    projection, vtb_cuda_model_set_q8_activations): greedy ids and logits equal
    the oracle run with the same option, in decode and in prefill."""
    from vantablack_b200.model import CudaModel, CudaState
    w, ctx, _ = small
    qs = {n: S.Q8_0 for n in ("attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down")}
    hw = HostWeights(SMALL, seed=19, quants=dict(qs, token_embd=S.Q8_0, output=S.Q8_0))
    ids_ref, lr = O.Model(hw, q8_activations=True).generate_greedy([5, 6, 7], 8, use_prefill=False)
    m = CudaModel(ctx, hw, q8_activations=True)
    ids, lg = CudaState(m, 1).generate_greedy([5, 6, 7], 8, use_prefill=False)
    assert ids == ids_ref and rel(lg, lr) <= LTOL
    prompt = list(range(5, 21))
    ids_p, lgp = CudaState(m, 1, max_rows=16).generate_greedy(prompt, 4)
    ids_pr, lpr = O.Model(hw, q8_activations=True).generate_greedy(prompt, 4, use_prefill=True)
    assert ids_p == ids_pr and rel(lgp, lpr) <= LTOL
    # the option changes the arithmetic: the f32-activation oracle differs
    _, lf = O.Model(hw).generate_greedy([5, 6, 7], 8, use_prefill=False)
    assert rel(lf, lr) > 0
