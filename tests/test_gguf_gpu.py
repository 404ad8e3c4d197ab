"""A Llama model loaded from a GGUF file (vtb_cuda_model_create_gguf) runs
bit-identically to the same weights handed over as host arrays, and matches
the CPU oracle's greedy ids; tied embeddings, the max_seq override and the
type checks of the loader."""
import numpy as np
import pytest

import oracle as O
from vantablack_b200 import _lib
from vantablack_b200 import synth as S
from vantablack_b200.gguf import GgufFile
from vantablack_b200.model import Context, CudaModel, CudaState, HostWeights, LlamaConfig

from gguf_util import write_llama_gguf

pytestmark = pytest.mark.gpu
SMALL = LlamaConfig(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab_size=512,
                    max_seq=600, rope_base=10000.0)


def _run(model, prompt, n_gen):
    st = CudaState(model, 1, max_rows=len(prompt))
    ids, lg = st.generate_greedy(prompt, n_gen, use_prefill=True)
    st.close()
    return ids, lg


@pytest.mark.parametrize("tied", [False, True])
def test_gguf_model_matches_host_weights_and_oracle(tmp_path, tied):
    w = HostWeights(SMALL, seed=12, quants={"attn_v": S.Q6_K, "ffn_gate": S.Q5_K})
    if tied:
        w.output = w.token_embd
    p = tmp_path / "small.gguf"
    write_llama_gguf(p, w, tied=tied)
    prompt = np.random.default_rng(120).integers(3, SMALL.vocab_size, 32)
    ctx = Context(0)
    with GgufFile(p) as g:
        mg = CudaModel.from_gguf(ctx, g)
    ids_g, lg_g = _run(mg, prompt, 24)
    ids_h, lg_h = _run(CudaModel(ctx, w), prompt, 24)
    assert ids_g == ids_h and np.array_equal(lg_g, lg_h)
    ids_ref, lg_ref = O.Model(w).generate_greedy(prompt, 24, use_prefill=True)
    assert ids_g == ids_ref
    assert float(np.abs(lg_g - lg_ref).max() / np.abs(lg_ref).max()) <= 1e-3


def test_gguf_max_seq_override_and_type_checks(tmp_path):
    w = HostWeights(SMALL, seed=13)
    p = tmp_path / "small.gguf"
    write_llama_gguf(p, w)
    ctx = Context(0)
    with GgufFile(p) as g:
        m = CudaModel.from_gguf(ctx, g, max_seq=40)
    st = CudaState(m, 1, max_rows=40)
    st.prefill(np.arange(3, 43))  # exactly fills the 40-position cache
    with pytest.raises(_lib.VtbError) as e:
        st.step([5])
    assert e.value.status == -7  # KV cache full (KvCacheFull)
    st.close()
    # an f16 norm is not a layout this path takes: refused, not converted
    w.layers[0]["attn_norm"] = w.layers[0]["attn_norm"].astype(np.float16)
    p2 = tmp_path / "f16norm.gguf"
    write_llama_gguf(p2, w)
    with GgufFile(p2) as g:
        with pytest.raises(_lib.VtbError) as e:
            CudaModel.from_gguf(ctx, g)
    assert e.value.status == -8
