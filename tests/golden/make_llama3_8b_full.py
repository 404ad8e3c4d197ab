"""Generates tests/golden/llama3_8b_p2048_g512.npz: the CPU oracle's greedy
run of the full-size Llama-3-8B workload — Llama-3-8B architecture, Q4_K_M-style
random init (HostWeights seed 5), a seeded 2048-token prompt (batched
prefill) and 512 greedy decode steps.  Stored: the 512 token ids, the
16 largest logits (indices and values) of each of the 512 logit vectors the
ids were chosen from, and the final logits (f32), so the GPU test checks the
full configuration step by step without re-running the ~30-minute oracle.

Run from the repository root:  python tests/golden/make_llama3_8b_full.py
"""
import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))
import oracle as O  # noqa: E402
from vantablack_b200.model import LLAMA3_8B, HostWeights  # noqa: E402

N_PROMPT, N_GEN, SEED_W, SEED_P = 2048, 512, 5, 55


def main():
    O.set_threads(os.cpu_count() or 8)
    t0 = time.time()
    w = HostWeights(LLAMA3_8B, seed=SEED_W)
    prompt = np.random.default_rng(SEED_P).integers(3, LLAMA3_8B.vocab_size, N_PROMPT)
    model = O.Model(w)
    logits = model.prefill(prompt)
    ids, top_i, top_v = [], [], []
    for _ in range(N_GEN):
        top = np.argsort(-logits, kind="stable")[:16]
        top_i.append(top.astype(np.int32))
        top_v.append(logits[top].astype(np.float32))
        nxt = O.argmax(logits)
        ids.append(nxt)
        logits = model.step(nxt)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "llama3_8b_p2048_g512.npz")
    np.savez_compressed(out, ids=np.asarray(ids, np.int32), logits=np.asarray(logits, np.float32),
                        top_idx=np.stack(top_i), top_val=np.stack(top_v),
                        n_prompt=N_PROMPT, n_gen=N_GEN, seed_w=SEED_W, seed_p=SEED_P)
    print(f"wrote {out} in {time.time() - t0:.0f} s; first ids {ids[:8]}")


if __name__ == "__main__":
    main()
