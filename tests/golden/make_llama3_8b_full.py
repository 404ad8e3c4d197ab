"""Generates tests/golden/llama3_8b_p2048_g512.npz: the CPU oracle's greedy
run of BASELINE config 5 at full size — Llama-3-8B architecture, Q4_K_M-style
random init (HostWeights seed 5), a seeded 2048-token prompt (batched
prefill) and 512 greedy decode steps.  Stored: the 512 token ids and the
final logits (f32), so the GPU test checks the full configuration without
re-running the ~25-minute oracle.

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
    ids, logits = O.Model(w).generate_greedy(prompt, N_GEN, use_prefill=True)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "llama3_8b_p2048_g512.npz")
    np.savez_compressed(out, ids=np.asarray(ids, np.int32), logits=np.asarray(logits, np.float32),
                        n_prompt=N_PROMPT, n_gen=N_GEN, seed_w=SEED_W, seed_p=SEED_P)
    print(f"wrote {out} in {time.time() - t0:.0f} s; first ids {ids[:8]}")


if __name__ == "__main__":
    main()
