"""Generates tests/golden/llama3_8b_b32.npz: the CPU oracle's greedy runs of
the batch-32 decode workload on the Llama-3-8B architecture (Q4_K_M-style
random init, HostWeights seed 6).  The 32 sequences are independent, each
starts from one seeded token at position 0 (the reference decodes one
sequence per KV cache; forward.zig:152-172).  Each sequence is fed its own
seeded stream of input tokens (teacher forcing: with random weights a
self-fed greedy sequence repeats one token after a few steps, which makes
every later attention step trivial), and every step records the greedy
choice (argmax) and the 16 largest logits (indices and values):

  * all 32 sequences for the first 16 steps,
  * sequences 0 and 17 for 512 steps.

The GPU test runs the 32 sequences as one batch (one token per sequence per
step) on the same input streams and checks them against this file.

Run from the repository root:  python tests/golden/make_llama3_8b_b32.py
"""
import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..", "..")))
import oracle as O  # noqa: E402
from vantablack_b200.model import LLAMA3_8B, HostWeights  # noqa: E402

SEED_W, SEED_T, N_SEQ, N_SHORT, N_LONG, LONG = 6, 66, 32, 16, 512, (0, 17)


def run(model, stream):
    model.reset()
    ids, top_i, top_v = [], [], []
    for tok in stream:
        logits = model.step(int(tok))
        top = np.argsort(-logits, kind="stable")[:16]
        top_i.append(top.astype(np.int32))
        top_v.append(logits[top].astype(np.float32))
        ids.append(O.argmax(logits))
    return np.asarray(ids, np.int32), np.stack(top_i), np.stack(top_v)


def main():
    O.set_threads(os.cpu_count() or 8)
    t0 = time.time()
    w = HostWeights(LLAMA3_8B, seed=SEED_W)
    toks = np.random.default_rng(SEED_T).integers(3, LLAMA3_8B.vocab_size, (N_SEQ, N_LONG)).astype(np.int32)
    model = O.Model(w)
    short = [run(model, toks[s, :N_SHORT]) for s in range(N_SEQ)]
    long_ = [run(model, toks[s]) for s in LONG]
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "llama3_8b_b32.npz")
    np.savez_compressed(out, tokens=toks,
                        short_ids=np.stack([r[0] for r in short]), short_top_idx=np.stack([r[1] for r in short]),
                        short_top_val=np.stack([r[2] for r in short]),
                        long_seqs=np.asarray(LONG, np.int32), long_ids=np.stack([r[0] for r in long_]),
                        long_top_idx=np.stack([r[1] for r in long_]), long_top_val=np.stack([r[2] for r in long_]),
                        seed_w=SEED_W, seed_t=SEED_T)
    print(f"wrote {out} in {time.time() - t0:.0f} s")


if __name__ == "__main__":
    main()
