"""Tensor-parallel host logic on CPU with two gloo ranks (no GPU): each rank
takes its shard through the library's own shard plan and slicer
(vtb_cuda_tp_shard_plan / vtb_cuda_tp_slice), computes its partial products
with the CPU oracle, and the all-reduce / all-gather of the partials must
reproduce the full projections."""
import os
import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

from vantablack_b200 import synth as S

CFG = dict(dim=512, n_layers=1, n_heads=8, n_kv_heads=4, head_dim=64, ffn_dim=1024, vocab_size=768, max_seq=16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch
    import oracle as O
    from vantablack_b200.model import LlamaConfig, shard_plan, tp_slice
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = LlamaConfig(**CFG)
        rng = np.random.default_rng(0)  # every rank generates the same full tensors
        d, f, V = cfg.dim, cfg.ffn_dim, cfg.vocab_size
        wq = S.quant_tensor(rng, S.Q4_K, d, d)
        wo = S.quant_tensor(rng, S.Q4_K, d, d)
        wdown = S.quant_tensor(rng, S.Q6_K, d, f)
        wout = S.quant_tensor(rng, S.Q6_K, V, d)
        x = S.activations(rng, d)
        h = S.activations(rng, f)
        sh = shard_plan(cfg, rank, world)
        # column-parallel Q: this rank's head rows; all-gather
        q_loc = O.matmul(S.Q4_K, tp_slice(S.Q4_K, wq, d, d, sh.q_row0, sh.q_rows, 0, d), x, sh.q_rows, d)
        parts = [torch.zeros(sh.q_rows) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(q_loc))
        q_full = torch.cat(parts).numpy()
        # row-parallel O (K split on head columns) and down (K split on ffn columns); all-reduce
        o_loc = O.matmul(S.Q4_K, tp_slice(S.Q4_K, wo, d, d, 0, d, sh.o_col0, sh.o_cols),
                         x[sh.o_col0:sh.o_col0 + sh.o_cols].copy(), d, sh.o_cols)
        t = torch.from_numpy(o_loc.copy()); dist.all_reduce(t); o_full = t.numpy()
        dn_loc = O.matmul(S.Q6_K, tp_slice(S.Q6_K, wdown, d, f, 0, d, sh.down_col0, sh.down_cols),
                          h[sh.down_col0:sh.down_col0 + sh.down_cols].copy(), d, sh.down_cols)
        t = torch.from_numpy(dn_loc.copy()); dist.all_reduce(t); dn_full = t.numpy()
        # vocab-parallel LM head; all-gather
        lg_loc = O.matmul(S.Q6_K, tp_slice(S.Q6_K, wout, V, d, sh.vocab_row0, sh.vocab_rows, 0, d), x,
                          sh.vocab_rows, d)
        parts = [torch.zeros(sh.vocab_rows) for _ in range(world)]
        dist.all_gather(parts, torch.from_numpy(lg_loc))
        lg_full = torch.cat(parts).numpy()
        if rank == 0:
            def rel(a, b):
                return float(np.abs(a - b).max() / np.abs(b).max())
            q.put({
                "q": rel(q_full, O.matmul(S.Q4_K, wq, x, d, d)),
                "o": rel(o_full, O.matmul(S.Q4_K, wo, x, d, d)),
                "down": rel(dn_full, O.matmul(S.Q6_K, wdown, h, d, f)),
                "logits": rel(lg_full, O.matmul(S.Q6_K, wout, x, V, d)),
                "plan": [sh.heads, sh.kv_heads, sh.o_cols, sh.down_cols, sh.vocab_rows],
            })
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_reproduce_full_projections():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res["plan"] == [4, 2, 256, 512, 384]
    assert res["q"] == 0.0 and res["logits"] == 0.0          # row splits: bit-identical rows
    assert res["o"] <= 1e-5 and res["down"] <= 1e-5          # K splits: only the summation order changes


def test_shard_plan_rejects_unaligned_or_indivisible():
    import pytest
    from vantablack_b200 import _lib
    from vantablack_b200.model import LlamaConfig, shard_plan
    cfg = LlamaConfig(**CFG)
    with pytest.raises(_lib.VtbError):
        shard_plan(cfg, 0, 3)          # 8 heads do not divide by 3
    with pytest.raises(_lib.VtbError):
        shard_plan(cfg.with_(dim=512, ffn_dim=1024 + 256 * 2 + 0), 0, 8)  # kv heads 4 < 8
    small = LlamaConfig(dim=256, n_layers=1, n_heads=4, n_kv_heads=4, head_dim=64, ffn_dim=512, vocab_size=64,
                        max_seq=8)
    with pytest.raises(_lib.VtbError):
        shard_plan(small, 0, 4)         # O's K shard of 64 columns is not a whole 256-weight block


def _partition(shards, start_attr, len_attr, total):
    spans = sorted((getattr(s, start_attr), getattr(s, len_attr)) for s in shards)
    pos = 0
    for a, n in spans:
        assert a == pos and n > 0
        pos += n
    assert pos == total


def test_shard_plans_partition_every_tensor():
    """The shard plan at 1, 2, 4 and 8 ranks for both model configurations:
    heads, kv heads, ffn rows, O / down columns and vocabulary rows are each
    split into contiguous, disjoint, covering ranges; K splits fall on whole
    256-weight blocks, and configurations whose ffn split would not are refused."""
    import pytest
    from vantablack_b200 import _lib
    from vantablack_b200.model import LLAMA3_8B, TINYLLAMA, shard_plan
    for cfg in (LLAMA3_8B, TINYLLAMA):
        for world in (1, 2, 4, 8):
            kvd = cfg.n_kv_heads * cfg.head_dim
            if (cfg.ffn_dim // world) % 256:
                with pytest.raises(_lib.VtbError):
                    shard_plan(cfg, 0, world)
                continue
            shards = [shard_plan(cfg, r, world) for r in range(world)]
            for s in shards:
                assert s.heads == cfg.n_heads // world and s.kv_heads == cfg.n_kv_heads // world
                assert s.o_col0 % 256 == 0 and s.down_col0 % 256 == 0
            _partition(shards, "q_row0", "q_rows", cfg.n_heads * cfg.head_dim)
            _partition(shards, "kv_row0", "kv_rows", kvd)
            _partition(shards, "ffn_row0", "ffn_rows", cfg.ffn_dim)
            _partition(shards, "o_col0", "o_cols", cfg.n_heads * cfg.head_dim)
            _partition(shards, "down_col0", "down_cols", cfg.ffn_dim)
            _partition(shards, "vocab_row0", "vocab_rows", cfg.vocab_size)
