"""Tensor parallel on 2 GPUs (NCCL): TinyLlama-architecture prefill + greedy
decode split across the GPUs must produce the oracle's token ids.  Needs at
least 2 GPUs; skipped otherwise."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("source", ["host", "gguf"])
def test_tp2_tinyllama_greedy_identical(tmp_path, source):
    out = tmp_path / "tp.json"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={29533 + (source == 'gguf')}", os.path.join(HERE, "tp_worker.py"),
           str(out), "64"] + ([str(tmp_path / "tiny.gguf")] if source == "gguf" else [])
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["ranks_agree"]
    assert res["p2p"], "the all-reduce fell back to NCCL instead of NVLink peer memory"
    assert res["match"], (res["ids"], res["ids_ref"])
    assert res["logits_rel"] <= 1e-3
