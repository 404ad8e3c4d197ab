"""One rank of the multi-GPU (tensor-parallel) parity run; launched by
tests/test_tp_gpu.py through torch.distributed.run, one process per GPU.

Every rank builds the same seeded TinyLlama-architecture weights, uploads its
shard (vtb_cuda_model_create_tp; or, given a GGUF path as argv[3], rank 0
writes the weights to that file and every rank uploads its shard from it with
vtb_cuda_model_create_gguf_tp), runs a batched prefill of a 128-token prompt
and greedy decode; rank 0 compares the token ids with the CPU oracle and
writes the verdict to the JSON path given as argv[1]."""
import json
import os
import sys

import numpy as np
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    out_path, n_gen = sys.argv[1], int(sys.argv[2])
    gguf_path = sys.argv[3] if len(sys.argv) > 3 else None  # load the shards from one GGUF file
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    dist.init_process_group("gloo")

    def exchange(b: bytes) -> bytes:
        obj = [b]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    from vantablack_b200.model import TINYLLAMA, Context, CudaModel, CudaState, HostWeights, TensorParallel
    w = HostWeights(TINYLLAMA, seed=4)
    prompt = np.random.default_rng(44).integers(3, TINYLLAMA.vocab_size, 128)
    ctx = Context(local)
    tp = TensorParallel(local, rank, world, exchange)
    if gguf_path:  # rank 0 writes the file, every rank uploads its shard from it
        from vantablack_b200.gguf import GgufFile
        from vantablack_b200.model import write_synthetic_gguf
        if rank == 0:
            write_synthetic_gguf(gguf_path, TINYLLAMA, seed=4)
        dist.barrier()
        with GgufFile(gguf_path) as g:
            model = CudaModel.from_gguf(ctx, g, tp=tp)
    else:
        model = CudaModel(ctx, w, tp)
    st = CudaState(model, 1, max_rows=128)
    ids, logits = st.generate_greedy(prompt, n_gen, use_prefill=True)
    from vantablack_b200 import _lib
    _lib.check(_lib.load().vtb_cuda_check_device_error(), "device error word")  # no peer wait timed out
    res = {"rank": rank, "ids": ids, "p2p": st.tp_p2p()}
    if rank == 0:
        import oracle as O
        O.set_threads(os.cpu_count() or 8)
        ids_ref, lg_ref = O.Model(w).generate_greedy(prompt, n_gen, use_prefill=True)
        res.update(ids_ref=ids_ref, match=ids == ids_ref,
                   logits_rel=float(np.abs(logits - lg_ref).max() / np.abs(lg_ref).max()))
    gathered = [None] * world
    dist.all_gather_object(gathered, ids)
    if rank == 0:
        res["ranks_agree"] = all(g == ids for g in gathered)
        with open(out_path, "w") as f:
            json.dump(res, f)
    st.close()
    tp.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
