"""Benchmark of the Q4_K decode GEMV (TinyLlama-1.1B
ffn_up, W = 5632 x 2048 Q4_K, x = f32[2048]).

One step = one GEMV over each of N_COPIES distinct, seeded copies of W
(415 MB in total, > 3x the 126 MB L2, so every timed launch streams its
weights from HBM), launched back to back with programmatic dependent launch
and replayed as one CUDA graph.  `value` is algorithmic bytes (W + x + y per
GEMV) per second with inputs resident in HBM; `e2e` is the same metric
through the C-ABI context API with host buffers (x copied H2D from pinned
memory, every y read back D2H, inside the timed region).

`--impl reference` times the reference's CPU algorithm (the oracle port in
oracle/; the Zig reference cannot be compiled here) on all host threads.
Multi-GPU (torchrun): every rank runs an independent replica (the GEMV
shards by rows with no exchange), value = all ranks' bytes / max rank time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, K = 5632, 2048
N_COPIES = 64
Q4_K = 12
W_BYTES = M * (K // 256) * 144
ALG_BYTES = W_BYTES + 4 * K + 4 * M  # per GEMV (6,518,784 B)
METRIC = "Q4_K GEMV HBM GB/s (TinyLlama ffn_up 5632x2048, batch 1)"
CONFIG = {"workload": "q4_k_gemv_5632x2048", "m": M, "k": K, "quant": "Q4_K", "weight_copies": N_COPIES,
          "l2": "inputs > L2: 64 distinct weight copies = 415 MB per step"}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    return int(os.environ.get("RANK", "0")), ws, int(os.environ.get("LOCAL_RANK", "0"))


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown," \
             "clocks_event_reasons.sw_power_cap"

    def __init__(self, index: int):
        self.index = index
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.p = None
        return self

    def __exit__(self, *a):
        self.out = ""
        if self.p:
            time.sleep(0.15)
            self.p.terminate()
            try:
                self.out, _ = self.p.communicate(timeout=5)
            except Exception:
                self.p.kill()

    def summary(self):
        rows = []
        for line in (self.out or "").splitlines():
            f = [s.strip() for s in line.split(",")]
            if len(f) >= 8:
                try:
                    rows.append((float(f[1]), float(f[2]), f[4:8]))
                except ValueError:
                    pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": rows[0][1], "reasons": reasons,
                "samples": len(rows)}


def make_weights(rank: int):
    from vantablack_b200 import synth as S
    rng = np.random.default_rng(1000 + rank)
    ws = [S.quant_tensor(rng, S.Q4_K, M, K) for _ in range(N_COPIES)]
    x = S.activations(rng, K)
    return ws, x


def cpu_gemv_rate(ws, x, budget_s: float, threads: int):
    """Oracle (reference algorithm, row-striped pool) GB/s on a bounded sample."""
    import oracle as O
    O.set_threads(threads)
    O.matmul(Q4_K, ws[0], x, M, K)
    n, t0 = 0, time.perf_counter()
    while True:
        O.matmul(Q4_K, ws[n % len(ws)], x, M, K)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return n * ALG_BYTES / el / 1e9, n


def run_reference(args):
    rank, ws_, _ = dist_env()
    if ws_ > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="env://")
        if rank != 0:
            dist.destroy_process_group()
            return
    import oracle as O
    ws, x = make_weights(0)
    threads = os.cpu_count() or 1
    O.set_threads(threads)
    per_step = 4  # bounded sample: 4 GEMVs (distinct copies) per step
    for s in range(args.warmup):
        for i in range(per_step):
            O.matmul(Q4_K, ws[(s * per_step + i) % N_COPIES], x, M, K)
    t0 = time.perf_counter()
    for s in range(args.steps):
        for i in range(per_step):
            O.matmul(Q4_K, ws[(s * per_step + i) % N_COPIES], x, M, K)
    el = time.perf_counter() - t0
    v = args.steps * per_step * ALG_BYTES / el / 1e9
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(CONFIG, per_step_sample=f"{per_step} GEMVs"),
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{per_step} GEMVs of 5632x2048 Q4_K per step, oracle port of "
                                       "simd.zig matmul_q4_k with pool.zig row striping"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    if ws_ > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_ours(args):
    import torch
    import torch.distributed as dist
    from vantablack_b200 import _lib, ops

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", init_method="env://", device_id=dev)
    lib = _lib.load()

    ws, x = make_weights(rank)
    dws = [torch.from_numpy(w).to(dev) for w in ws]
    dx = torch.from_numpy(x).to(dev)
    dys = [torch.empty(M, dtype=torch.float32, device=dev) for _ in range(N_COPIES)]
    stream = torch.cuda.Stream(device=dev)

    def step():
        for i in range(N_COPIES):
            ops.gemv(Q4_K, dws[i], dx, M, K, out=dys[i], pdl=True)

    with torch.cuda.stream(stream):
        step()
        stream.synchronize()
        ops.check_device_error()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            step()
        for _ in range(max(args.warmup, 3)):
            g.replay()
        stream.synchronize()

        # Device-timed region (CUDA events on the launching stream).
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        smi_idx = int(vis.split(",")[local]) if vis else local
        with ClockSampler(smi_idx) as clk:
            e0.record(stream)
            for _ in range(args.steps):
                g.replay()
            e1.record(stream)
            e1.synchronize()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = e0.elapsed_time(e1)
        t = torch.tensor([ms], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
        ops.check_device_error()

        # Correctness spot check of the timed outputs (one copy) vs the oracle.
        import oracle as O
        if rank == 0:
            ref = O.matmul(Q4_K, ws[0], x, M, K)
            err = float(np.abs(dys[0].cpu().numpy() - ref).max() / np.abs(ref).max())
        else:
            err = None

    # End-to-end through the C-ABI context API with host buffers.
    ctx = lib.vtb_cuda_init(local)
    wbufs = [lib.vtb_cuda_upload(ctx, w.ctypes.data, w.nbytes) for w in ws]
    xb = lib.vtb_cuda_alloc(ctx, K * 4, None)
    ybufs = [lib.vtb_cuda_alloc(ctx, M * 4, None) for _ in range(N_COPIES)]
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.empty(N_COPIES, M, dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 200))

    def e2e_step():
        _lib.check(lib.vtb_cuda_copy_h2d(ctx, xb, 0, hx.data_ptr(), K * 4), "h2d")
        for i in range(N_COPIES):
            _lib.check(lib.vtb_cuda_matmul_q4_k(ctx, ybufs[i], wbufs[i], 0, xb, M, K), "matmul")
        for i in range(N_COPIES):  # read back after one wait, as the Metal bridge reads after waitIdle
            _lib.check(lib.vtb_cuda_copy_d2h_async(ctx, hy[i].data_ptr(), ybufs[i], 0, M * 4), "d2h")
        _lib.check(lib.vtb_cuda_wait_idle(ctx), "wait_idle")

    for _ in range(3):
        e2e_step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    e2e_s = time.perf_counter() - t0
    tt = torch.tensor([e2e_s], device=dev)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    e2e_s = float(tt.item())
    for b in wbufs + ybufs + [xb]:
        lib.vtb_cuda_release(b)
    lib.vtb_cuda_destroy(ctx)

    # The 8B model metrics build the whole seeded weight set (~5 GB host memory)
    # on every rank, so they run at N <= 2 only; an error there is reported in
    # the line instead of failing the GEMV measurement.
    model = None
    if args.model_steps > 0 and world <= 2:
        try:
            model = model_metrics(rank, world, local, dist, args)
        except Exception as ex:  # noqa: BLE001 -- recorded in the JSON line
            model = {"error": f"{type(ex).__name__}: {ex}"[:300]}
    elif args.model_steps > 0:
        model = {"skipped": "Llama-3-8B tensor-parallel metrics run at 1 or 2 GPUs (host memory per rank)"}

    if rank == 0:
        hbm, peak_kind = peaks()
        launches = args.steps * N_COPIES
        value = world * launches * ALG_BYTES / (ms_max / 1e3) / 1e9
        per_launch_ms = ms / launches
        achieved = ALG_BYTES / (per_launch_ms / 1e3) / 1e9
        cpu_v, cpu_n = cpu_gemv_rate(ws, x, args.cpu_budget, os.cpu_count() or 1) if world == 1 else (None, 0)
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded GGUF Q4_K bytes)",
            "config": dict(CONFIG, parallelism=f"replicas x{world}"),
            "gpu_launches": launches,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "peak_kind": peak_kind,
                         "traffic": ALG_BYTES_TRAFFIC if ALG_BYTES_TRAFFIC else None},
            "e2e": {"value": world * e2e_steps * N_COPIES * ALG_BYTES / e2e_s / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": K * 4, "d2h_bytes_per_step": N_COPIES * M * 4},
            "clocks": clk.summary(),
            "max_rel_err_vs_oracle": err,
        }
        if model:
            line["config"]["model_8b"] = model
        if cpu_v is not None:
            line["cpu_baseline"] = {"value": cpu_v, "unit": "GB/s", "cores": os.cpu_count() or 1, "kind": "port",
                                    "sample": f"{cpu_n} GEMVs of 5632x2048 Q4_K over {args.cpu_budget:.0f} s, "
                                              "oracle port of simd.zig matmul_q4_k + pool.zig row striping"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


# DRAM bytes (read + write) of one config-1 launch, from the ncu capture summarised in
# profiles/q4k_gemv_5632x2048.md (6,545,152 read, ~0 written; algorithmic 6,518,784).
ALG_BYTES_TRAFFIC = 6545152


def model_metrics(rank: int, world: int, local: int, dist, args) -> dict:
    """BASELINE config 5 (Llama-3-8B architecture, random init, Q4_K_M-style):
    decode tok/s at batch 1 and 32 and prefill tok/s of a 2048-token prompt,
    tensor parallel over all ranks (NCCL).  Wall-clocked per call (each call
    ends with its logits/argmax on the host), max over ranks."""
    import torch
    from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState, HostWeights, TensorParallel

    def exchange(b: bytes) -> bytes:
        if world == 1:
            return b
        obj = [b]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    def tmax(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if world > 1:
            dist.barrier()

    cfg = LLAMA3_8B
    w = HostWeights(cfg, seed=8)
    ctx = Context(local)
    tp = TensorParallel(local, rank, world, exchange) if world > 1 else None
    m = CudaModel(ctx, w, tp)
    del w
    res = {"model": "llama3_8b_random_init_q4_k_m", "tp": world}
    rng = np.random.default_rng(1)
    # prefill: 2048-token prompt
    st = CudaState(m, 1, max_rows=2048)
    prompt = rng.integers(3, cfg.vocab_size, 2048)
    st.prefill(prompt[:64]); st.reset()  # warm-up
    barrier(); t0 = time.perf_counter()
    st.prefill(prompt)
    res["prefill_2048_tok_s"] = 2048 / tmax(time.perf_counter() - t0)
    # decode, batch 1, continuing after the prompt
    nxt = 5
    for _ in range(3):
        _, am = st.step([nxt], want_logits=False); nxt = int(am[0])
    n = args.model_steps
    barrier(); t0 = time.perf_counter()
    for _ in range(n):
        _, am = st.step([nxt], want_logits=False); nxt = int(am[0])
    res["decode_b1_tok_s"] = n / tmax(time.perf_counter() - t0)
    res["decode_b1_ctx"] = int(st.pos())
    st.close()
    # decode, batch 32 (32 independent sequences, one token each per step)
    st = CudaState(m, 32, max_rows=32)
    toks = rng.integers(3, cfg.vocab_size, 32)
    for _ in range(3):
        _, toks = st.step(toks, want_logits=False)
    nb = max(2, n // 4)
    barrier(); t0 = time.perf_counter()
    for _ in range(nb):
        _, toks = st.step(toks, want_logits=False)
    res["decode_b32_tok_s"] = 32 * nb / tmax(time.perf_counter() - t0)
    st.close()
    m.close()
    if tp:
        tp.close()
    ctx.close()
    return res


def run_profile_case(case: str) -> None:
    """Small, self-terminating workloads for ncu captures (one GPU)."""
    import torch
    from vantablack_b200 import ops, synth as S
    rng = np.random.default_rng(0)
    if case == "gemv":  # one config-1 launch, then one 311 MB streaming launch
        for m in (M, M * 48):
            w = torch.from_numpy(S.quant_tensor(rng, Q4_K, m, K)).cuda()
            x = torch.from_numpy(S.activations(rng, K)).cuda()
            ops.gemv(Q4_K, w, x, m, K)
            torch.cuda.synchronize()
    elif case == "gemv_q6k":  # Q6_K ffn_down 4096 x 14336, then the LM head 128256 x 4096 (431 MB)
        for m, k in ((4096, 14336), (128256, 4096)):
            w = torch.from_numpy(S.quant_tensor(rng, S.Q6_K, m, k)).cuda()
            x = torch.from_numpy(S.activations(rng, k)).cuda()
            ops.gemv(S.Q6_K, w, x, m, k)
            torch.cuda.synchronize()
    elif case == "gemm":  # config 3: Q4_K 14336 x 4096, B = 2048, bf16 mode, two launches
        m, k, b = 14336, 4096, 2048
        w = torch.from_numpy(S.quant_tensor(rng, Q4_K, m, k)).cuda()
        acts = torch.from_numpy(S.activations(rng, b, k)).cuda()
        for _ in range(2):
            ops.gemm(Q4_K, w, acts, m, k, precise=False)
    elif case == "gemm_b32":  # batch decode shape: Q6_K ffn_down 4096 x 14336, B = 32, precise mode, two launches
        m, k, b = 4096, 14336, 32
        w = torch.from_numpy(S.quant_tensor(rng, S.Q6_K, m, k)).cuda()
        acts = torch.from_numpy(S.activations(rng, b, k)).cuda()
        for _ in range(2):
            ops.gemm(S.Q6_K, w, acts, m, k, precise=True)
    elif case == "decode8b_b32":  # Llama-3-8B, 32 sequences: 3 decode steps of one token each
        from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState, HostWeights
        ctx = Context(0)
        st = CudaState(CudaModel(ctx, HostWeights(LLAMA3_8B, seed=1)), 32, max_rows=32)
        toks = np.arange(3, 35)
        for _ in range(3):
            _, toks = st.step(toks, want_logits=False)
    elif case in ("decode", "decode8b"):  # 128-token prefill + 5 decode steps (TinyLlama / Llama-3-8B)
        from vantablack_b200.model import LLAMA3_8B, TINYLLAMA, Context, CudaModel, CudaState, HostWeights
        ctx = Context(0)
        cfg = TINYLLAMA if case == "decode" else LLAMA3_8B
        st = CudaState(CudaModel(ctx, HostWeights(cfg, seed=1)), 1, max_rows=128)
        st.prefill(np.arange(3, 131))
        for i in range(5):
            st.step([5 + i], want_logits=False)
    else:
        raise SystemExit(f"unknown profile case {case}")
    torch.cuda.synchronize()
    ops.check_device_error()
    print("ok", case)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--model-steps", type=int, default=32, help="decode steps of the 8B model metrics (0 = skip)")
    ap.add_argument("--profile", choices=["gemv", "gemv_q6k", "gemm", "decode", "decode8b", "decode8b_b32", "gemm_b32"], help="run a small case for ncu and exit")
    args = ap.parse_args()
    if args.profile:
        run_profile_case(args.profile)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
