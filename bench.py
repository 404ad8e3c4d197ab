"""Benchmark of vantablack's quantized-matmul hot path on B200.

Headline (the JSON line's `value`): the Q4_K decode GEMV at the TinyLlama-1.1B
ffn_up shape (W = 5632 x 2048 Q4_K, x = f32[2048]), the reference's
matmul_q4_k (src/kernels/simd.zig:245-273).  One step = one GEMV over each of
N_COPIES distinct seeded copies of W (415 MB, > 3x the 126 MB L2, so every
launch streams its weights from HBM), chained with programmatic dependent
launch in one CUDA graph, i.e. each GEMV is timed as it runs in a dependent
decode chain.  `e2e` is the same metric through the C-ABI context API with
host buffers (x copied H2D from pinned memory, every y read back D2H), driven
by a compiled caller (native/bridge_loop.c) with one segment per step.

The same line carries, under `workloads`:
  * gemv_sweep   -- Q6_K, Q8_0, Q8_0xQ8_0 and Q5_K GEMVs at the Llama-3-8B decode
                    shapes (GB/s, roofline fraction, oracle parity on sampled
                    rows, the oracle's GB/s on the host cores);
  * prefill_gemm -- the batched prefill GEMM (prefill.zig:325-378) for Q4_K
                    14336x4096 and Q6_K 4096x14336 at B in {87, 512, 2048}, in
                    bf16 and precise mode (TFLOP/s, fraction of the bf16 peak,
                    oracle parity on sampled rows, oracle GFLOP/s);
  * tinyllama    -- the TinyLlama-1.1B architecture end to end: 128-token
                    prefill + 256 greedy decode steps, greedy ids checked
                    against the oracle run on the same weights, GPU and oracle
                    tok/s;
  * llama3_8b    -- the Llama-3-8B architecture (Q4_K_M-style random init)
                    tensor parallel over all ranks: 2048-token prefill, 512
                    greedy decode steps at batch 1 whose ids and per-step top-16
                    logits are checked against the committed oracle fixture
                    tests/golden/llama3_8b_p2048_g512.npz, and batch-32 decode.
                    Every rank maps one GGUF file written once by rank 0 and
                    uploads only its shard.
The first three run on one GPU (N = 1 only); llama3_8b runs at every N.

`--impl reference` times the reference's CPU algorithm (the oracle port in
oracle/; the Zig reference cannot be compiled here) on the host cores.
Multi-GPU (torchrun): the headline GEMV runs as independent replicas (it has
no exchange step), value = all ranks' bytes / max rank time.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M, K = 5632, 2048
N_COPIES = 64
Q8_0, Q4_K, Q5_K, Q6_K = 8, 12, 13, 14
W_BYTES = M * (K // 256) * 144
ALG_BYTES = W_BYTES + 4 * K + 4 * M  # per GEMV: W + x + y = 6,518,784 B
METRIC = "Q4_K GEMV HBM GB/s (TinyLlama ffn_up 5632x2048, batch 1)"
CONFIG = {"workload": "q4_k_gemv_5632x2048", "m": M, "k": K, "quant": "Q4_K", "weight_copies": N_COPIES,
          "l2": "inputs > L2: 64 distinct weight copies = 415 MB per step"}
L2_BYTES = 126 * 2 ** 20
FIXTURE = os.path.join(ROOT, "tests", "golden", "llama3_8b_p2048_g512.npz")
GGUF_VERSION = 1  # bump when the synthetic weight generator changes


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def host_cores() -> int:
    """Physical cores of this host (the reference's pool sizes itself from them)."""
    try:
        import psutil
        n = psutil.cpu_count(logical=False)
        if n:
            return int(n)
    except Exception:
        pass
    return os.cpu_count() or 1


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
    """The reference's CPU Q4_K GEMV (oracle port of simd.zig matmul_q4_k with
    pool.zig row striping) on all physical host cores.  Each step is a bounded
    sample of GEMVs over distinct weight copies, sized from a calibration run
    so that the K timed steps together last at least ~2 s."""
    rank, ws_, _ = dist_env()
    if ws_ > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method="env://")
        if rank != 0:
            dist.destroy_process_group()
            return
    import oracle as O
    ws, x = make_weights(0)
    threads = host_cores()
    O.set_threads(threads)
    O.matmul(Q4_K, ws[0], x, M, K)
    t0 = time.perf_counter()
    for i in range(8):
        O.matmul(Q4_K, ws[i], x, M, K)
    t_one = (time.perf_counter() - t0) / 8
    steps = max(1, args.steps)
    per_step = max(4, math.ceil(0.05 / t_one), math.ceil(2.0 / (steps * t_one)))
    per_step = min(per_step, max(4, int(60.0 / (steps * t_one))))  # whole run within about a minute
    for s in range(args.warmup):
        for i in range(per_step):
            O.matmul(Q4_K, ws[(s * per_step + i) % N_COPIES], x, M, K)
    t0 = time.perf_counter()
    for s in range(steps):
        for i in range(per_step):
            O.matmul(Q4_K, ws[(s * per_step + i) % N_COPIES], x, M, K)
    el = time.perf_counter() - t0
    v = steps * per_step * ALG_BYTES / el / 1e9
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": args.warmup, "ms_per_step": el * 1e3 / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(CONFIG),
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"{per_step} GEMVs of 5632x2048 Q4_K per step ({el:.1f} s timed), oracle "
                                       "port of simd.zig matmul_q4_k with pool.zig row striping",
                             "reference_default_threads": (threads + 1) // 2},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    if ws_ > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


# DRAM bytes (read + write) of one config-1 launch, from the ncu capture summarised in
# profiles/q4k_gemv_5632x2048.md (6,545,152 read, ~0 written; algorithmic 6,518,784).
ALG_BYTES_TRAFFIC = 6545152


def time_graph(build, replays: int, stream):
    """Captures build() into a CUDA graph on `stream`, replays it 3 times
    untimed, then `replays` times between CUDA events; returns ms per replay."""
    import torch
    with torch.cuda.stream(stream):
        build()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            build()
        for _ in range(3):
            g.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(replays):
            g.replay()
        e1.record(stream)
        e1.synchronize()
    del g
    return e0.elapsed_time(e1) / replays


def mlx_gemv(dev, hbm: float, cpu_threads: int) -> dict:
    """MLX affine 4-bit GEMV (mlx.zig:283-330 matmulQ4; Metal matmul_mlx_q4,
    bridge.m:245-291) at 14336 x 4096, group 64, bf16 scales: 8 weight copies
    (264 MB > L2) in a CUDA graph; oracle parity and rate on 512 rows."""
    import torch
    import oracle as O
    from vantablack_b200 import ops, synth as S
    m, k, g = 14336, 4096, 64
    rng = np.random.default_rng(3)
    hw, hs, hb = S.mlx_tensor(rng, m, k, 4, g, True)
    base = tuple(torch.from_numpy(a).to(dev) for a in (hw, hs, hb))
    copies = [base] + [tuple(t.clone() for t in base) for _ in range(7)]
    hx = S.activations(rng, k)
    x = torch.from_numpy(hx).to(dev)
    nbytes = hw.nbytes + hs.nbytes + hb.nbytes
    stream = torch.cuda.Stream(device=dev)

    def build():
        for c in copies:
            ops.gemv_mlx(*c, x, m, k, 4, g, True)
    ms = time_graph(build, 10, stream)
    gbs = nbytes * len(copies) / (ms / 1e3) / 1e9
    y0 = ops.gemv_mlx(*base, x, m, k, 4, g, True).cpu().numpy()
    rows = 512
    O.set_threads(cpu_threads)
    sw, ss = hw[:rows * k // 2], hs[:rows * (k // g) * 2]
    sb = hb[:rows * (k // g) * 2]
    ref = O.mlx_matmul(sw, ss, sb, hx, rows, k, 4, g, True)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < 0.5:
        O.mlx_matmul(sw, ss, sb, hx, rows, k, 4, g, True)
        n += 1
    cpu_s = (time.perf_counter() - t0) / n
    ops.check_device_error()
    return {"shape": f"{m}x{k}", "group": g, "scales": "bf16", "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4),
            "us_per_launch": round(ms * 1e3 / len(copies), 2), "bytes_per_launch": nbytes,
            "max_rel_err_vs_oracle": float(np.abs(y0[:rows] - ref).max() / np.abs(ref).max()),
            "oracle_rows_checked": rows,
            "cpu_gbs_single_thread": round((sw.nbytes + ss.nbytes + sb.nbytes) / cpu_s / 1e9, 2)}


def sampler_leg(dev, cpu_threads: int) -> dict:
    """Device sampler (Sampler.sample, sampler.zig:44-104) at the Llama-3-8B
    vocabulary, batch 1 and 32: CUDA-event time per launch over 20 launches in
    a CUDA graph (replays re-sample the rows the first replay rewrote), the
    f32[vocab] read-back it replaces, and token parity with the oracle on
    fresh rows with the same draws."""
    import torch
    import oracle as O
    from vantablack_b200 import ops
    V = 128256
    stream = torch.cuda.Stream(device=dev)
    gen = torch.Generator(device=dev).manual_seed(4)
    out = {}
    for rows in (1, 32):
        lg = torch.randn(rows, V, device=dev, generator=gen) * 3
        u = np.random.default_rng(rows).random(rows, dtype=np.float32)
        for name, cfg in (("greedy", (0.0, 0, 0.0)), ("temp0.8", (0.8, 0, 0.0)),
                          ("temp0.7_k50_p0.95", (0.7, 50, 0.95))):
            bufs = [lg.clone() for _ in range(20)]

            def build():
                for b in bufs:
                    ops.sample(b, *cfg, u)
            ms = time_graph(build, 5, stream)
            fresh = lg.clone()
            tok = ops.sample(fresh, *cfg, u).cpu().numpy()
            host = lg.cpu().numpy()
            probs = fresh.cpu().numpy()
            agree, checked = 0, 0
            for r in range(min(rows, 4)):
                otok, op = O.sample(host[r], *cfg, float(u[r]))
                c = np.cumsum(op.astype(np.float64))
                if cfg[0] == 0.0 or np.abs(c - u[r]).min() >= 1e-3:
                    checked += 1
                    agree += int(otok == int(tok[r]))
            out[f"b{rows}_{name}"] = {"us_per_launch": round(ms * 1e3 / 20, 2), "tokens_equal_oracle": agree,
                                      "rows_checked": checked}
        h = torch.empty(rows, V, pin_memory=True)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(10):
                h.copy_(lg, non_blocking=True)
            e1.record(stream)
            e1.synchronize()
        out[f"b{rows}_logits_d2h_us"] = round(e0.elapsed_time(e1) * 1e3 / 10, 2)
    ops.check_device_error()
    return out


def gemv_sweep(dev, hbm: float, cpu_threads: int) -> dict:
    """Q6_K / Q8_0 / Q8_0xQ8_0 / Q5_K GEMVs at the Llama-3-8B decode shapes
    (simd.zig:159-190, 406-434, 290-347; dot_i8 :40-62 for the int8 variant), each a PDL
    chain over distinct weight copies totalling > 4x L2.  The weights are one
    seeded buffer per format (the largest shape's; smaller shapes use a prefix,
    which is whole blocks), copied on the device."""
    import torch
    import oracle as O
    from vantablack_b200 import ops, synth as S
    shapes = [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]
    rng = np.random.default_rng(2)
    stream = torch.cuda.Stream(device=dev)
    O.set_threads(cpu_threads)
    out = {}
    for quant, name in ((Q6_K, "q6_k"), (Q8_0, "q8_0"), (-1, "q8_0xq8_0"), (Q5_K, "q5_k")):
        q = Q8_0 if quant < 0 else quant
        if quant != -1:
            host = S.quant_tensor(rng, q, 128256, 4096)
        base = torch.from_numpy(host).to(dev)
        for m, k in shapes:
            nbytes = m * S.row_bytes(q, k)
            copies = max(1, min(64, math.ceil(4 * L2_BYTES / nbytes)))
            ws = [base[:nbytes]] + [base[:nbytes].clone() for _ in range(copies - 1)]
            x = torch.from_numpy(S.activations(rng, k)).to(dev)
            ys = [torch.empty(m, dtype=torch.float32, device=dev) for _ in range(copies)]
            xq = torch.empty(k, dtype=torch.int8, device=dev)
            dx = torch.empty(k // 32, dtype=torch.float32, device=dev)
            per = max(1, 32 // copies)

            def build():
                for _ in range(per):
                    for i in range(copies):
                        if quant == -1:
                            ops.gemv_q8_0_q8_0(ws[i], x, m, k, out=ys[i], scratch=(xq, dx), pdl=True)
                        else:
                            ops.gemv(q, ws[i], x, m, k, out=ys[i], pdl=True)
            ms = time_graph(build, 10, stream)
            launches = per * copies
            alg = nbytes + 4 * k + 4 * m
            gbs = alg * launches / (ms / 1e3) / 1e9
            # parity and the oracle's rate on a row sample (whole GEMV for small shapes)
            rows = min(m, max(64, (48 << 20) // S.row_bytes(q, k)))
            hw = host[:rows * S.row_bytes(q, k)]
            hx = x.cpu().numpy()
            fn = (lambda: O.matmul_q8_0_q8_0(hw, hx, rows, k)) if quant == -1 else (lambda: O.matmul(q, hw, hx, rows, k))
            ref = fn()
            n, t0 = 0, time.perf_counter()
            while time.perf_counter() - t0 < 0.5:
                fn()
                n += 1
            cpu_s = (time.perf_counter() - t0) / n
            got = ys[0][:rows].cpu().numpy()
            out[f"{name}_{m}x{k}"] = {
                "gbs": round(gbs, 1), "frac_hbm": round(gbs / hbm, 4), "us_per_launch": round(ms * 1e3 / launches, 3),
                "chain_copies": copies, "max_rel_err_vs_oracle": float(np.abs(got - ref).max() / np.abs(ref).max()),
                "oracle_rows_checked": rows,
                "cpu_gbs": round((rows * S.row_bytes(q, k) + 4 * k + 4 * rows) / cpu_s / 1e9, 2)}
            del ws, ys
        del base
        torch.cuda.empty_cache()
    ops.check_device_error()
    return out


def prefill_gemm(dev, bf16_peak: float, cpu_threads: int) -> dict:
    """The batched prefill GEMM (prefill.zig:325-378 matmulBatched) on tcgen05:
    out[B, m] = acts[B, k] . W^T for Q4_K 14336x4096 and Q6_K 4096x14336."""
    import torch
    import oracle as O
    from vantablack_b200 import ops, synth as S
    rng = np.random.default_rng(3)
    O.set_threads(cpu_threads)
    out = {}
    for q, name, m, k in ((Q4_K, "q4_k", 14336, 4096), (Q6_K, "q6_k", 4096, 14336)):
        host = S.quant_tensor(rng, q, m, k)
        w = torch.from_numpy(host).to(dev)
        ws = [w] + [w.clone() for _ in range(3)]  # 4 copies: weights rotate through > L2
        for B in (87, 512, 2048):
            acts_h = S.activations(rng, B, k)
            acts = torch.from_numpy(acts_h).to(dev)
            o = torch.empty(B, m, dtype=torch.float32, device=dev)
            # the oracle on a row sample (rows [0, r)): parity and its GFLOP/s
            r = 64
            t0 = time.perf_counter()
            ref = O.matmul_batched(q, host[:r * S.row_bytes(q, k)], acts_h, r, k, B)
            cpu_s = time.perf_counter() - t0
            for precise in (False, True):
                for i in range(2):
                    ops.gemm(q, ws[i], acts, m, k, precise=precise, out=o)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                reps = 20
                e0.record()
                for i in range(reps):
                    ops.gemm(q, ws[i % 4], acts, m, k, precise=precise, out=o)
                e1.record()
                e1.synchronize()
                ms = e0.elapsed_time(e1) / reps
                tf = 2.0 * B * m * k / (ms / 1e3) / 1e12
                got = o[:, :r].cpu().numpy()
                out[f"{name}_{m}x{k}_b{B}_{'precise' if precise else 'bf16'}"] = {
                    "tflops": round(tf, 1), "frac_bf16": round(tf / bf16_peak, 4), "ms": round(ms, 4),
                    "max_rel_err_vs_oracle": float(np.abs(got - ref).max() / np.abs(ref).max()),
                    "tolerance": 1e-4 if precise else 2e-2,
                    "cpu_gflops": round(2.0 * B * r * k / cpu_s / 1e9, 2), "oracle_rows_checked": r}
        del ws, w
        torch.cuda.empty_cache()
    ops.check_device_error()
    return out


def tinyllama(local: int, hbm: float, cpu_threads: int) -> dict:
    """The TinyLlama-1.1B architecture end to end (forward.zig step +
    prefill.zig prefillCpu): 128-token prompt, 256 greedy decode steps with
    the logits read back every step, ids compared with the oracle's."""
    import oracle as O
    from vantablack_b200.model import TINYLLAMA, Context, CudaModel, CudaState, HostWeights
    cfg = TINYLLAMA
    w = HostWeights(cfg, seed=4)
    prompt = np.random.default_rng(44).integers(3, cfg.vocab_size, 128)
    ctx = Context(local)
    m = CudaModel(ctx, w)
    st = CudaState(m, 1, max_rows=128)
    st.prefill(prompt[:16])
    st.reset()
    t0 = time.perf_counter()
    lg, nxt = st.prefill(prompt)
    t_pre = time.perf_counter() - t0
    ids = []
    t0 = time.perf_counter()
    for _ in range(256):
        ids.append(nxt)
        lgs, am = st.step([nxt])
        nxt = int(am[0])
    t_dec = time.perf_counter() - t0
    lg = lgs[0]
    st.close(); m.close(); ctx.close()
    O.set_threads(cpu_threads)
    om = O.Model(w)
    t0 = time.perf_counter()
    lgr = om.prefill(prompt)
    cpu_pre = time.perf_counter() - t0
    ids_ref = []
    t0 = time.perf_counter()
    for _ in range(256):
        nr = O.argmax(lgr)
        ids_ref.append(nr)
        lgr = om.step(nr)
    cpu_dec = time.perf_counter() - t0
    wbytes = w.nbytes() - w.token_embd[1].nbytes  # the embedding is gathered one row per token
    ctx_mid = 128 + 128
    kv = 2 * cfg.n_layers * ctx_mid * cfg.n_kv_heads * cfg.head_dim * 4
    dec = 256 / t_dec
    return {"prefill_128_tok_s": round(128 / t_pre, 1), "decode_b1_tok_s": round(dec, 1),
            "decode_frac_hbm": round(dec * (wbytes + kv) / 1e9 / hbm, 4),
            "ids_equal_oracle": ids == ids_ref,
            "first_diff": next((i for i, (a, b) in enumerate(zip(ids, ids_ref)) if a != b), None),
            "final_logits_rel_err": float(np.abs(lg - lgr).max() / np.abs(lgr).max()),
            "cpu_prefill_128_tok_s": round(128 / cpu_pre, 2), "cpu_decode_b1_tok_s": round(256 / cpu_dec, 2),
            "cpu_threads": cpu_threads, "timing": "wall clock per call; each decode step reads its logits back"}


def shared_gguf_path(name: str) -> str:
    d = "/dev/shm" if os.path.isdir("/dev/shm") and os.access("/dev/shm", os.W_OK) else None
    if d:
        st = os.statvfs(d)
        if st.f_bavail * st.f_frsize < 8 << 30:
            d = None
    import tempfile
    return os.path.join(d or tempfile.gettempdir(), name)


def llama3_8b(rank: int, world: int, local: int, dist, args, hbm: float, cpu_threads: int) -> dict:
    """Llama-3-8B architecture (Q4_K_M-style random init, the committed oracle
    fixture's weights) tensor parallel over all ranks: QKV and gate/up split by
    output rows, O and down along K with the all-reduce over NVLink peer
    memory, the LM head by vocabulary rows.  Rank 0 writes the GGUF file once
    (tensor by tensor); every rank maps it and uploads only its shard."""
    import torch
    from vantablack_b200.gguf import GgufFile
    from vantablack_b200.model import LLAMA3_8B, Context, CudaModel, CudaState, TensorParallel, \
        write_synthetic_gguf

    def barrier():
        if world > 1:
            dist.barrier()

    def tmax(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    g = np.load(FIXTURE)
    seed_w, seed_p = int(g["seed_w"]), int(g["seed_p"])
    n_prompt, n_fix = int(g["n_prompt"]), int(g["n_gen"])
    n_gen = max(1, min(args.model_steps, n_fix))
    path = shared_gguf_path(f"vtb_bench_llama3_8b_s{seed_w}_v{GGUF_VERSION}.gguf")
    res = {"model": "llama3_8b_random_init_q4_k_m", "tp": world, "gguf": path}
    t0 = time.perf_counter()
    if rank == 0 and not os.path.exists(path):
        write_synthetic_gguf(path, LLAMA3_8B, seed=seed_w)
    barrier()
    res["gguf_write_s"] = round(time.perf_counter() - t0, 1)

    def exchange(b: bytes) -> bytes:
        if world == 1:
            return b
        obj = [b]
        dist.broadcast_object_list(obj, src=0)
        return obj[0]

    ctx = Context(local)
    tp = TensorParallel(local, rank, world, exchange) if world > 1 else None
    t0 = time.perf_counter()
    with GgufFile(path) as gf:
        m = CudaModel.from_gguf(ctx, gf, max_seq=LLAMA3_8B.max_seq, tp=tp)
    res["upload_s"] = round(tmax(time.perf_counter() - t0), 1)
    prompt = np.random.default_rng(seed_p).integers(3, LLAMA3_8B.vocab_size, n_prompt)
    st = CudaState(m, 1, max_rows=n_prompt)
    res["p2p"] = bool(st.tp_p2p()) if world > 1 else None
    st.prefill(prompt[:64])
    st.reset()
    barrier()
    t0 = time.perf_counter()
    lg, _ = st.prefill(prompt)
    res["prefill_2048_tok_s"] = round(n_prompt / tmax(time.perf_counter() - t0), 1)
    # batch-1 decode over the fixture's steps; the logits come back to the host every
    # step (the sampler reads them there), and are checked after the timed loop
    ids, tops = [], []
    barrier()
    t0 = time.perf_counter()
    for step in range(n_gen):
        tops.append(lg[g["top_idx"][step]])
        nxt = int(np.argmax(lg))
        ids.append(nxt)
        lgs, _ = st.step([nxt])
        lg = lgs[0]
    dt = tmax(time.perf_counter() - t0)
    res["decode_b1_tok_s"] = round(n_gen / dt, 1)
    res["decode_b1_steps"] = n_gen
    ctx_mid = n_prompt + n_gen // 2
    wb = m.weight_bytes
    kv = 2 * LLAMA3_8B.n_layers * ctx_mid * LLAMA3_8B.n_kv_heads * LLAMA3_8B.head_dim * 4 / world
    res["decode_b1_frac_hbm_per_gpu"] = round((n_gen / dt) * (wb + kv) / 1e9 / hbm, 4)
    ref_ids = [int(v) for v in g["ids"][:n_gen]]
    errs = [float(np.abs(t - g["top_val"][i]).max() / np.abs(g["top_val"][i]).max()) for i, t in enumerate(tops)]
    res["parity"] = {"ids_equal": ids == ref_ids,
                     "first_diff": next((i for i, (a, b) in enumerate(zip(ids, ref_ids)) if a != b), None),
                     "max_top16_rel_err": max(errs), "tolerance": 1e-3,
                     "reference": "oracle fixture tests/golden/llama3_8b_p2048_g512.npz"}
    if n_gen == n_fix:
        lr = g["logits"]
        res["parity"]["final_logits_rel_err"] = float(np.abs(lg - lr).max() / np.abs(lr).max())
    st.close()
    # batch-32 decode: 32 independent sequences, one token each per step
    st = CudaState(m, 32, max_rows=32)
    toks = np.random.default_rng(1).integers(3, LLAMA3_8B.vocab_size, 32)
    for _ in range(3):
        _, toks = st.step(toks, want_logits=False)
    nb = 64
    barrier()
    t0 = time.perf_counter()
    for _ in range(nb):
        _, toks = st.step(toks, want_logits=False)
    dt32 = tmax(time.perf_counter() - t0)
    res["decode_b32_tok_s"] = round(32 * nb / dt32, 1)
    res["decode_b32_frac_hbm_per_gpu"] = round((nb / dt32) * wb / 1e9 / hbm, 4)
    st.close()
    m.close()
    if tp:
        tp.close()
    ctx.close()
    res["timing"] = "wall clock per call, max over ranks; decode reads logits (b1) or argmax ids (b32) back per step"
    if rank == 0 and world == 1:
        res["cpu_baseline"] = llama3_8b_cpu(path, cpu_threads)
    return res


def llama3_8b_cpu(path: str, threads: int) -> dict:
    """The oracle's 8B forward on the host cores over the same GGUF (memmap):
    decode tok/s at batch 1 over a few steps after a 16-token prompt, and
    prefill tok/s of that prompt."""
    import oracle as O
    from vantablack_b200.model import HostWeights
    O.set_threads(threads)
    w = HostWeights.from_gguf(path)
    om = O.Model(w)
    prompt = np.arange(3, 19)
    t0 = time.perf_counter()
    lg = om.prefill(prompt)
    t_pre = time.perf_counter() - t0
    n = 4
    t0 = time.perf_counter()
    for _ in range(n):
        lg = om.step(O.argmax(lg))
    t_dec = time.perf_counter() - t0
    return {"decode_b1_tok_s": round(n / t_dec, 3), "prefill_16_tok_s": round(16 / t_pre, 2), "threads": threads,
            "kind": "port", "sample": f"16-token prompt + {n} decode steps (context < 32)"}


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
    hbm, bf16, peak_kind = peaks()
    cores = host_cores()

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
        y0 = dys[0].cpu().numpy()
    del g

    # End-to-end through the C-ABI context API with host buffers, driven by a
    # compiled caller (vantablack_b200/native/bridge_loop.c) as the reference's
    # Zig host drives its bridge: per step the activations go in from pinned
    # host memory, the 64 matmuls run as one segment (vtb_cuda_segment_*, the
    # vtb_metal_segment_* counterpart) and every result comes back to pinned
    # host memory before the step ends.  The same loop with the one-shot calls
    # is recorded beside it.
    import ctypes
    ctx = lib.vtb_cuda_init(local)
    wbufs = [lib.vtb_cuda_upload(ctx, w.ctypes.data, w.nbytes) for w in ws]
    xb = lib.vtb_cuda_alloc(ctx, K * 4, None)
    ybufs = [lib.vtb_cuda_alloc(ctx, M * 4, None) for _ in range(N_COPIES)]
    hx = torch.from_numpy(x).pin_memory()
    hy = torch.empty(N_COPIES, M, dtype=torch.float32).pin_memory()
    e2e_steps = max(3, min(args.steps, 200))
    loop = ctypes.CDLL(os.path.join(ROOT, "vantablack_b200", "libvtbbridgeloop.so"))
    loop.vtb_bench_bridge_q4k.restype = ctypes.c_int
    loop.vtb_bench_bridge_q4k.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_size_t, ctypes.c_size_t,
                                                                  ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                                  ctypes.POINTER(ctypes.c_double)]
    warr = (ctypes.c_void_p * N_COPIES)(*wbufs)
    yarr = (ctypes.c_void_p * N_COPIES)(*ybufs)

    def bridge_loop(segment: int) -> float:
        if world > 1:
            dist.barrier()
        sec = ctypes.c_double(0.0)
        rc = loop.vtb_bench_bridge_q4k(ctx, warr, yarr, xb, hx.data_ptr(), hy.data_ptr(), N_COPIES, M, K,
                                       max(args.warmup, 3), e2e_steps, segment, ctypes.byref(sec))
        if rc != 0:
            _lib.check(rc, "native bridge loop")
        tt = torch.tensor([sec.value], device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return float(tt.item())

    e2e_s = bridge_loop(1)
    e2e_one_shot_s = bridge_loop(0)
    e2e_ok = bool(np.array_equal(hy[0].numpy(), y0))
    for b in wbufs + ybufs + [xb]:
        lib.vtb_cuda_release(b)
    lib.vtb_cuda_destroy(ctx)
    del dws, dys
    torch.cuda.empty_cache()

    # Correctness spot check of the timed outputs (one copy) vs the oracle -- after
    # the host-timed e2e loop, so the oracle's worker threads never compete with it.
    import oracle as O
    if rank == 0:
        O.set_threads(cores)
        ref = O.matmul(Q4_K, ws[0], x, M, K)
        err = float(np.abs(y0 - ref).max() / np.abs(ref).max())
    else:
        err = None

    work = {}

    def leg(name, fn):
        try:
            work[name] = fn()
        except Exception as ex:  # noqa: BLE001 -- recorded in the JSON line
            work[name] = {"error": f"{type(ex).__name__}: {ex}"[:300]}

    if world == 1 and not args.no_sweeps:
        leg("gemv_sweep", lambda: gemv_sweep(dev, hbm, cores))
        leg("prefill_gemm", lambda: prefill_gemm(dev, bf16, cores))
        leg("tinyllama", lambda: tinyllama(local, hbm, cores))
        leg("mlx_q4_gemv", lambda: mlx_gemv(dev, hbm, cores))
        leg("sampler", lambda: sampler_leg(dev, cores))
    if args.model_steps > 0:
        leg("llama3_8b", lambda: llama3_8b(rank, world, local, dist, args, hbm, cores))

    if rank == 0:
        launches = args.steps * N_COPIES
        value = world * launches * ALG_BYTES / (ms_max / 1e3) / 1e9
        per_launch_ms = ms / launches
        achieved = ALG_BYTES / (per_launch_ms / 1e3) / 1e9
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
                    "h2d_bytes_per_step": K * 4, "d2h_bytes_per_step": N_COPIES * M * 4,
                    "caller": "compiled C loop (native/bridge_loop.c): vtb_cuda_segment_* per step, "
                              "host buffers pinned, wall clock",
                    "one_shot_value": world * e2e_steps * N_COPIES * ALG_BYTES / e2e_one_shot_s / 1e9,
                    "results_equal_device_run": e2e_ok},
            "clocks": clk.summary(),
            "max_rel_err_vs_oracle": err,
            "workloads": work,
        }
        if world == 1:
            cpu_v, cpu_n = cpu_gemv_rate(ws, x, args.cpu_budget, cores)
            cpu_half, _ = cpu_gemv_rate(ws, x, min(args.cpu_budget, 3.0), (cores + 1) // 2)
            line["cpu_baseline"] = {"value": cpu_v, "unit": "GB/s", "cores": cores, "kind": "port",
                                    "sample": f"{cpu_n} GEMVs of 5632x2048 Q4_K over {args.cpu_budget:.0f} s, "
                                              "oracle port of simd.zig matmul_q4_k + pool.zig row striping",
                                    "reference_default_threads": (cores + 1) // 2,
                                    "value_at_reference_default_threads": cpu_half}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


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
    elif case == "gemv_chain":  # the bench's chained config-1 launches, 3 replays of 64
        ws = [torch.from_numpy(S.quant_tensor(rng, Q4_K, M, K)).cuda() for _ in range(N_COPIES)]
        x = torch.from_numpy(S.activations(rng, K)).cuda()
        ys = [torch.empty(M, device="cuda") for _ in range(N_COPIES)]
        for _ in range(3):
            for i in range(N_COPIES):
                ops.gemv(Q4_K, ws[i], x, M, K, out=ys[i], pdl=True)
    elif case == "gemv_q6k":  # Q6_K ffn_down 4096 x 14336, then the LM head 128256 x 4096 (431 MB)
        for m, k in ((4096, 14336), (128256, 4096)):
            w = torch.from_numpy(S.quant_tensor(rng, S.Q6_K, m, k)).cuda()
            x = torch.from_numpy(S.activations(rng, k)).cuda()
            ops.gemv(S.Q6_K, w, x, m, k)
            torch.cuda.synchronize()
    elif case == "gemv_q8":  # Q8_0 4096 x 14336 and 14336 x 4096 (f32 x), then Q8_0 x Q8_0 at 14336 x 4096
        for m, k in ((4096, 14336), (14336, 4096)):
            w = torch.from_numpy(S.quant_tensor(rng, Q8_0, m, k)).cuda()
            x = torch.from_numpy(S.activations(rng, k)).cuda()
            ops.gemv(Q8_0, w, x, m, k)
            torch.cuda.synchronize()
        ops.gemv_q8_0_q8_0(w, x, m, k)
        torch.cuda.synchronize()
    elif case == "gemm":  # Q4_K 14336 x 4096, B = 2048, bf16 mode, two launches
        m, k, b = 14336, 4096, 2048
        w = torch.from_numpy(S.quant_tensor(rng, Q4_K, m, k)).cuda()
        acts = torch.from_numpy(S.activations(rng, b, k)).cuda()
        for _ in range(2):
            ops.gemm(Q4_K, w, acts, m, k, precise=False)
    elif case == "gemm_precise":  # the model prefill's mode: Q4_K 14336 x 4096, B = 2048, precise, two launches
        m, k, b = 14336, 4096, 2048
        w = torch.from_numpy(S.quant_tensor(rng, Q4_K, m, k)).cuda()
        acts = torch.from_numpy(S.activations(rng, b, k)).cuda()
        for _ in range(2):
            ops.gemm(Q4_K, w, acts, m, k, precise=True)
    elif case == "gemm_b32":  # batch decode shape: Q6_K ffn_down 4096 x 14336, B = 32, precise mode, two launches
        m, k, b = 4096, 14336, 32
        w = torch.from_numpy(S.quant_tensor(rng, S.Q6_K, m, k)).cuda()
        acts = torch.from_numpy(S.activations(rng, b, k)).cuda()
        for _ in range(2):
            ops.gemm(S.Q6_K, w, acts, m, k, precise=True)
    elif case == "gemm_b32_q4k":  # batch decode shape: Q4_K gate|up 28672 x 4096, B = 32, precise mode, two launches
        m, k, b = 28672, 4096, 32
        w = torch.from_numpy(S.quant_tensor(rng, Q4_K, m, k)).cuda()
        acts = torch.from_numpy(S.activations(rng, b, k)).cuda()
        for _ in range(2):
            ops.gemm(Q4_K, w, acts, m, k, precise=True)
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
    elif case == "mlx":  # MLX 4-bit GEMV at 14336 x 4096 (G 64, bf16), 8 weight copies > L2, in a CUDA graph
        m, k, g = 14336, 4096, 64
        copies = []
        for _ in range(8):
            w, sc, bi = S.mlx_tensor(rng, m, k, 4, g, True)
            copies.append(tuple(torch.from_numpy(a).cuda() for a in (w, sc, bi)))
        x = torch.from_numpy(S.activations(rng, k)).cuda()
        nbytes = sum(t.numel() for t in copies[0])
        for c in copies:
            ops.gemv_mlx(*c, x, m, k, 4, g, True)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for c in copies:
                ops.gemv_mlx(*c, x, m, k, 4, g, True)
        for _ in range(3):
            graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / 80
        print(f"MLX-Q4 GEMV {m}x{k}: {us:.2f} us per launch, {nbytes / us / 1e3:.0f} GB/s ({nbytes} bytes)")
    elif case == "sampler":  # device sampler: 20 launches per (vocabulary, rows, config), D2H beside it
        for rows, n in ((1, 32000), (1, 128256), (32, 128256)):
            lg = torch.randn(rows, n, device="cuda") * 3
            u = np.random.default_rng(0).random(rows, dtype=np.float32)
            for cfg in ((0.0, 0, 0.0), (0.8, 0, 0.0), (0.8, 40, 0.0), (0.8, 0, 0.9), (0.7, 50, 0.95)):
                bufs = [lg.clone() for _ in range(20)]
                for b in bufs[:3]:
                    ops.sample(b, *cfg, u)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for b in bufs[3:]:
                    ops.sample(b, *cfg, u)
                e1.record()
                torch.cuda.synchronize()
                print(f"rows {rows} n {n} cfg {cfg}: {e0.elapsed_time(e1) / 17 * 1000:.1f} us per call (host-paced)")
            h = torch.empty(rows, n, pin_memory=True)
            e0.record()
            for _ in range(17):
                h.copy_(lg, non_blocking=True)
            e1.record()
            torch.cuda.synchronize()
            print(f"rows {rows} n {n}: D2H of the logits {e0.elapsed_time(e1) / 17 * 1000:.1f} us")
    else:
        raise SystemExit(f"unknown profile case {case}")
    torch.cuda.synchronize()
    ops.check_device_error()
    print("ok", case)


PROFILE_CASES = ["gemv", "gemv_chain", "gemv_q6k", "gemv_q8", "gemm", "gemm_precise", "gemm_b32", "gemm_b32_q4k", "decode", "decode8b",
                 "decode8b_b32", "sampler", "mlx"]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--model-steps", type=int, default=512,
                    help="batch-1 decode steps of the Llama-3-8B workload (<= 512; 0 = skip it)")
    ap.add_argument("--no-sweeps", action="store_true", help="skip the single-GPU workload sweeps")
    ap.add_argument("--profile", choices=PROFILE_CASES, help="run a small case for ncu and exit")
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
