"""Host side of the Llama forward loop: configs, seeded random-init GGUF-style
weights, and the CUDA model/state handles behind the C ABI.

Names follow the reference: ``LlamaConfig`` (src/runtime/model.zig:40-149),
``LayerWeights`` (:172-189), ``step`` (forward.zig:119-172), ``prefill``
(prefill.zig:111-147).  Weights live on the host as numpy arrays standing in
for the GGUF mmap and are uploaded once by ``vtb_cuda_model_create``.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, replace

import numpy as np

from . import _lib
from .synth import Q4_K, Q6_K, activations, norm_weight, quant_tensor  # noqa: F401

MATS = ("attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down")


@dataclass(frozen=True)
class LlamaConfig:
    dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn_dim: int
    vocab_size: int
    max_seq: int
    rope_base: float = 10000.0
    rms_eps: float = 1e-5

    def with_(self, **kw) -> "LlamaConfig":
        return replace(self, **kw)


# TinyLlama-1.1B architecture.
TINYLLAMA = LlamaConfig(dim=2048, n_layers=22, n_heads=32, n_kv_heads=4, head_dim=64, ffn_dim=5632,
                        vocab_size=32000, max_seq=2048, rope_base=10000.0)
# Llama-3-8B architecture (max_seq covers a 2048-token prefill + 512 decode steps).
LLAMA3_8B = LlamaConfig(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336,
                        vocab_size=128256, max_seq=2560, rope_base=500000.0)

# Q4_K_M-style layout of both configs: ffn_down and output Q6_K, the rest Q4_K.
DEFAULT_QUANTS = {"attn_q": Q4_K, "attn_k": Q4_K, "attn_v": Q4_K, "attn_o": Q4_K, "ffn_gate": Q4_K,
                  "ffn_up": Q4_K, "ffn_down": Q6_K, "token_embd": Q4_K, "output": Q6_K}


# GGUF tensor names of the per-layer matrices (llama.cpp convention, read by
# Model.init in src/runtime/model.zig:201-243).
GGUF_NAMES = {"attn_q": "attn_q", "attn_k": "attn_k", "attn_v": "attn_v", "attn_o": "attn_output",
              "ffn_gate": "ffn_gate", "ffn_up": "ffn_up", "ffn_down": "ffn_down"}


def mat_shapes(cfg: LlamaConfig) -> dict:
    """(rows, k) of each per-layer matrix."""
    d, kvd, f = cfg.dim, cfg.n_kv_heads * cfg.head_dim, cfg.ffn_dim
    return {"attn_q": (d, d), "attn_k": (kvd, d), "attn_v": (kvd, d), "attn_o": (d, d),
            "ffn_gate": (f, d), "ffn_up": (f, d), "ffn_down": (d, f)}


def synth_tensors(cfg: LlamaConfig, seed: int = 0, quants: dict | None = None, emit: bool = True):
    """The seeded random-init tensors of a Llama config, in generation order.

    Yields (gguf_name, key, layer, quant, rows, k, array): per layer the seven
    matrices (MATS order), then attn_norm and ffn_norm (f32, quant 0); then
    token_embd, output_norm and output.  One PCG64 stream, so the bytes depend
    only on (cfg, seed, quants).  With emit=False only the metadata is yielded
    (array None, nothing generated)."""
    q = dict(DEFAULT_QUANTS, **(quants or {}))
    rng = np.random.default_rng(seed) if emit else None
    shp = mat_shapes(cfg)
    d = cfg.dim
    for i in range(cfg.n_layers):
        for n in MATS:
            rows, k = shp[n]
            yield (f"blk.{i}.{GGUF_NAMES[n]}.weight", n, i, q[n], rows, k,
                   quant_tensor(rng, q[n], rows, k) if emit else None)
        for n in ("attn_norm", "ffn_norm"):
            yield f"blk.{i}.{n}.weight", n, i, 0, 1, d, norm_weight(rng, d) if emit else None
    yield ("token_embd.weight", "token_embd", -1, q["token_embd"], cfg.vocab_size, d,
           quant_tensor(rng, q["token_embd"], cfg.vocab_size, d) if emit else None)
    yield "output_norm.weight", "output_norm", -1, 0, 1, d, norm_weight(rng, d) if emit else None
    yield ("output.weight", "output", -1, q["output"], cfg.vocab_size, d,
           quant_tensor(rng, q["output"], cfg.vocab_size, d) if emit else None)


class HostWeights:
    """Seeded random-init weights of a Llama config (numpy, host memory)."""

    def __init__(self, cfg: LlamaConfig, seed: int = 0, quants: dict | None = None):
        self.cfg = cfg
        self.layers = [{} for _ in range(cfg.n_layers)]
        self._absorb(synth_tensors(cfg, seed, quants))

    def _absorb(self, items):
        for _, key, layer, q, _, _, arr in items:
            if layer >= 0:
                self.layers[layer][key] = (q, arr) if key in MATS else arr
            elif key == "output_norm":
                self.output_norm = arr
            else:
                setattr(self, key, (q, arr))

    @classmethod
    def from_gguf(cls, path: str) -> "HostWeights":
        """Zero-copy numpy views of a llama GGUF file (np.memmap over the file,
        offsets from the library's own reader), e.g. for the CPU oracle."""
        from .gguf import GgufFile
        with GgufFile(path) as g:
            cfg = g.llama_config()
            base = g.info()["data_offset"]
            ts = {t["name"]: t for t in g.tensors()}
        mm = np.memmap(path, np.uint8, "r")
        self = cls.__new__(cls)
        self.cfg = cfg
        self.layers = [{} for _ in range(cfg.n_layers)]
        self._mm = mm
        items = []
        for name, key, layer, _, _, _, _ in synth_tensors(cfg, emit=False):
            t = ts.get(name) or (ts["token_embd.weight"] if name == "output.weight" else None)
            if t is None:
                raise KeyError(name)
            a = mm[base + t["rel_offset"]: base + t["rel_offset"] + t["size"]]
            if t["type"] == 0:
                a = a.view(np.float32)
            items.append((name, key, layer, t["type"], 0, 0, a))
        self._absorb(items)
        return self

    def nbytes(self) -> int:
        n = sum(a.nbytes for lw in self.layers for k, v in lw.items() for a in ([v[1]] if k in MATS else [v]))
        return n + self.token_embd[1].nbytes + self.output[1].nbytes + self.output_norm.nbytes


def write_synthetic_gguf(path: str, cfg: LlamaConfig, seed: int = 0, quants: dict | None = None) -> None:
    """Streams synth_tensors(cfg, seed, quants) into a llama GGUF file tensor by
    tensor (host memory holds one tensor at a time); the file loads through
    vtb_cuda_model_create_gguf[_tp] to the same weights as HostWeights(cfg, seed, quants)."""
    from .gguf import write_gguf
    meta = [("general.architecture", "str", "llama"),
            ("llama.context_length", "u32", cfg.max_seq),
            ("llama.embedding_length", "u32", cfg.dim),
            ("llama.block_count", "u32", cfg.n_layers),
            ("llama.feed_forward_length", "u32", cfg.ffn_dim),
            ("llama.attention.head_count", "u32", cfg.n_heads),
            ("llama.attention.head_count_kv", "u32", cfg.n_kv_heads),
            ("llama.rope.freq_base", "f32", cfg.rope_base),
            ("llama.attention.layer_norm_rms_epsilon", "f32", cfg.rms_eps),
            ("llama.vocab_size", "u32", cfg.vocab_size)]
    infos = [(name, q, [k] if q == 0 else [k, rows]) for name, _, _, q, rows, k, _ in
             synth_tensors(cfg, seed, quants, emit=False)]
    write_gguf(path, meta, infos, (a for *_, a in synth_tensors(cfg, seed, quants)))


class _CConfig(C.Structure):
    _fields_ = [(n, C.c_int32) for n in
                ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn_dim", "vocab_size", "max_seq")] + \
               [("rope_base", C.c_float), ("rms_eps", C.c_float)]


class _CLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in MATS] + [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p)] + \
               [("q_" + n, C.c_int32) for n in MATS]


_vp = C.c_void_p


def _lib_loaded():
    return _lib.load()


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


class Context:
    """A device context (vtb_cuda_init): one stream on one GPU."""

    def __init__(self, device: int = 0):
        self.lib = _lib_loaded()
        self.h = self.lib.vtb_cuda_init(device)
        if not self.h:
            raise _lib.VtbError(-5, "vtb_cuda_init")
        self.device = device

    def close(self):
        if self.h:
            self.lib.vtb_cuda_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TensorParallel:
    """One rank of a tensor-parallel group (NCCL communicator, vtb_cuda_tp_init).

    ``exchange(id_bytes) -> id_bytes`` shares rank 0's communicator id with the
    other ranks (e.g. a torch.distributed broadcast over gloo)."""

    def __init__(self, device: int, rank: int, world: int, exchange):
        self.lib = _lib_loaded()
        self.rank, self.world = rank, world
        buf = (C.c_uint8 * 128)()
        if rank == 0:
            _lib.check(self.lib.vtb_cuda_tp_unique_id(buf), "vtb_cuda_tp_unique_id")
        raw = exchange(bytes(buf))
        buf = (C.c_uint8 * 128).from_buffer_copy(raw)
        self.h = self.lib.vtb_cuda_tp_init(device, rank, world, buf)
        if not self.h:
            raise _lib.VtbError(-10, "vtb_cuda_tp_init")

    def close(self):
        if self.h:
            self.lib.vtb_cuda_tp_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TpShard(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("heads", "kv_heads", "q_row0", "q_rows", "kv_row0", "kv_rows", "ffn_row0",
                                         "ffn_rows", "o_col0", "o_cols", "down_col0", "down_cols", "vocab_row0",
                                         "vocab_rows")]


def shard_plan(cfg: LlamaConfig, rank: int, world: int, k_block: int = 256) -> TpShard:
    """vtb_cuda_tp_shard_plan (host-only)."""
    lib = _lib_loaded()
    cc = _CConfig(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.vocab_size,
                  cfg.max_seq, cfg.rope_base, cfg.rms_eps)
    out = TpShard()
    _lib.check(lib.vtb_cuda_tp_shard_plan(C.byref(cc), rank, world, k_block, C.byref(out)), "tp_shard_plan")
    return out


def tp_slice(quant: int, t: np.ndarray, rows: int, k: int, row0: int, nrows: int, col0: int, ncols: int):
    """vtb_cuda_tp_slice (host-only): a row x column block of a quantized tensor."""
    from .synth import row_bytes
    lib = _lib_loaded()
    out = np.empty(nrows * row_bytes(quant, ncols), np.uint8)
    _lib.check(lib.vtb_cuda_tp_slice(quant, _ptr(t), rows, k, row0, nrows, col0, ncols, _ptr(out)), "tp_slice")
    return out


class CudaModel:
    """Weights resident in HBM (vtb_cuda_model_create / _tp)."""

    def __init__(self, ctx: Context, w: HostWeights, tp: "TensorParallel | None" = None,
                 q8_activations: bool = False):
        self.ctx, self.cfg, self.lib, self.tp = ctx, w.cfg, ctx.lib, tp
        c = w.cfg
        cc = _CConfig(c.dim, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn_dim, c.vocab_size, c.max_seq,
                      c.rope_base, c.rms_eps)
        layers = (_CLayer * c.n_layers)()
        for i, lw in enumerate(w.layers):
            L = layers[i]
            for n in MATS:
                q, arr = lw[n]
                setattr(L, n, _ptr(arr))
                setattr(L, "q_" + n, q)
            L.attn_norm = _ptr(lw["attn_norm"])
            L.ffn_norm = _ptr(lw["ffn_norm"])
        qe, emb = w.token_embd
        qo, out = w.output
        self.h = self.lib.vtb_cuda_model_create_tp(ctx.h, tp.h if tp else None, C.byref(cc), C.cast(layers, _vp),
                                                   _ptr(emb), qe, _ptr(w.output_norm), _ptr(out), qo)
        if not self.h:
            raise _lib.VtbError(-1, "vtb_cuda_model_create")
        if q8_activations:  # Q8_0 projections on the Q8_0 x Q8_0 path (states created from now on)
            _lib.check(self.lib.vtb_cuda_model_set_q8_activations(self.h, 1), "set_q8_activations")

    @classmethod
    def from_gguf(cls, ctx: Context, gguf, max_seq: int = 0, tp: "TensorParallel | None" = None) -> "CudaModel":
        """Model.init from a GGUF file (vtb_cuda_model_create_gguf[_tp]); `gguf` is a
        vantablack_b200.gguf.GgufFile.  max_seq > 0 replaces the file's context length."""
        self = cls.__new__(cls)
        self.ctx, self.lib, self.tp = ctx, ctx.lib, tp
        cfg = gguf.llama_config()
        self.cfg = cfg.with_(max_seq=max_seq) if max_seq > 0 else cfg
        self.h = self.lib.vtb_cuda_model_create_gguf_tp(ctx.h, tp.h if tp else None, gguf.h, max_seq)
        if not self.h:
            raise _lib.VtbError(self.lib.vtb_cuda_last_status(), "vtb_cuda_model_create_gguf")
        return self

    @property
    def weight_bytes(self) -> int:
        return self.lib.vtb_cuda_model_weight_bytes(self.h)

    def close(self):
        if self.h:
            self.lib.vtb_cuda_model_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class CudaState:
    """KV cache + scratch for n_seqs sequences (vtb_cuda_state_create)."""

    def __init__(self, model: CudaModel, n_seqs: int = 1, max_rows: int = 256):
        self.model, self.lib, self.cfg = model, model.lib, model.cfg
        self.n_seqs = n_seqs
        self.h = self.lib.vtb_cuda_state_create(model.h, n_seqs, max(max_rows, n_seqs))
        if not self.h:
            raise _lib.VtbError(-4, "vtb_cuda_state_create")

    def close(self):
        if self.h:
            self.lib.vtb_cuda_state_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _lib.check(self.lib.vtb_cuda_state_reset(self.h), "reset")

    def pos(self, seq: int = 0) -> int:
        return self.lib.vtb_cuda_state_pos(self.h, seq)

    def tp_p2p(self) -> bool:
        """True when tensor-parallel all-reduces go over NVLink peer memory."""
        return bool(self.lib.vtb_cuda_state_tp_p2p(self.h))

    def step(self, tokens, want_logits: bool = True, graph: bool = True):
        """One token per sequence; returns (logits [n_seqs, vocab] or None, argmax [n_seqs])."""
        t = np.ascontiguousarray(np.atleast_1d(tokens), np.int32)
        assert t.size == self.n_seqs
        am = np.empty(self.n_seqs, np.int32)
        lg = np.empty((self.n_seqs, self.cfg.vocab_size), np.float32) if want_logits else None
        lp = _ptr(lg) if want_logits else None
        if graph:
            _lib.check(self.lib.vtb_cuda_step(self.h, _ptr(t), lp, _ptr(am)), "vtb_cuda_step")
        else:  # the vtable slot by slot
            _lib.check(self.lib.vtb_cuda_begin_token(self.h, _ptr(t)), "begin_token")
            for layer in range(self.cfg.n_layers):
                _lib.check(self.lib.vtb_cuda_layer_step(self.h, layer), "layer_step")
            _lib.check(self.lib.vtb_cuda_final_step(self.h), "final_step")
            _lib.check(self.lib.vtb_cuda_finalize_token(self.h, lp, _ptr(am)), "finalize_token")
        return lg, am

    def prefill(self, tokens, seq: int = 0, want_logits: bool = True):
        t = np.ascontiguousarray(tokens, np.int32)
        am = np.empty(1, np.int32)
        lg = np.empty(self.cfg.vocab_size, np.float32) if want_logits else None
        _lib.check(self.lib.vtb_cuda_prefill(self.h, seq, _ptr(t), t.size, _ptr(lg) if want_logits else None,
                                             _ptr(am)), "vtb_cuda_prefill")
        return lg, int(am[0])

    def sample(self, temperature: float, top_k: int = 0, top_p: float = 0.0, u=None, rows: int | None = None):
        """Sample the state's current logits on the device (vtb_cuda_state_sample):
        one token per row, one uniform draw per row; only the tokens are read back."""
        rows = self.n_seqs if rows is None else rows
        cfg = _lib.SamplerConfig(float(temperature), int(top_k), float(top_p), 0)
        ua = None if u is None else np.ascontiguousarray(np.atleast_1d(u), np.float32)
        out = np.empty(rows, np.int32)
        _lib.check(self.lib.vtb_cuda_state_sample(self.h, rows, C.byref(cfg), None if ua is None else _ptr(ua),
                                                  _ptr(out)), "vtb_cuda_state_sample")
        return out

    def generate_greedy(self, prompt, n_gen: int, use_prefill: bool = True):
        """Prompt then greedy decode of one sequence (n_seqs == 1)."""
        assert self.n_seqs == 1
        if use_prefill:
            logits, nxt = self.prefill(prompt)
        else:
            for tok in prompt:
                lg, am = self.step([int(tok)])
            logits, nxt = lg[0], int(am[0])
        out = []
        for _ in range(n_gen):
            out.append(nxt)
            lg, am = self.step([nxt])
            logits, nxt = lg[0], int(am[0])
        return out, logits
