"""ctypes front end of the CPU oracle (oracle/vtb_oracle.c).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, by ``__graft_entry__.smoke()``
as the checker, and by ``bench.py`` for the timed CPU baseline.  The product
(``vantablack_b200``) never imports it.

The C library restates the reference's CPU kernels bit-for-bit (see the file
header of vtb_oracle.c for the citation map and how the restatement is
pinned).  The reference itself is Zig 0.16 and cannot be compiled here, so
there is no ``oracle/_ref`` build.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libvtb_oracle.so")

F32, Q8_0, Q4_K, Q5_K, Q6_K, TQ2_0 = 0, 8, 12, 13, 14, 32

_u8p = C.POINTER(C.c_uint8)
_f32p = C.POINTER(C.c_float)
_i8p = C.POINTER(C.c_int8)
_i32p = C.POINTER(C.c_int32)
_u32p = C.POINTER(C.c_uint32)
_sz = C.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def _load():
    if not os.path.exists(LIB_PATH):
        build()
    lib = C.CDLL(LIB_PATH)
    sig = {
        "vtbo_f16_to_f32": (C.c_float, [C.c_uint16]),
        "vtbo_dot_f32": (C.c_float, [_f32p, _f32p, _sz]),
        "vtbo_dot_i8": (C.c_int32, [_i8p, _i8p, _sz]),
        "vtbo_dequant": (C.c_int, [C.c_int, _u8p, _f32p, _sz]),
        "vtbo_row_bytes": (_sz, [C.c_int, _sz]),
        "vtbo_matmul_q8_0": (None, [_f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_matmul_q4_k": (None, [_f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_matmul_q5_k": (None, [_f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_matmul_q6_k": (None, [_f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_matmul_tq2_0": (None, [_f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_pool_init": (C.c_int, [C.c_int]),
        "vtbo_pool_threads": (C.c_int, []),
        "vtbo_pool_shutdown": (None, []),
        "vtbo_matmul": (C.c_int, [C.c_int, _f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_matmul_batched": (C.c_int, [C.c_int, _f32p, _u8p, _f32p, _sz, _sz, _sz]),
        "vtbo_quantize_q8_0": (None, [_f32p, _sz, _i8p, _f32p]),
        "vtbo_q8_0_block_dots": (None, [_i32p, _u8p, _i8p, _sz, _sz]),
        "vtbo_matmul_q8_0_q8_0": (C.c_int, [_f32p, _u8p, _f32p, _sz, _sz]),
        "vtbo_rms_norm": (None, [_f32p, _f32p, _sz, C.c_float]),
        "vtbo_rope": (None, [_f32p, _sz, _sz, C.c_float]),
        "vtbo_softmax": (None, [_f32p, _sz]),
        "vtbo_swiglu": (None, [_f32p, _f32p, _sz]),
        "vtbo_geglu": (None, [_f32p, _f32p, _sz]),
        "vtbo_add_into": (None, [_f32p, _f32p, _sz]),
        "vtbo_argmax": (_sz, [_f32p, _sz]),
        "vtbo_mlx_dequant": (C.c_int, [_f32p, _u8p, _u8p, _u8p, _sz, _sz, C.c_uint, _sz, C.c_int]),
        "vtbo_mlx_matmul": (C.c_int, [_f32p, _u8p, _u8p, _u8p, _f32p, _sz, _sz, C.c_uint, _sz, C.c_int]),
        "vtbo_sample": (C.c_uint32, [_f32p, _sz, C.c_float, _sz, C.c_float, C.c_float]),
        "vtbo_model_create": (C.c_void_p, [C.c_void_p, C.c_void_p, _u8p, C.c_int, _f32p, _u8p, C.c_int]),
        "vtbo_model_destroy": (None, [C.c_void_p]),
        "vtbo_model_set_q8_activations": (None, [C.c_void_p, C.c_int]),
        "vtbo_model_reset": (None, [C.c_void_p]),
        "vtbo_model_pos": (C.c_int64, [C.c_void_p]),
        "vtbo_step": (C.c_int, [C.c_void_p, C.c_uint32, _f32p]),
        "vtbo_prefill": (C.c_int, [C.c_void_p, _u32p, _sz, _f32p]),
        "vtbo_kv_keys": (_f32p, [C.c_void_p, _sz]),
        "vtbo_kv_values": (_f32p, [C.c_void_p, _sz]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(t)


def set_threads(n: int) -> None:
    """Size the persistent row-striping pool (pool.zig:44-78)."""
    if lib.vtbo_pool_init(int(n)) != 0:
        raise RuntimeError("oracle thread pool init failed")


def threads() -> int:
    return lib.vtbo_pool_threads()


def f16_to_f32(bits: int) -> float:
    return lib.vtbo_f16_to_f32(bits)


def row_bytes(quant: int, k: int) -> int:
    return lib.vtbo_row_bytes(quant, k)


def dequant(quant: int, w: np.ndarray, n: int) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.empty(n, np.float32)
    if lib.vtbo_dequant(quant, _p(w, _u8p), _p(out, _f32p), n) != 0:
        raise ValueError(f"unsupported quant {quant}")
    return out


def dot_f32(a: np.ndarray, b: np.ndarray) -> float:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    return lib.vtbo_dot_f32(_p(a, _f32p), _p(b, _f32p), a.size)


def dot_i8(a: np.ndarray, b: np.ndarray) -> int:
    a = np.ascontiguousarray(a, np.int8)
    b = np.ascontiguousarray(b, np.int8)
    return lib.vtbo_dot_i8(_p(a, _i8p), _p(b, _i8p), a.size)


_SINGLE = {Q8_0: "vtbo_matmul_q8_0", Q4_K: "vtbo_matmul_q4_k", Q5_K: "vtbo_matmul_q5_k", Q6_K: "vtbo_matmul_q6_k",
           TQ2_0: "vtbo_matmul_tq2_0"}


def matmul_single(quant: int, w: np.ndarray, x: np.ndarray, m: int, k: int) -> np.ndarray:
    """The per-quant simd.zig kernel on one thread."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    out = np.empty(m, np.float32)
    getattr(lib, _SINGLE[quant])(_p(out, _f32p), _p(w, _u8p), _p(x, _f32p), m, k)
    return out


def matmul(quant: int, w: np.ndarray, x: np.ndarray, m: int, k: int) -> np.ndarray:
    """matmulRuntime's CPU branch: rows striped over the pool."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    out = np.empty(m, np.float32)
    if lib.vtbo_matmul(quant, _p(out, _f32p), _p(w, _u8p), _p(x, _f32p), m, k) != 0:
        raise ValueError("bad matmul arguments")
    return out


def matmul_batched(quant: int, w: np.ndarray, acts: np.ndarray, m: int, k: int, B: int) -> np.ndarray:
    """prefill.zig matmulBatched: out[B, m]."""
    acts = np.ascontiguousarray(acts, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    out = np.empty((B, m), np.float32)
    if lib.vtbo_matmul_batched(quant, _p(out, _f32p), _p(w, _u8p), _p(acts, _f32p), m, k, B) != 0:
        raise ValueError("bad batched matmul arguments")
    return out


def quantize_q8_0(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    qs = np.empty(x.size, np.int8)
    d = np.empty(x.size // 32, np.float32)
    lib.vtbo_quantize_q8_0(_p(x, _f32p), x.size, _p(qs, _i8p), _p(d, _f32p))
    return qs, d


def q8_0_block_dots(w: np.ndarray, xq: np.ndarray, m: int, k: int) -> np.ndarray:
    dots = np.empty((m, k // 32), np.int32)
    lib.vtbo_q8_0_block_dots(_p(dots, _i32p), _p(np.ascontiguousarray(w, np.uint8), _u8p),
                             _p(np.ascontiguousarray(xq, np.int8), _i8p), m, k)
    return dots


def matmul_q8_0_q8_0(w: np.ndarray, x: np.ndarray, m: int, k: int) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.uint8)
    out = np.empty(m, np.float32)
    if lib.vtbo_matmul_q8_0_q8_0(_p(out, _f32p), _p(w, _u8p), _p(x, _f32p), m, k) != 0:
        raise ValueError("bad q8_0 x q8_0 arguments")
    return out


def rms_norm(x, w, eps):
    x = np.array(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    lib.vtbo_rms_norm(_p(x, _f32p), _p(w, _f32p), x.size, eps)
    return x


def rope(x, pos, base):
    x = np.array(x, np.float32)
    lib.vtbo_rope(_p(x, _f32p), x.size, pos, base)
    return x


def softmax(x):
    x = np.array(x, np.float32)
    lib.vtbo_softmax(_p(x, _f32p), x.size)
    return x


def swiglu(g, u):
    g = np.array(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    lib.vtbo_swiglu(_p(g, _f32p), _p(u, _f32p), g.size)
    return g


def geglu(g, u):
    g = np.array(g, np.float32)
    u = np.ascontiguousarray(u, np.float32)
    lib.vtbo_geglu(_p(g, _f32p), _p(u, _f32p), g.size)
    return g


def add_into(a, b):
    a = np.array(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    lib.vtbo_add_into(_p(a, _f32p), _p(b, _f32p), a.size)
    return a


def argmax(x) -> int:
    x = np.ascontiguousarray(x, np.float32)
    return lib.vtbo_argmax(_p(x, _f32p), x.size)


def mlx_dequant(w, scales, biases, rows: int, k: int, bits: int, group: int, bf16: bool) -> np.ndarray:
    """dequantRow (mlx.zig:62-135) over `rows` rows -> f32 [rows, k]."""
    out = np.empty((rows, k), np.float32)
    rc = lib.vtbo_mlx_dequant(_p(out, _f32p), _p(np.ascontiguousarray(w, np.uint8), _u8p),
                              _p(np.ascontiguousarray(scales, np.uint8), _u8p),
                              _p(np.ascontiguousarray(biases, np.uint8), _u8p), rows, k, bits, group, int(bf16))
    if rc:
        raise ValueError("unsupported MLX arguments")
    return out


def mlx_matmul(w, scales, biases, x, m: int, k: int, bits: int, group: int, bf16: bool) -> np.ndarray:
    """matmul (mlx.zig:213-235): y[m] = W . x."""
    out = np.empty(m, np.float32)
    xa = np.ascontiguousarray(x, np.float32)
    rc = lib.vtbo_mlx_matmul(_p(out, _f32p), _p(np.ascontiguousarray(w, np.uint8), _u8p),
                             _p(np.ascontiguousarray(scales, np.uint8), _u8p),
                             _p(np.ascontiguousarray(biases, np.uint8), _u8p), _p(xa, _f32p), m, k, bits, group,
                             int(bf16))
    if rc:
        raise ValueError("unsupported MLX arguments")
    return out


def sample(logits, temperature: float, top_k: int, top_p: float, u: float):
    """Sampler.sample (sampler.zig:44-104) with the draw ``u`` supplied.
    Returns (token, logits after the in-place pipeline)."""
    a = np.ascontiguousarray(logits, dtype=np.float32).copy()
    t = lib.vtbo_sample(_p(a, _f32p), a.size, float(temperature), int(top_k), float(top_p), float(u))
    return int(t), a


class _Config(C.Structure):
    _fields_ = [(n, C.c_int64) for n in
                ("dim", "n_layers", "n_heads", "n_kv_heads", "head_dim", "ffn_dim", "vocab_size", "max_seq")] + \
               [("rope_base", C.c_float), ("rms_eps", C.c_float)]


_LAYER_MATS = ("attn_q", "attn_k", "attn_v", "attn_o", "ffn_gate", "ffn_up", "ffn_down")


class _Layer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _LAYER_MATS] + \
               [("attn_norm", C.c_void_p), ("ffn_norm", C.c_void_p)] + \
               [("q_" + n, C.c_int) for n in _LAYER_MATS]


class Model:
    """The reference's CPU forward (forward.zig step + prefill.zig prefillCpu)
    over host weights held by a ``vantablack_b200.model.HostWeights``:
    ``cfg`` plus per-layer dicts of (quant, ndarray).  ``q8_activations``:
    Q8_0 projections take Q8_0-quantized activations (the Q8_0 x Q8_0 path)."""

    def __init__(self, weights, q8_activations: bool = False):
        cfg = weights.cfg
        self.cfg = cfg
        self._keep = weights
        c = _Config(cfg.dim, cfg.n_layers, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim,
                    cfg.ffn_dim, cfg.vocab_size, cfg.max_seq, cfg.rope_base, cfg.rms_eps)
        layers = (_Layer * cfg.n_layers)()
        for i, lw in enumerate(weights.layers):
            L = layers[i]
            for n in _LAYER_MATS:
                q, arr = lw[n]
                setattr(L, n, arr.ctypes.data)
                setattr(L, "q_" + n, q)
            L.attn_norm = lw["attn_norm"].ctypes.data
            L.ffn_norm = lw["ffn_norm"].ctypes.data
        qe, emb = weights.token_embd
        qo, out = weights.output
        self._h = lib.vtbo_model_create(C.byref(c), C.cast(layers, C.c_void_p), _p(emb, _u8p), qe,
                                        _p(weights.output_norm, _f32p), _p(out, _u8p), qo)
        if q8_activations:
            lib.vtbo_model_set_q8_activations(self._h, 1)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib.vtbo_model_destroy(h)
            self._h = None

    @property
    def pos(self) -> int:
        return lib.vtbo_model_pos(self._h)

    def reset(self) -> None:
        lib.vtbo_model_reset(self._h)

    def step(self, token: int) -> np.ndarray:
        logits = np.empty(self.cfg.vocab_size, np.float32)
        rc = lib.vtbo_step(self._h, token, _p(logits, _f32p))
        if rc != 0:
            raise RuntimeError(f"oracle step failed ({rc})")
        return logits

    def prefill(self, tokens) -> np.ndarray:
        t = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self.cfg.vocab_size, np.float32)
        rc = lib.vtbo_prefill(self._h, _p(t, _u32p), t.size, _p(logits, _f32p))
        if rc != 0:
            raise RuntimeError(f"oracle prefill failed ({rc})")
        return logits

    def kv(self, layer: int):
        c = self.cfg
        n = c.max_seq * c.n_kv_heads * c.head_dim
        k = np.ctypeslib.as_array(lib.vtbo_kv_keys(self._h, layer), shape=(n,)).copy()
        v = np.ctypeslib.as_array(lib.vtbo_kv_values(self._h, layer), shape=(n,)).copy()
        return k.reshape(c.max_seq, -1), v.reshape(c.max_seq, -1)

    def generate_greedy(self, prompt, n_gen: int, use_prefill: bool = True):
        """Prompt (batched prefill or per-token), then greedy decode."""
        if use_prefill:
            logits = self.prefill(prompt)
        else:
            for t in prompt:
                logits = self.step(int(t))
        out = []
        for _ in range(n_gen):
            nxt = argmax(logits)
            out.append(nxt)
            logits = self.step(nxt)
        return out, logits
