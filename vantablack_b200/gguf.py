"""GGUF files through the library's own reader (vtb_cuda_gguf_*, C ABI):
the mirror of the reference's ModelMapper / parseHeader / LlamaConfig.fromCatalog
(src/core/mapper.zig, src/core/parser.zig, src/runtime/model.zig).  Parsing
is host-only; no GPU is needed until a model is uploaded."""
from __future__ import annotations

import ctypes as C

from . import _lib
from .model import LlamaConfig, _CConfig


class GgufFile:
    """A read-only mapped GGUF file (vtb_cuda_gguf_open)."""

    def __init__(self, path: str):
        self.lib = _lib.load()
        self.h = self.lib.vtb_cuda_gguf_open(str(path).encode())
        if not self.h:
            raise _lib.VtbError(self.lib.vtb_cuda_last_status(), f"vtb_cuda_gguf_open({path})")

    def close(self):
        if self.h:
            self.lib.vtb_cuda_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def info(self) -> dict:
        v, al, n_t, n_m = C.c_uint32(), C.c_uint32(), C.c_int64(), C.c_int64()
        off = C.c_uint64()
        _lib.check(self.lib.vtb_cuda_gguf_info(self.h, C.byref(v), C.byref(al), C.byref(off), C.byref(n_t),
                                               C.byref(n_m)), "vtb_cuda_gguf_info")
        return {"version": v.value, "alignment": al.value, "data_offset": off.value, "n_tensors": n_t.value,
                "n_meta": n_m.value}

    def tensors(self) -> list[dict]:
        out = []
        for i in range(self.info()["n_tensors"]):
            name, t, nd = C.c_char_p(), C.c_uint32(), C.c_uint32()
            dims = (C.c_uint64 * 8)()
            rel, size = C.c_uint64(), C.c_uint64()
            _lib.check(self.lib.vtb_cuda_gguf_tensor_info(self.h, i, C.byref(name), C.byref(t), C.byref(nd), dims,
                                                          C.byref(rel), C.byref(size)), "vtb_cuda_gguf_tensor_info")
            out.append({"name": name.value.decode(), "type": t.value, "dims": list(dims[:min(nd.value, 8)]),
                        "rel_offset": rel.value, "size": size.value})
        return out

    def tensor_bytes(self, name: str) -> bytes:
        t, size = C.c_uint32(), C.c_uint64()
        p = self.lib.vtb_cuda_gguf_tensor(self.h, name.encode(), C.byref(t), C.byref(size))
        if not p:
            raise _lib.VtbError(-3, f"vtb_cuda_gguf_tensor({name})")
        return C.string_at(p, size.value)

    def meta_int(self, key: str) -> int:
        v = C.c_int64()
        _lib.check(self.lib.vtb_cuda_gguf_meta_int(self.h, key.encode(), C.byref(v)), key)
        return v.value

    def meta_float(self, key: str) -> float:
        v = C.c_double()
        _lib.check(self.lib.vtb_cuda_gguf_meta_float(self.h, key.encode(), C.byref(v)), key)
        return v.value

    def meta_string(self, key: str) -> str:
        p, n = C.c_char_p(), C.c_uint64()
        _lib.check(self.lib.vtb_cuda_gguf_meta_string(self.h, key.encode(), C.byref(p), C.byref(n)), key)
        return C.string_at(p, n.value).decode()

    def meta_array(self, key: str) -> tuple[int, int]:
        t, n = C.c_uint32(), C.c_uint64()
        _lib.check(self.lib.vtb_cuda_gguf_meta_array(self.h, key.encode(), C.byref(t), C.byref(n)), key)
        return t.value, n.value

    def llama_config(self) -> LlamaConfig:
        cc = _CConfig()
        _lib.check(self.lib.vtb_cuda_gguf_llama_config(self.h, C.byref(cc)), "vtb_cuda_gguf_llama_config")
        return LlamaConfig(cc.dim, cc.n_layers, cc.n_heads, cc.n_kv_heads, cc.head_dim, cc.ffn_dim, cc.vocab_size,
                           cc.max_seq, cc.rope_base, cc.rms_eps)
