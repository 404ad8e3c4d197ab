"""GGUF files through the library's own reader (vtb_cuda_gguf_*, C ABI):
the mirror of the reference's ModelMapper / parseHeader / LlamaConfig.fromCatalog
(src/core/mapper.zig, src/core/parser.zig, src/runtime/model.zig).  Parsing
is host-only; no GPU is needed until a model is uploaded."""
from __future__ import annotations

import ctypes as C
import os
import struct

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


# ---- writer -----------------------------------------------------------------
# GGUF v3 layout (the format parser.zig:285-355 reads): magic "GGUF", u32
# version, u64 tensor count, u64 metadata count; metadata key/value pairs;
# tensor infos (name, u32 n_dims, u64 dims innermost first, u32 ggml type,
# u64 offset relative to the data section); zero padding to the alignment;
# tensor data, each tensor starting on an aligned offset.
_META_FMT = {"u32": (4, "<I"), "i32": (5, "<i"), "f32": (6, "<f"), "u64": (10, "<Q"), "f64": (12, "<d")}
_BLOCK = {0: (1, 4), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210), 32: (256, 66)}  # type: (elems, bytes)


def _gstr(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def tensor_nbytes(ggml_type: int, dims) -> int:
    elems, nbytes = _BLOCK[ggml_type]
    n = 1
    for d in dims:
        n *= int(d)
    if n % elems:
        raise ValueError("element count is not a whole number of blocks")
    return n // elems * nbytes


def write_gguf(path: str, meta, infos, arrays, alignment: int = 32) -> None:
    """Writes a GGUF v3 file.  meta: [(key, kind, value)] with kind in
    {"str", "u32", "i32", "f32", "u64", "f64"}; infos: [(name, ggml_type, dims)]
    with dims innermost first ([k, rows] for a matrix); arrays: an iterable
    of the tensors' bytes (numpy arrays) in the order of infos, consumed one at
    a time.  Written to path + ".tmp" and renamed, so a reader never sees a
    partial file."""
    hdr = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(infos), len(meta)))
    for key, kind, val in meta:
        hdr += _gstr(key)
        if kind == "str":
            hdr += struct.pack("<I", 8) + _gstr(val)
        else:
            code, fmt = _META_FMT[kind]
            hdr += struct.pack("<I", code) + struct.pack(fmt, val)
    sizes, off = [], 0
    for name, t, dims in infos:
        nb = tensor_nbytes(t, dims)
        hdr += _gstr(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", int(d)) for d in dims)
        hdr += struct.pack("<IQ", t, off)
        sizes.append(nb)
        off += (nb + alignment - 1) // alignment * alignment
    hdr += b"\0" * (-len(hdr) % alignment)
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(hdr)
        n = 0
        for a, nb in zip(arrays, sizes):
            b = memoryview(a).cast("B")
            if b.nbytes != nb:
                raise ValueError(f"tensor {infos[n][0]}: {b.nbytes} bytes, expected {nb}")
            f.write(b)
            f.write(b"\0" * (-nb % alignment))
            n += 1
        if n != len(infos):
            raise ValueError("fewer arrays than tensor infos")
    os.replace(tmp, path)
