"""The library's GGUF reader (vtb_cuda_gguf_*) on CPU: the reference parser's
own known-answer file (src/core/parser.zig tests), its rejection cases, and
round trips of seeded Llama models written by gguf-py, checked against
gguf-py's reader and the source arrays."""
import struct

import numpy as np
import pytest

from vantablack_b200 import _lib
from vantablack_b200 import synth as S
from vantablack_b200.gguf import GgufFile
from vantablack_b200.model import MATS, HostWeights, LlamaConfig

from gguf_util import GGUF_NAMES, write_llama_gguf

SMALL = LlamaConfig(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab_size=512,
                    max_seq=600, rope_base=500000.0, rms_eps=1e-6)


def _s(x: str) -> bytes:
    return struct.pack("<Q", len(x)) + x.encode()


def minimal_v3(version=3, magic=0x46554747, n_dims=2, dims=(4, 4), ggml_type=0, rel=0, tail=64):
    """parser.zig's 'minimal valid v3 file with one F32 tensor'."""
    b = struct.pack("<IIQQ", magic, version, 1, 2)
    b += _s("general.architecture") + struct.pack("<I", 8) + _s("test")
    b += _s("general.alignment") + struct.pack("<II", 4, 32)
    b += _s("w") + struct.pack("<I", n_dims) + b"".join(struct.pack("<Q", d) for d in dims)
    b += struct.pack("<IQ", ggml_type, rel)
    b += b"\0" * ((-len(b)) % 32)
    return b + b"\0" * tail


def open_status(path) -> int:
    with pytest.raises(_lib.VtbError) as e:
        GgufFile(path)
    return e.value.status


def test_reference_minimal_file(tmp_path):
    p = tmp_path / "m.gguf"
    raw = minimal_v3()
    p.write_bytes(raw)
    with GgufFile(p) as g:
        info = g.info()
        assert info == {"version": 3, "alignment": 32, "data_offset": len(raw) - 64, "n_tensors": 1, "n_meta": 2}
        (t,) = g.tensors()
        assert t == {"name": "w", "type": 0, "dims": [4, 4], "rel_offset": 0, "size": 64}
        assert g.meta_string("general.architecture") == "test"
        assert g.meta_int("general.alignment") == 32
        assert g.tensor_bytes("w") == b"\0" * 64


@pytest.mark.parametrize("kind,status", [
    ("bad_magic", -3), ("version1", -3), ("truncated", -3), ("missing", -2), ("empty", -2), ("too_small", -3),
    ("partial_block", -3), ("deep_array", -3), ("bad_meta_type", -3), ("numel_overflow", -3), ("size_overflow", -3)])
def test_rejections(tmp_path, kind, status):
    p = tmp_path / f"{kind}.gguf"
    if kind == "bad_magic":
        p.write_bytes(minimal_v3(magic=0xDEADBEEF))
    elif kind == "version1":
        p.write_bytes(minimal_v3(version=1))
    elif kind == "truncated":
        p.write_bytes(minimal_v3()[:60])
    elif kind == "empty":
        p.write_bytes(b"")
    elif kind == "too_small":
        p.write_bytes(b"GGUF\x03\0\0\0")
    elif kind == "partial_block":  # 100 Q4_K elements: not a whole 256-element block
        p.write_bytes(minimal_v3(n_dims=1, dims=(100,), ggml_type=12))
    elif kind == "numel_overflow":
        p.write_bytes(minimal_v3(dims=(1 << 40, 1 << 40)))
    elif kind == "size_overflow":  # 2^62 f32 elements: the count fits, the byte size does not
        p.write_bytes(minimal_v3(dims=(1 << 31, 1 << 31)))
    elif kind in ("deep_array", "bad_meta_type"):
        b = struct.pack("<IIQQ", 0x46554747, 3, 0, 1) + _s("k")
        if kind == "deep_array":  # 6 levels of arrays of arrays: nesting deeper than 4
            b += struct.pack("<I", 9) + struct.pack("<IQ", 9, 1) * 5 + struct.pack("<IQ", 4, 1) + struct.pack("<I", 7)
        else:
            b += struct.pack("<I", 99) + b"\0" * 16
        p.write_bytes(b)
    assert open_status(p) == status


def test_tensor_outside_file(tmp_path):
    p = tmp_path / "oob.gguf"
    p.write_bytes(minimal_v3(rel=1 << 20))
    with GgufFile(p) as g:
        with pytest.raises(_lib.VtbError):
            g.tensor_bytes("w")


@pytest.mark.parametrize("tied,vocab_in_meta", [(False, True), (True, False)])
def test_llama_round_trip(tmp_path, tied, vocab_in_meta):
    import gguf as gg
    w = HostWeights(SMALL, seed=3, quants={"attn_v": S.Q6_K, "ffn_up": S.Q5_K, "attn_o": S.Q8_0})
    p = tmp_path / "llama.gguf"
    write_llama_gguf(p, w, tied=tied, vocab_in_meta=vocab_in_meta)
    ref = gg.GGUFReader(str(p))
    with GgufFile(p) as g:
        assert g.llama_config() == SMALL.with_(rms_eps=float(np.float32(SMALL.rms_eps)))  # f32 metadata
        assert g.meta_string("general.architecture") == "llama"
        ours = {t["name"]: t for t in g.tensors()}
        assert set(ours) == {t.name for t in ref.tensors}
        for t in ref.tensors:
            o = ours[t.name]
            assert o["type"] == int(t.tensor_type)
            assert o["dims"] == [int(d) for d in t.shape]
            assert g.info()["data_offset"] + o["rel_offset"] == int(t.data_offset)
            assert o["size"] == int(t.n_bytes)
        for i, lw in enumerate(w.layers):
            for n in MATS:
                assert g.tensor_bytes(f"blk.{i}.{GGUF_NAMES[n]}.weight") == lw[n][1].tobytes()
            assert g.tensor_bytes(f"blk.{i}.attn_norm.weight") == lw["attn_norm"].tobytes()
        assert g.tensor_bytes("token_embd.weight") == w.token_embd[1].tobytes()
        assert ("output.weight" in ours) == (not tied)
        if not vocab_in_meta:
            assert g.meta_array("tokenizer.ggml.tokens") == (8, SMALL.vocab_size)


def test_defaults_and_unsupported_arch(tmp_path):
    p = tmp_path / "gemma.gguf"
    write_llama_gguf(p, HostWeights(SMALL.with_(n_layers=1), seed=1), arch="gemma")
    with GgufFile(p) as g:
        with pytest.raises(_lib.VtbError) as e:
            g.llama_config()
        assert e.value.status == -8


def test_status_codes_of_a_failed_open(tmp_path):
    """A NULL handle leaves its status and message for vtb_cuda_last_status /
    vtb_cuda_last_error (the -2 / -3 codes reuse the reference's
    VTB_ERR_FILE_OPEN / VTB_ERR_PARSE)."""
    lib = _lib.load()
    assert not lib.vtb_cuda_gguf_open(str(tmp_path / "absent.gguf").encode())
    assert lib.vtb_cuda_last_status() == -2
    assert b"cannot open" in lib.vtb_cuda_last_error()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(minimal_v3(magic=0x12345678))
    assert not lib.vtb_cuda_gguf_open(str(bad).encode())
    assert lib.vtb_cuda_last_status() == -3
    assert b"not a GGUF file" in lib.vtb_cuda_last_error()
    assert lib.vtb_cuda_status_string(-2) == b"file cannot be opened"
    assert lib.vtb_cuda_status_string(-3) == b"malformed model file"


def test_library_writer_streams_the_seeded_model(tmp_path):
    """write_synthetic_gguf (the library's own streaming writer) produces a file
    that gguf-py reads back to the HostWeights bytes, and that the library's
    reader maps to the same arrays (HostWeights.from_gguf)."""
    import gguf
    from vantablack_b200.model import write_synthetic_gguf
    quants = {"attn_v": S.Q6_K, "ffn_gate": S.Q5_K, "ffn_up": S.Q8_0}
    w = HostWeights(SMALL, seed=21, quants=quants)
    p = str(tmp_path / "w.gguf")
    write_synthetic_gguf(p, SMALL, seed=21, quants=quants)
    r = gguf.GGUFReader(p)
    by_name = {t.name: t for t in r.tensors}
    for i, lw in enumerate(w.layers):
        for n in MATS:
            q, arr = lw[n]
            t = by_name[f"blk.{i}.{GGUF_NAMES[n]}.weight"]
            assert int(t.tensor_type) == q
            assert np.array_equal(np.asarray(t.data).reshape(-1).view(np.uint8), arr)
        assert np.array_equal(np.asarray(by_name[f"blk.{i}.ffn_norm.weight"].data), lw["ffn_norm"])
    assert np.array_equal(np.asarray(by_name["output.weight"].data).reshape(-1).view(np.uint8), w.output[1])
    g = HostWeights.from_gguf(p)
    assert g.cfg.dim == SMALL.dim and g.cfg.vocab_size == SMALL.vocab_size and g.cfg.n_kv_heads == 2
    for i in range(SMALL.n_layers):
        for n in MATS:
            assert g.layers[i][n][0] == w.layers[i][n][0]
            assert np.array_equal(g.layers[i][n][1], w.layers[i][n][1])
        assert np.array_equal(g.layers[i]["attn_norm"], w.layers[i]["attn_norm"])
    assert np.array_equal(g.token_embd[1], w.token_embd[1]) and np.array_equal(g.output_norm, w.output_norm)
