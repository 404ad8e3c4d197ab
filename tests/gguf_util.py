"""Writes a HostWeights model as a GGUF file with gguf-py (ggml's own Python
writer), the independent producer the library's reader is tested against."""
import numpy as np
from gguf import GGMLQuantizationType, GGUFWriter

from vantablack_b200.model import GGUF_NAMES, MATS  # noqa: F401 -- GGUF_NAMES re-exported for the tests


def _rows(cfg, n):
    kvd = cfg.n_kv_heads * cfg.head_dim
    return {"attn_q": cfg.dim, "attn_k": kvd, "attn_v": kvd, "attn_o": cfg.dim, "ffn_gate": cfg.ffn_dim,
            "ffn_up": cfg.ffn_dim, "ffn_down": cfg.dim}[n]


def _quant(wr, name, q, arr, rows):
    wr.add_tensor(name, np.ascontiguousarray(arr).reshape(rows, -1), raw_dtype=GGMLQuantizationType(q))


def write_llama_gguf(path, w, tied=False, vocab_in_meta=True, arch="llama"):
    c = w.cfg
    wr = GGUFWriter(str(path), arch)
    wr.add_context_length(c.max_seq)
    wr.add_embedding_length(c.dim)
    wr.add_block_count(c.n_layers)
    wr.add_feed_forward_length(c.ffn_dim)
    wr.add_head_count(c.n_heads)
    wr.add_head_count_kv(c.n_kv_heads)
    wr.add_rope_freq_base(c.rope_base)
    wr.add_layer_norm_rms_eps(c.rms_eps)
    if vocab_in_meta:
        wr.add_vocab_size(c.vocab_size)
    else:
        wr.add_token_list([f"t{i}".encode() for i in range(c.vocab_size)])
    for i, lw in enumerate(w.layers):
        wr.add_tensor(f"blk.{i}.attn_norm.weight", lw["attn_norm"])
        for n in MATS:
            q, arr = lw[n]
            _quant(wr, f"blk.{i}.{GGUF_NAMES[n]}.weight", q, arr, _rows(c, n))
        wr.add_tensor(f"blk.{i}.ffn_norm.weight", lw["ffn_norm"])
    qe, emb = w.token_embd
    _quant(wr, "token_embd.weight", qe, emb, c.vocab_size)
    wr.add_tensor("output_norm.weight", w.output_norm)
    if not tied:
        qo, out = w.output
        _quant(wr, "output.weight", qo, out, c.vocab_size)
    wr.write_header_to_file()
    wr.write_kv_data_to_file()
    wr.write_tensors_to_file()
    wr.close()
