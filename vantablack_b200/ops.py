"""Tensor-level front end of the CUDA kernels.

Device memory and streams come from PyTorch (plumbing only); every call goes
through the C ABI of libvtbcuda.so on torch's current stream.  Weight
tensors are flat ``torch.uint8`` CUDA tensors of packed GGUF blocks.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from .synth import BLOCK_ELEMS, F32, Q4_K, Q5_K, Q6_K, Q8_0, row_bytes  # noqa: F401

lib = _lib.load()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _dev(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def gemv(quant: int, w: torch.Tensor, x: torch.Tensor, m: int, k: int, out: torch.Tensor | None = None,
         pdl: bool = False) -> torch.Tensor:
    """y[m] = W[m, k] . x[k] (f32)."""
    _dev(w, "w"); _dev(x, "x")
    if x.dtype != torch.float32 or x.numel() != k:
        raise ValueError("x must be f32[k]")
    if w.numel() < m * row_bytes(quant, k):
        raise ValueError("w is smaller than m rows")
    y = torch.empty(m, dtype=torch.float32, device=x.device) if out is None else out
    _lib.check(lib.vtb_cuda_gemv(quant, w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, _stream(), int(pdl)),
               "vtb_cuda_gemv")
    return y


def dequant(quant: int, w: torch.Tensor, n: int) -> torch.Tensor:
    _dev(w, "w")
    out = torch.empty(n, dtype=torch.float32, device=w.device)
    _lib.check(lib.vtb_cuda_dequant(quant, w.data_ptr(), out.data_ptr(), n, _stream()), "vtb_cuda_dequant")
    return out


def embed(quant: int, table: torch.Tensor, ids: torch.Tensor, dim: int) -> torch.Tensor:
    _dev(table, "table"); _dev(ids, "ids")
    ids = ids.to(torch.int32)
    out = torch.empty(ids.numel(), dim, dtype=torch.float32, device=table.device)
    _lib.check(lib.vtb_cuda_embed(quant, table.data_ptr(), ids.data_ptr(), out.data_ptr(), dim, ids.numel(),
                                  _stream()), "vtb_cuda_embed")
    return out


def gemv_mlx(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, x: torch.Tensor, m: int, k: int,
             bits: int, group: int, bf16: bool, w_off: int = 0) -> torch.Tensor:
    """MLX affine GEMV (mlx.zig matmul): y[m] = W . x.  w, scales, biases are
    flat uint8 CUDA tensors; w_off shifts the weight pointer by bytes."""
    for t, nm in ((w, "w"), (scales, "scales"), (biases, "biases"), (x, "x")):
        _dev(t, nm)
    y = torch.empty(m, dtype=torch.float32, device=x.device)
    _lib.check(lib.vtb_cuda_gemv_mlx(w.data_ptr() + w_off, scales.data_ptr(), biases.data_ptr(), x.data_ptr(),
                                     y.data_ptr(), m, k, bits, group, int(bf16), _stream()), "vtb_cuda_gemv_mlx")
    return y


def dequant_mlx(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, rows: int, k: int, bits: int,
                group: int, bf16: bool, w_off: int = 0) -> torch.Tensor:
    for t, nm in ((w, "w"), (scales, "scales"), (biases, "biases")):
        _dev(t, nm)
    out = torch.empty(rows, k, dtype=torch.float32, device=w.device)
    _lib.check(lib.vtb_cuda_dequant_mlx(w.data_ptr() + w_off, scales.data_ptr(), biases.data_ptr(), out.data_ptr(),
                                        rows, k, bits, group, int(bf16), _stream()), "vtb_cuda_dequant_mlx")
    return out


def sample(logits: torch.Tensor, temperature: float, top_k: int = 0, top_p: float = 0.0, u=None) -> torch.Tensor:
    """Sampler.sample (sampler.zig:44-104) per row of f32 logits [rows, n] on the
    device, with one caller-supplied uniform draw per row; logits are rewritten
    in place.  Returns int32 tokens [rows] on the device."""
    import numpy as np
    _dev(logits, "logits")
    if logits.dtype != torch.float32:
        raise ValueError("logits must be f32")
    lg = logits if logits.dim() == 2 else logits.view(1, -1)
    rows, n = lg.shape
    cfg = _lib.SamplerConfig(float(temperature), int(top_k), float(top_p), 0)
    ua = None if u is None else np.ascontiguousarray(np.atleast_1d(u), np.float32)
    if ua is not None and ua.size != rows:
        raise ValueError("one draw per row")
    tok = torch.empty(rows, dtype=torch.int32, device=logits.device)
    _lib.check(lib.vtb_cuda_sample(lg.data_ptr(), rows, n, n, C.byref(cfg),
                                   None if ua is None else ua.ctypes.data, tok.data_ptr(), _stream()),
               "vtb_cuda_sample")
    return tok


def quantize_q8_0(x: torch.Tensor):
    _dev(x, "x")
    k = x.numel()
    qs = torch.empty(k, dtype=torch.int8, device=x.device)
    d = torch.empty(k // 32, dtype=torch.float32, device=x.device)
    _lib.check(lib.vtb_cuda_quantize_q8_0(x.data_ptr(), k, qs.data_ptr(), d.data_ptr(), _stream()),
               "vtb_cuda_quantize_q8_0")
    return qs, d


def q8_0_block_dots(w: torch.Tensor, xq: torch.Tensor, m: int, k: int) -> torch.Tensor:
    _dev(w, "w"); _dev(xq, "xq")
    dots = torch.empty(m, k // 32, dtype=torch.int32, device=w.device)
    _lib.check(lib.vtb_cuda_q8_0_block_dots(w.data_ptr(), xq.data_ptr(), dots.data_ptr(), m, k, _stream()),
               "vtb_cuda_q8_0_block_dots")
    return dots


def gemv_q8_0_q8_0(w: torch.Tensor, x: torch.Tensor, m: int, k: int, out=None, scratch=None,
                   pdl: bool = False) -> torch.Tensor:
    _dev(w, "w"); _dev(x, "x")
    y = torch.empty(m, dtype=torch.float32, device=x.device) if out is None else out
    if scratch is None:
        scratch = (torch.empty(k, dtype=torch.int8, device=x.device),
                   torch.empty(k // 32, dtype=torch.float32, device=x.device))
    xq, dx = scratch
    _lib.check(lib.vtb_cuda_gemv_q8_0_q8_0(w.data_ptr(), x.data_ptr(), y.data_ptr(), m, k, xq.data_ptr(),
                                           dx.data_ptr(), _stream(), int(pdl)), "vtb_cuda_gemv_q8_0_q8_0")
    return y


def gemm(quant: int, w: torch.Tensor, acts: torch.Tensor, m: int, k: int, precise: bool = False,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """out[B, m] = acts[B, k] . W^T on the tcgen05 tensor cores (prefill)."""
    _dev(w, "w"); _dev(acts, "acts")
    nb = acts.shape[0]
    if acts.dtype != torch.float32 or acts.numel() != nb * k:
        raise ValueError("acts must be f32[B, k]")
    o = torch.empty(nb, m, dtype=torch.float32, device=acts.device) if out is None else out
    wsb = lib.vtb_cuda_gemm_workspace_bytes(k, nb, int(precise))
    ws = torch.empty(wsb, dtype=torch.uint8, device=acts.device)
    _lib.check(lib.vtb_cuda_gemm(quant, w.data_ptr(), acts.data_ptr(), o.data_ptr(), m, k, nb, int(precise),
                                 ws.data_ptr(), wsb, _stream()), "vtb_cuda_gemm")
    return o


def check_device_error() -> None:
    _lib.check(lib.vtb_cuda_check_device_error(), "device error word")
