"""ctypes binding of libvtbcuda.so (the C ABI in include/vtb_cuda.h).

The library is the product: there is no CPU or PyTorch fallback.  Loading
fails loudly if it has not been built.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvtbcuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "vtb_cuda.h")

OK = 0
STATUS = {0: "ok", -1: "invalid argument", -2: "file cannot be opened", -3: "malformed model file", -4: "out of device memory", -5: "no usable CUDA device",
          -6: "kernel dispatch failed", -8: "unsupported quant type", -9: "device-side wait timed out",
          -10: "collective communication failed"}

_vp, _i64, _i32, _int, _sz = C.c_void_p, C.c_int64, C.c_int32, C.c_int, C.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "vtb_cuda_version_string": (C.c_char_p, []),
    "vtb_cuda_available": (_int, []),
    "vtb_cuda_status_string": (C.c_char_p, [_int]),
    "vtb_cuda_last_error": (C.c_char_p, []),
    "vtb_cuda_last_status": (_int, []),
    "vtb_cuda_row_bytes": (_i64, [_int, _i64]),
    "vtb_cuda_check_device_error": (_int, []),
    "vtb_cuda_gemv": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _vp, _int]),
    "vtb_cuda_dequant": (_int, [_int, _vp, _vp, _i64, _vp]),
    "vtb_cuda_embed": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _vp]),
    "vtb_cuda_quantize_q8_0": (_int, [_vp, _i64, _vp, _vp, _vp]),
    "vtb_cuda_q8_0_block_dots": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "vtb_cuda_gemv_q8_0_q8_0": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _int]),
    "vtb_cuda_gemv_q8_0_q8_0_noalloc": (_int, [_vp, _vp, _vp, _i64, _i64, _vp, _int]),
    "vtb_cuda_gemm_workspace_bytes": (_sz, [_i64, _i64, _int]),
    "vtb_cuda_gemm": (_int, [_int, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp, _sz, _vp]),
    "vtb_cuda_capabilities": (_int, [_vp, _vp]),
    "vtb_cuda_init": (_vp, [_int]),
    "vtb_cuda_destroy": (None, [_vp]),
    "vtb_cuda_stream": (_vp, [_vp]),
    "vtb_cuda_alloc": (_vp, [_vp, _sz, C.POINTER(_vp)]),
    "vtb_cuda_upload": (_vp, [_vp, _vp, _sz]),
    "vtb_cuda_release": (None, [_vp]),
    "vtb_cuda_buf_ptr": (_vp, [_vp]),
    "vtb_cuda_buf_size": (_sz, [_vp]),
    "vtb_cuda_copy_h2d": (_int, [_vp, _vp, _sz, _vp, _sz]),
    "vtb_cuda_copy_d2h": (_int, [_vp, _vp, _vp, _sz, _sz]),
    "vtb_cuda_copy_d2h_async": (_int, [_vp, _vp, _vp, _sz, _sz]),
    "vtb_cuda_wait_idle": (_int, [_vp]),
    "vtb_cuda_matmul_q8_0": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_matmul_q4_k": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_matmul_q5_k": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_matmul_q6_k": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_matmul_tq2_0": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_segment_begin": (_vp, [_vp]),
    "vtb_cuda_segment_commit": (_int, [_vp]),
    "vtb_cuda_segment_matmul_q8_0": (None, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_segment_matmul_q4_k": (None, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_segment_matmul_q5_k": (None, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_segment_matmul_q6_k": (None, [_vp, _vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_segment_copy": (None, [_vp, _vp, _sz, _vp, _sz, _sz]),
    "vtb_cuda_segment_copy_h2d": (None, [_vp, _vp, _sz, _vp, _sz]),
    "vtb_cuda_segment_copy_d2h": (None, [_vp, _vp, _vp, _sz, _sz]),
    "vtb_cuda_model_create": (_vp, [_vp, _vp, _vp, _vp, _i32, _vp, _vp, _i32]),
    "vtb_cuda_model_destroy": (None, [_vp]),
    "vtb_cuda_model_weight_bytes": (_sz, [_vp]),
    "vtb_cuda_model_set_q8_activations": (_int, [_vp, _int]),
    "vtb_cuda_state_create": (_vp, [_vp, _i32, _i32]),
    "vtb_cuda_state_destroy": (None, [_vp]),
    "vtb_cuda_state_reset": (_int, [_vp]),
    "vtb_cuda_state_pos": (_i64, [_vp, _i32]),
    "vtb_cuda_state_tp_p2p": (_i32, [_vp]),
    "vtb_cuda_begin_token": (_int, [_vp, _vp]),
    "vtb_cuda_layer_step": (_int, [_vp, _i32]),
    "vtb_cuda_final_step": (_int, [_vp]),
    "vtb_cuda_finalize_token": (_int, [_vp, _vp, _vp]),
    "vtb_cuda_step": (_int, [_vp, _vp, _vp, _vp]),
    "vtb_cuda_prefill": (_int, [_vp, _i32, _vp, _i32, _vp, _vp]),
    "vtb_cuda_gemv_mlx": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _int, _vp]),
    "vtb_cuda_dequant_mlx": (_int, [_vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _int, _vp]),
    "vtb_cuda_matmul_mlx_q4": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _sz, _sz, _sz, C.c_uint32,
                                      C.c_uint32]),
    "vtb_cuda_sample": (_int, [_vp, _i64, _i64, _i64, _vp, _vp, _vp, _vp]),
    "vtb_cuda_state_sample": (_int, [_vp, _i32, _vp, _vp, _vp]),
    "vtb_cuda_tp_unique_id": (_int, [_vp]),
    "vtb_cuda_tp_init": (_vp, [_int, _int, _int, _vp]),
    "vtb_cuda_tp_destroy": (None, [_vp]),
    "vtb_cuda_tp_rank": (_int, [_vp]),
    "vtb_cuda_tp_world": (_int, [_vp]),
    "vtb_cuda_tp_shard_plan": (_int, [_vp, _int, _int, _i32, _vp]),
    "vtb_cuda_tp_slice": (_int, [_int, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "vtb_cuda_model_create_tp": (_vp, [_vp, _vp, _vp, _vp, _vp, _i32, _vp, _vp, _i32]),
    "vtb_cuda_gguf_open": (_vp, [C.c_char_p]),
    "vtb_cuda_gguf_close": (None, [_vp]),
    "vtb_cuda_gguf_info": (_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "vtb_cuda_gguf_tensor_info": (_int, [_vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "vtb_cuda_gguf_tensor": (_vp, [_vp, C.c_char_p, _vp, _vp]),
    "vtb_cuda_gguf_meta_int": (_int, [_vp, C.c_char_p, _vp]),
    "vtb_cuda_gguf_meta_float": (_int, [_vp, C.c_char_p, _vp]),
    "vtb_cuda_gguf_meta_string": (_int, [_vp, C.c_char_p, _vp, _vp]),
    "vtb_cuda_gguf_meta_array": (_int, [_vp, C.c_char_p, _vp, _vp]),
    "vtb_cuda_gguf_llama_config": (_int, [_vp, _vp]),
    "vtb_cuda_model_create_gguf": (_vp, [_vp, _vp, _i32]),
    "vtb_cuda_model_create_gguf_tp": (_vp, [_vp, _vp, _vp, _i32]),
}


class SamplerConfig(C.Structure):
    """VtbCudaSamplerConfig: the reference's VtbSamplerConfig (include/vantablack.h:46-51)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_size_t), ("top_p", C.c_float), ("seed", C.c_uint64)]


class VtbError(RuntimeError):
    def __init__(self, status: int, where: str):
        detail = ""
        if _lib is not None:
            detail = (_lib.vtb_cuda_last_error() or b"").decode(errors="replace")
        super().__init__(f"{where}: {STATUS.get(status, status)} ({status}) {detail}".rstrip())
        self.status = status


_lib = None


def header_symbols(path: str = HEADER) -> list[str]:
    """Function names declared in include/vtb_cuda.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vtb_cuda_\w+)\s*\(", text)))


def load(path: str = LIB_PATH):
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -m vantablack_b200.build` "
                          "(there is no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int, where: str) -> None:
    if status != OK:
        raise VtbError(status, where)
