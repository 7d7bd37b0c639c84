"""ctypes binding of libgpt_b200.so (the C ABI declared in include/gpt_b200.h).

The shared library is built in-tree by ``cutilegpt_b200/csrc/build.py`` into
``cutilegpt_b200/lib/``. There is no fallback: if the library is missing,
importing an operator raises, so a GPU run can never silently execute
anything but these kernels.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libgpt_b200.so")

GPT_OK, GPT_ERR_SHAPE, GPT_ERR_ALIGN, GPT_ERR_DTYPE = 0, 1, 2, 3
GPT_ERR_UNSUPPORTED, GPT_ERR_CUDA, GPT_ERR_TIMEOUT, GPT_ERR_ARG = 4, 5, 6, 7
GPT_F32, GPT_BF16 = 0, 1
EPI_NONE, EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_RESIDUAL = 0, 1, 2, 3

_STATUS_NAMES = {
    GPT_ERR_SHAPE: "GPT_ERR_SHAPE", GPT_ERR_ALIGN: "GPT_ERR_ALIGN", GPT_ERR_DTYPE: "GPT_ERR_DTYPE",
    GPT_ERR_UNSUPPORTED: "GPT_ERR_UNSUPPORTED", GPT_ERR_CUDA: "GPT_ERR_CUDA",
    GPT_ERR_TIMEOUT: "GPT_ERR_TIMEOUT", GPT_ERR_ARG: "GPT_ERR_ARG",
}

_i64, _p, _i32, _f32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_int, ctypes.c_float
_pi64 = ctypes.POINTER(ctypes.c_int64)



class GemmFusion(ctypes.Structure):
    """struct gpt_gemm_fusion (include/gpt_b200.h): optional extras of gpt_gemm_fused."""
    _fields_ = [
        ("ln_stats", _p), ("ln_parts", _i64), ("ln_eps", _f32), ("ln_u", _p), ("ln_v", _p),
        ("row_stats", _p),
        ("k_cache", _p), ("v_cache", _p), ("kv_heads", _i64), ("kv_dim", _i64), ("kv_tmax", _i64),
        ("kv_pos0", _i64), ("kv_pos_dev", _p), ("ln_sums", _p), ("row_sums", _p),
    ]


# name -> (restype, argtypes); mirrors include/gpt_b200.h
SIGNATURES = {
    "gpt_version": (_i32, []),
    "gpt_last_error_string": (ctypes.c_char_p, []),
    "gpt_device_error": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "gpt_sm_count": (_i32, []),
    "gpt_set_wait_limit_ns": (_i32, [ctypes.c_uint64]),
    "gpt_selftest_wait": (_i32, [_i32, _i32, _p, _p]),
    "gpt_launch_count": (_i64, []),
    "gpt_embedding": (_i32, [_p, _i64, _p, _i64, _i64, _p, _i32, _p]),
    "gpt_embedding_pos": (_i32, [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i32, _p]),
    "gpt_layernorm": (_i32, [_p, _p, _p, _p, _i64, _i64, _f32, _i32, _p]),
    "gpt_gelu": (_i32, [_p, _p, _i64, _i32, _p]),
    "gpt_gemm": (_i32, [_p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i32, _i32, _p]),
    "gpt_attention_prefill": (_i32, [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _pi64, _pi64, _pi64,
                                     _pi64, _f32, _i32, _p]),
    "gpt_kv_append": (_i32, [_p, _i64, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _i32, _p]),
    "gpt_attention_decode_workspace_size": (_i64, [_i64, _i64, _i64, _i64]),
    "gpt_attention_decode": (_i32, [_p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p,
                                    _f32, _p, _i32, _p]),
    "gpt_attention_decode_noalloc": (_i32, [_p, _i64, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _p,
                                            _f32, _i32, _p]),
    "gpt_decode_advance": (_i32, [_p, _i64, _p, _i64, _i64, _p, _p]),
    "gpt_argmax": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p]),
    "gpt_sample": (_i32, [_p, _i64, _i64, _i64, ctypes.c_float, _i64, _p, _p, _i64, _p, _i32, _p]),
    "gpt_gemm_fused": (_i32, [_p, _i64, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _i64, _i32,
                              ctypes.POINTER(GemmFusion), _i32, _p]),
    "gpt_row_stats": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p]),
    "gpt_row_sums": (_i32, [_p, _i64, _i64, _i64, _p, _p, _i64, _i32, _p]),
    "gpt_lnfold_weights": (_i32, [_p, _p, _p, _p, _i64, _i64, _p, _p, _p, _i32, _p]),
}

_lib = None
_lock = threading.Lock()


class GptError(RuntimeError):
    """A libgpt_b200 call returned a non-OK status."""

    def __init__(self, status: int, what: str, msg: str):
        self.status = status
        super().__init__(f"{what}: {_STATUS_NAMES.get(status, status)}: {msg}")


class GptValueError(GptError, ValueError):
    """Shape / alignment / dtype / argument rejection (the reference raises ValueError)."""


def lib() -> ctypes.CDLL:
    """Loads the library once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"libgpt_b200.so not found at {LIB_PATH}; build it with "
                        "`python cutilegpt_b200/csrc/build.py` (or __graft_entry__.build())")
                handle = ctypes.CDLL(LIB_PATH)
                for name, (res, args) in SIGNATURES.items():
                    fn = getattr(handle, name)
                    fn.restype = res
                    fn.argtypes = args
                _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status == GPT_OK:
        return
    msg = lib().gpt_last_error_string().decode(errors="replace")
    if status in (GPT_ERR_SHAPE, GPT_ERR_ALIGN, GPT_ERR_DTYPE, GPT_ERR_ARG):
        raise GptValueError(status, what, msg)
    raise GptError(status, what, msg)


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return GPT_F32
    if dt == torch.bfloat16:
        return GPT_BF16
    raise ValueError(f"unsupported dtype {dt}; libgpt_b200 computes in float32 or bfloat16")


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def strides3(*vals: int):
    return (ctypes.c_int64 * 3)(*vals)


def device_error() -> int:
    """Reads (and clears) the device error word; raises on a recorded error."""
    code = ctypes.c_int(0)
    check(lib().gpt_device_error(ctypes.byref(code)), "gpt_device_error")
    return code.value
