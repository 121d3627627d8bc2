"""ctypes binding of libtpp_b200.so (the C-ABI declared in include/tpp_b200.h).

The library is built in-tree by ``torchplusplus_b200.build``.  There is no CPU
fallback anywhere in the package: if the shared library is missing or a tensor
is not on a CUDA device, the calling op raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("TPP_LIB") or
                Path(__file__).resolve().parent / "_lib" / "libtpp_b200.so")

TPP_OK = 0
STATUS_NAMES = {
    1: "TPP_ERR_SHAPE",
    2: "TPP_ERR_DTYPE",
    3: "TPP_ERR_ALIGN",
    4: "TPP_ERR_LAUNCH",
    5: "TPP_ERR_TIMEOUT",
    6: "TPP_ERR_UNSUPPORTED",
    7: "TPP_ERR_WORKSPACE",
}

DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

ACT_CODE = {"none": 0, "silu": 1, "gelu": 2, "relu": 3, "swiglu": 4}

_p = C.c_void_p
_i64 = C.c_int64
_i32 = C.c_int
_f32 = C.c_float

# name -> (restype, argtypes); mirrors include/tpp_b200.h
SIGNATURES: dict[str, tuple] = {
    "tpp_last_error": (C.c_char_p, []),
    "tpp_version": (C.c_char_p, []),
    "tpp_launch_count": (C.c_uint64, []),
    "tpp_device_error": (_i32, [_p]),
    "tpp_set_sm_budget": (_i32, [_i32]),
    "tpp_decode_step_persistent_workspace": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "tpp_decode_step_persistent": (_i32, [_p, _i64, _p, _p, _p, _p, _i64, _p, _p, _p, _p, _i64,
                                          _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                          _i64, _f32, _i32, _p]),
    "tpp_debug_expire_wait": (_i32, [C.c_uint32, _i32, _p]),
    "tpp_rmsnorm": (_i32, [_p, _i64, _p, _p, _i64, _i64, _i64, _f32, _i32, _p]),
    "tpp_add_rmsnorm": (_i32, [_p, _p, _p, _p, _i64, _i64, _f32, _i32, _p]),
    "tpp_layernorm": (_i32, [_p, _p, _p, _p, _i64, _i64, _f32, _i32, _p]),
    "tpp_rope": (_i32, [_p, _i64, _i64, _i64, _p, _p, _i64, _i32, _p, _i64, _i64, _i64, _i64,
                        _i64, _i32, _p]),
    "tpp_qkrope": (_i32, [_p, _p, _p, _p, _i64, _i32, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                          _i32, _p]),
    "tpp_linear": (_i32, [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i32, _i32, _p]),
    "tpp_rmsnorm_linear": (_i32, [_p, _i64, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32, _i32,
                                  _i32, _p]),
    "tpp_hgemv": (_i32, [_p, _p, _p, _i64, _i64, _i32, _p]),
    "tpp_l2_prefetch": (_i32, [_p, _i64, _p]),
    "tpp_sample": (_i32, [_p, _i64, _i64, _i64, _f32, _i64, _f32, C.c_uint64, _p, _p, _i32, _p]),
    "tpp_fp8_weight_bytes": (_i64, [_i64, _i64]),
    "tpp_quantize_weight_fp8": (_i32, [_p, _i64, _i64, _i32, _p, _p, _p]),
    "tpp_dequantize_weight_fp8": (_i32, [_p, _p, _i64, _i64, _i32, _p, _p]),
    "tpp_linear_fp8": (_i32, [_p, _i64, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _f32, _i32,
                              _i32, _p]),
    "tpp_packed_weight_bytes": (_i64, [_i64, _i64, _i32]),
    "tpp_packed_activation_bytes": (_i64, [_i64, _i64]),
    "tpp_pack_weight": (_i32, [_p, _i64, _i64, _i32, _i32, _p, _p]),
    "tpp_pack_activation": (_i32, [_p, _i64, _i64, _i64, _i32, _p, _p]),
    "tpp_linear_packed": (_i32, [_p, _p, _p, _p, _p, _i64, _p, _i64, _i64, _i64, _f32, _i32,
                                 _i32, _p]),
    "tpp_attention_prefill": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64,
                                     _i64, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                     _i64, _i32, _i64, _f32, _i32, _p]),
    "tpp_attention_decode_workspace": (_i64, [_i64, _i64, _i64, _i64]),
    "tpp_attention_decode_workspace_exact": (_i64, [_i64, _i64, _i64, _i64, _i64, _i64]),
    "tpp_attention_decode_qkv": (_i32, [_p, _i64, _p, _p, _f32, _p, _p, _i64, _i32, _p, _p, _p,
                                        _i64, _i64, _i64, _p, _i64, _p, _i64, _i64, _i64, _i64,
                                        _i64, _i64, _i64, _f32, _p, _i64, _i32, _p]),
    "tpp_attention_decode_paged": (_i32, [_p, _i64, _i64, _p, _p, _i64, _p, _i64, _p, _i64, _p,
                                          _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p,
                                          _i64, _i32, _p]),
    "tpp_attention_decode_qkv_paged": (_i32, [_p, _i64, _p, _p, _f32, _p, _p, _i64, _i32, _p, _p,
                                              _p, _i64, _p, _i64, _p, _i64, _p, _i64, _i64, _i64,
                                              _i64, _i64, _i64, _i64, _f32, _p, _i64, _i32, _p]),
    "tpp_kv_append_paged": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _i64, _p,
                                   _i64, _p, _i64, _i64, _i64, _i64, _i64, _i32, _p]),
    "tpp_attention_decode": (_i32, [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64, _p, _i64,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _i64, _i32, _p]),
    "tpp_attention_decode_noalloc": (_i32, [_p, _i64, _i64, _p, _p, _i64, _i64, _i64, _p, _i64,
                                            _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32,
                                            _i32, _p]),
    "tpp_attention_decode_noalloc_max_bytes": (_i64, []),
    "tpp_qk_norm_rope_cache": (_i32, [_p, _i64, _p, _p, _f32, _p, _p, _i64, _i32, _p, _p, _p, _p,
                                      _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i32, _p]),
    "tpp_kv_append": (_i32, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _p, _i64, _i64, _i64,
                             _i64, _i64, _i64, _i64, _i64, _p, _i32, _p]),
    "tpp_argmax": (_i32, [_p, _i64, _i64, _i64, _p, _i32, _p]),
    "tpp_embedding": (_i32, [_p, _i64, _p, _i64, _i64, _p, _i32, _p]),
    "tpp_decode_advance": (_i32, [_p, _p, _i64, _i64, _p, _p, _i64, _p]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


class TppError(RuntimeError):
    """A C-ABI call returned a non-zero tpp_status."""

    def __init__(self, fn: str, status: int, msg: str):
        self.status = status
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(status, status)}: {msg}")


def lib() -> C.CDLL:
    """Loads the shared library once (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m torchplusplus_b200.build` "
                    "(this package has no CPU fallback)")
            h = C.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | os.RTLD_LOCAL)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(h, name)
                fn.restype = res
                fn.argtypes = args
            _lib = h
    return _lib


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def call(name: str, *args) -> None:
    """Calls a status-returning entry point and raises TppError on failure."""
    st = getattr(lib(), name)(*args)
    if st != TPP_OK:
        msg = lib().tpp_last_error().decode(errors="replace")
        raise TppError(name, st, msg)


def dtype_code(t: torch.dtype) -> int:
    try:
        return DTYPE_CODE[t]
    except KeyError:
        raise TypeError(f"unsupported dtype {t}; expected float16 or bfloat16") from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def launch_count() -> int:
    return int(lib().tpp_launch_count())
