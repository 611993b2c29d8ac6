"""ctypes binding of ``libengpt_b200.so`` (the C ABI declared in ``include/engpt_b200.h``).

The library is loaded lazily on first use.  There is no fallback: if the
shared object is missing or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libengpt_b200.so")

# enum engpt_dtype / engpt_status / engpt_aux_mode / engpt_attn_impl
F32, BF16 = 0, 1
OK = 0
STATUS_NAMES = {1: "shape", 2: "dtype", 3: "alignment", 4: "launch", 5: "device timeout", 6: "unsupported",
                7: "argument"}
AUX_NONE, AUX_BF16_Y, AUX_BF16_H, AUX_F32_H = 0, 1, 2, 3
QKV_BTHD, QKV_BHTD, QKV_INPLACE = 0, 1, 2
ATTN_AUTO, ATTN_TCGEN05, ATTN_SIMT, ATTN_TCGEN05_1TILE = 0, 1, 2, 3

_lock = threading.Lock()
_lib: Optional[ctypes.CDLL] = None

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float

SIGNATURES = {
    "engpt_last_error": (ctypes.c_char_p, []),
    "engpt_abi_version": (_i, []),
    "engpt_device_status": (_i, []),
    "engpt_clear_device_status": (_i, []),
    "engpt_selftest_wait_timeout": (_i, [_i64, _p, _p]),
    "engpt_qkv_postprocess": (_i, [_p, _i, _p, _p, _p, _i, _p, _f, _f, _i, _i, _i, _i, _p, _p, _p, _i, _p]),
    "engpt_causal_attention": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _p, _i, _p]),
    "engpt_ngpt_attention": (_i, [_p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _p, _p, _f, _p]),
    "engpt_carried_residual_gauge": (_i, [_p, _p, _p, _i, _p, _f, _i, _f, _f, _f, _i64, _i, _p, _p, _p, _i, _p]),
    "engpt_rotary_tables": (_i, [_i, _i, _f, _p, _p, _p]),
    "engpt_embed_carried": (_i, [_p, _p, _i64, _i, _i64, _p, _p, _p, _p]),
    "engpt_swiglu": (_i, [_p, _i, _p, _p, _f, _f, _i64, _i, _p, _i, _p]),
    "engpt_scale_rows_cast": (_i, [_p, _p, _f, _i64, _i64, _p, _i, _p]),
    "engpt_cast_f32_bf16_many": (_i, [_p, _p, _p, _i, _p]),
    "engpt_gemm_bf16": (_i, [_p, _i64, _p, _i64, _p, _i64, _i, _i, _i, _p]),
    "engpt_qkv_projection": (_i, [_p, _i, _p, _p, _p, _p, _i, _p, _f, _f, _i, _i, _i, _i, _p, _p]),
    "engpt_up_gate_swiglu": (_i, [_p, _p, _p, _p, _f, _f, _i64, _i, _i, _p, _p]),
    "engpt_gemm_carried_residual": (_i, [_p, _i64, _p, _i64, _i, _p, _p, _p, _f, _i, _f, _f, _f, _i64, _i, _p, _p,
                                         _p, _i, _p]),
    "engpt_cross_entropy": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _p, _p]),
    "engpt_logits_cross_entropy": (_i, [_p, _p, _i64, _i, _i64, _p, _i64, _p, _p, _p, _p, _p]),
    "engpt_cross_entropy_noalloc": (_i, [_p, _i, _i64, _i64, _i64, _p, _p, _p]),
    "engpt_normalize_rows": (_i, [_p, _i, _i64, _i64, _f, _p]),
    "engpt_normalize_columns": (_i, [_p, _i, _i64, _i64, _f, _p, _p]),
    "engpt_project_row_grad": (_i, [_p, _p, _i, _i64, _i64, _p]),
    "engpt_project_column_grad": (_i, [_p, _p, _i, _i64, _i64, _p, _p]),
    "engpt_column_scratch_floats": (_i64, [_i64, _i64]),
}
CE_NOALLOC_MAX_ROWS = 262144


class EngptError(RuntimeError):
    """Raised when a C-ABI call returns a non-zero engpt_status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({STATUS_NAMES.get(code, code)}): {msg}")
        self.code = code


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"engpt_b200 CUDA library not found at {LIB_PATH}; build it with `python -m engpt_b200.build`")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        msg = lib.engpt_last_error().decode(errors="replace")
        raise EngptError(name, rc, msg)


def device_status() -> int:
    """Device-side error word (synchronises the device); 0 when clean."""
    return int(load().engpt_device_status())


def clear_device_status() -> None:
    call("engpt_clear_device_status")


def raise_on_device_status(clear: bool = True) -> None:
    """Raise ``EngptError`` if a kernel recorded a failure (synchronises the device).

    The word holds the first failure since it was last cleared: an
    out-of-range token id or target (argument error) or a device wait that
    ran out (timeout), with the site that recorded it.  With ``clear`` the
    word is reset before raising, so the next check reports new failures only.
    """
    v = device_status()
    if v == 0:
        return
    if clear:
        clear_device_status()
    code, site = v & 0xFF, v >> 8
    raise EngptError("device status", code, f"recorded by a kernel at site {site} (word {v:#x})")


def stream_handle(device: Optional[torch.device] = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float32:
        return F32
    raise NotImplementedError(f"engpt_b200 kernels support float32 and bfloat16, got {dt}")
