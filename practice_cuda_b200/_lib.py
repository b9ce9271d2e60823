"""ctypes binding of libpcb200.so (the C ABI declared in include/pcb200.h).

There is no fallback: if the library is missing or cannot load, every entry
point raises.  Build it with ``python -m practice_cuda_b200.build``.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libpcb200.so")

PCB_OK = 0
PCB_ERR_INVALID = 1
PCB_ERR_UNSUPPORTED = 2
PCB_ERR_LAYOUT = 3
PCB_ERR_LAUNCH = 4
PCB_ERR_DEVICE = 5
PCB_ERR_TIMEOUT = 6

PCB_DTYPE = {
    torch.float32: 0,
    torch.float16: 1,
    torch.bfloat16: 2,
    torch.float8_e4m3fn: 3,
    torch.float8_e5m2: 4,
}

PCB_ACT = {"none": 0, "gelu": 1}

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float

# name -> (restype, argtypes)
_SIGNATURES = {
    "pcb_version": (_i, []),
    "pcb_status_name": (ctypes.c_char_p, [_i]),
    "pcb_last_error_text": (ctypes.c_char_p, []),
    "pcb_get_device_error": (_i, [ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "pcb_debug_inject_error": (_i, [_i]),
    "pcb_quant_per_block": (
        _i,
        [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
         _f, _vp],
    ),
    "pcb_quant_per_block_pow2": (
        _i,
        [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64, _i64,
         _f, _vp],
    ),
    "pcb_quant_per_channel": (
        _i,
        [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _i, _f, _vp],
    ),
    "pcb_quant_per_tensor_workspace_floats": (_i64, []),
    "pcb_quant_float8_dynamic": (
        _i,
        [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _i64, _i64, _i, _f, _vp, _vp],
    ),
    "pcb_quant_per_tensor": (
        _i,
        [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _vp, _i, _f, _f, _vp, _vp],
    ),
    "pcb_quant_per_tensor_noalloc": (
        _i,
        [_vp, _i, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i, _i64, _i64, _i64, _vp, _vp, _i, _f, _f, _vp],
    ),
    "pcb_bmm_scaled": (
        _i,
        [_vp, _i64, _i64, _i64,  # a
         _vp, _i64, _i64, _i64, _i,  # b, ab dtype
         _i64, _i64, _i64, _i64,  # batch m n k
         _vp, _i64, _i64, _i64, _i64,  # scale a, strides, qbm
         _vp, _i64, _i64, _i64, _i64,  # scale b, strides, qbn
         _i64,  # qbk
         _vp, _i, _i64, _i64, _i64,  # bias
         _vp, _i, _i64, _i64, _i64,  # c
         _i, _vp],
    ),
    "pcb_bmm_scaled_mixed": (
        _i,
        [_vp, _i64, _i64, _i64, _i,  # a, a dtype
         _vp, _i64, _i64, _i64, _i,  # b, b dtype
         _i64, _i64, _i64, _i64,  # batch m n k
         _vp, _i64, _i64, _i64, _i64,  # scale a, strides, qbm
         _vp, _i64, _i64, _i64, _i64,  # scale b, strides, qbn
         _i64,  # qbk
         _vp, _i, _i64, _i64, _i64,  # bias
         _vp, _i, _i64, _i64, _i64,  # c
         _i, _vp],
    ),
    "pcb_bmm_block_scaled_workspace_bytes": (_i64, [_i64, _i64, _i64, _i64]),
    "pcb_bmm_block_scaled": (
        _i,
        [_vp, _i64, _i64, _i64,  # a
         _vp, _i64, _i64, _i64, _i,  # b, ab dtype
         _i64, _i64, _i64, _i64,  # batch m n k
         _vp, _i64, _i64, _i64, _i64,  # scale a, strides, qbm
         _vp, _i64, _i64, _i64, _i64,  # scale b, strides, qbn
         _i64,  # qbk
         _vp, _i, _i64, _i64, _i64,  # bias
         _vp, _i, _i64, _i64, _i64,  # c
         _i, _vp, _i64, _vp]),
    "pcb_quant_bmm_fused": (
        _i,
        [_vp, _i, _i64, _i64, _i64,  # x
         _vp, _i64, _i64, _i64, _i,  # b
         _i64, _i64, _i64, _i64,  # batch m n k
         _vp, _i64, _i64, _i64, _i64,  # scale b, strides, qbn
         _vp, _i, _i64, _i64, _i64,  # bias
         _vp, _i, _i64, _i64, _i64,  # c
         _vp, _i64, _i64,  # xq
         _vp, _i64, _i64, _i64,  # xs
         _i, _f, _vp],
    ),
    "pcb_pack_u8": (_i, [_vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class Pcb200Error(RuntimeError):
    """A libpcb200 entry point returned a non-zero pcb_status."""

    def __init__(self, status: int, what: str, detail: str):
        self.status = status
        super().__init__(f"{what}: {status_name(status)}: {detail}")


def use_library(path: str) -> None:
    """Load another build of the same library (a ``PCB200_PROFILING`` build)
    instead of the in-tree one.  Must be called before the first entry point
    runs; for profiling and tests only."""
    global LIB_PATH
    with _lock:
        if _lib is not None:
            raise RuntimeError("libpcb200 is already loaded")
        LIB_PATH = path


def lib() -> ctypes.CDLL:
    """The loaded library; raises if it is missing (there is no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libpcb200.so not found at {LIB_PATH}; build it with "
                    "`python -m practice_cuda_b200.build` (nvcc, sm_100a)"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def status_name(status: int) -> str:
    return lib().pcb_status_name(status).decode()


def check(status: int, what: str) -> None:
    if status != PCB_OK:
        raise Pcb200Error(status, what, lib().pcb_last_error_text().decode())


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return PCB_DTYPE[dtype]
    except KeyError as exc:
        raise ValueError(f"unsupported dtype for libpcb200: {dtype}") from exc


def device_error() -> tuple[int, int, int]:
    """(code, site, info) of the device error word; reading clears it."""
    code, site, info = _i(0), _i(0), _i(0)
    check(lib().pcb_get_device_error(ctypes.byref(code), ctypes.byref(site), ctypes.byref(info)),
          "pcb_get_device_error")
    return code.value, site.value, info.value


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (libpcb200 has no CPU path), got {t.device}")
