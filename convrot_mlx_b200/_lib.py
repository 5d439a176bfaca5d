"""ctypes binding of ``libconvrot_b200.so`` (declared in ``include/convrot_b200.h``).

The library is the only compute path of this package: there is no CPU or
PyTorch fallback.  Loading fails with an explicit error when the library has
not been built, and every call raises when the library reports an error.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libconvrot_b200.so")

OK = 0
ERR_INVALID = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3

F32, F16, BF16 = 0, 1, 2
LAYOUT_NK, LAYOUT_KN = 0, 1

DTYPE_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I = ctypes.c_int

# name -> (restype, argtypes); must match include/convrot_b200.h
SIGNATURES: dict[str, tuple] = {
    "convrot_abi_version": (_I, []),
    "convrot_last_error": (ctypes.c_char_p, []),
    "convrot_prepare_i8": (_I, [_P, _I, _I64, _I64, _I, _P, _P, _P]),
    "convrot_prepare_packed": (_I, [_P, _I, _I64, _I64, _I, _P, _P, _P]),
    "convrot_rotate": (_I, [_P, _I, _I64, _I64, _I, _P, _P]),
    "convrot_modnorm_prepare_i8": (_I, [_P, _I, _I64, _I64, _I, _P, _P, _I64, _I64, ctypes.c_float, _P, _P, _P]),
    "convrot_gelu_concat_prepare_i8": (_I, [_P, _I64, _I64, _P, _I64, _I64, _I64, _I, _P, _P, _P]),
    "convrot_unpack_int4": (_I, [_P, _I64, _P, _P]),
    "convrot_pack_int4": (_I, [_P, _I64, _P, _P]),
    "convrot_repack_int4_transpose": (_I, [_P, _I64, _I64, _P, _P]),
    "convrot_w4a4_gemm": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P]),
    "convrot_w4a16_gemm": (_I, [_P, _I, _P, _I, _P, _P, _P, _I, _I64, _I64, _I64, _P]),
    "convrot_w4a4_gemm_gather": (_I, [_P, _P, _I, _P, _P, _P, ctypes.POINTER(_P), _I, _I64, _I64, _I, _I64, _I64,
                                      _I64, _P]),
    "convrot_peer_barrier": (_I, [ctypes.POINTER(_P), _I, _I, ctypes.c_uint32, _P]),
    "convrot_copy_2d": (_I, [_P, _I64, _P, _I64, _I64, _I64, _P]),
    "convrot_w4a4_linear_static": (_I, [_P, _I, _I, _P, _I, _P, _P, _P, _I, _I64, _I64, _I64, _P]),
    "convrot_set_gemm_route": (_I, [_I]),
    "convrot_take_device_error": (_I, [ctypes.POINTER(_I)]),
}

_lock = threading.Lock()
_lib = None


class ConvRotError(RuntimeError):
    """A non-validation failure reported by libconvrot_b200.so."""


def load():
    """Load the library once (raises if it was not built)."""

    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m convrot_mlx_b200.build` "
                    "(the CUDA library is the only compute path: there is no fallback)"
                )
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status == OK:
        return
    msg = load().convrot_last_error().decode(errors="replace")
    if status == ERR_INVALID:
        raise ValueError(msg)
    if status == ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    raise ConvRotError(f"{what}: {msg}")


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def ptr(t: torch.Tensor | None):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def take_device_error() -> int:
    code = _I(0)
    check(load().convrot_take_device_error(ctypes.byref(code)), "convrot_take_device_error")
    return int(code.value)
