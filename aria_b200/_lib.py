"""ctypes binding of libaria_q4.so (include/aria_q4.h).

There is deliberately no fallback: if the shared library is missing or the
current device is not a B200, every call raises.  Python is only the host-side
mirror of the reference's call surface; all arithmetic happens in the CUDA
kernels behind the C ABI.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libaria_q4.so")

# status codes (aria_q4_status)
OK, EINVAL, EUNSUPPORTED, EALIGN, ECUDA, ENODEVICE, ESIZE = range(7)
LAYOUT_KN, LAYOUT_NK = 0, 1
FLAG_CONST_WEIGHTS = 1
FLAG_KERNEL_STREAM = 2
FLAG_KERNEL_REGISTER = 4
FLAG_KERNEL_TENSOR = 8
FLAG_EPILOGUE_GELU = 16
F32, F16 = 0, 1

# every symbol include/aria_q4.h declares: (restype, argtypes)
_P = ctypes.c_void_p
_SZ = ctypes.c_size_t
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "aria_q4_0_packed_bytes": (_SZ, [_SZ]),
    "aria_q4_0_pack_f16": (_I, [_P, _SZ, _P, _P]),
    "aria_q4_0_pack_f32": (_I, [_P, _SZ, _P, _P]),
    "aria_q4_0_unpack_f32": (_I, [_P, _SZ, _P, _P]),
    "aria_q4_0_tiled_bytes": (_SZ, [_I, _I]),
    "aria_q4_0_repack": (_I, [_P, _I, _I, _I, _P, _SZ, _P]),
    "aria_q4_0_quantize_tiled": (_I, [_P, _I, _I, _I, _P, _SZ, _P]),
    "aria_q4_0_matmul": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _F, _F, _P]),
    "aria_q4_0_matmul_ex": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _F, _F, _I, _P]),
    "aria_q4_0_workspace_bytes": (_SZ, [_I, _I, _I]),
    "aria_q4_0_matmul_ws": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _F, _F, _P, _SZ, _I, _P]),
    "aria_q4_0_kernel_choice": (_I, [_I, _I, _I, _I, _SZ, _I]),
    "aria_q4_0_matmul_static_ws": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, _P, _F, _F, _I, _P]),
    "aria_q4_0_workspace_counter_bytes": (_SZ, []),
    "aria_q4_test_tensor_stall": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _I, _I, ctypes.c_uint, _P]),
    "aria_q4_0_matmul_ln": (_I, [_P, _I, _I, _I, _P, _I, _I, _P, _P, _F, _P, _I, _I, _P, _F, _F, _I, _P]),
    "aria_embed_f16": (_I, [_P, _P, _I, _I, _I, _P, _P, _I, _P, _P]),
    "aria_layernorm_f32": (_I, [_P, _I, _I, _P, _P, _F, _P, _I, _P]),
    "aria_attention_decode": (_I, [_P, _I, _I, _I, _P, _P, _I, _P, _P, _P]),
    "aria_flash_attn_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _F, _P]),
    "aria_attention_prefill": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _I, _P]),
    "aria_p2p_alloc": (_I, [_SZ, _P]),
    "aria_p2p_free": (_I, [_P]),
    "aria_p2p_ipc_handle": (_I, [_P, _P]),
    "aria_p2p_ipc_open": (_I, [_P, _P]),
    "aria_p2p_ipc_close": (_I, [_P]),
    "aria_p2p_allreduce_add": (_I, [_P, _P, _P, _I, _I, _P, _I, ctypes.c_uint, _P]),
    "aria_q4_strerror": (ctypes.c_char_p, [_I]),
    "aria_q4_last_cuda_error": (_I, []),
    "aria_q4_take_device_error": (_I, []),
    "aria_q4_abi_version": (_I, []),
}


class AriaQ4Error(RuntimeError):
    def __init__(self, fn: str, status: int, cuda_err: int = 0):
        msg = _lib().aria_q4_strerror(status).decode() if _LIB is not None else str(status)
        if status == ECUDA:
            msg += f" (cudaError {cuda_err})"
        super().__init__(f"{fn}: {msg}")
        self.status = status
        self.cuda_error = cuda_err


_LIB = None


def _lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m aria_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def lib() -> ctypes.CDLL:
    return _lib()


def check(fn: str, status: int) -> None:
    if status != OK:
        raise AriaQ4Error(fn, status, _lib().aria_q4_last_cuda_error())


def call(fn: str, *args) -> None:
    check(fn, getattr(_lib(), fn)(*args))
