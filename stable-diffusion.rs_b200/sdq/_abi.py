"""ctypes binding of libsdq.so (the C ABI declared in include/sdq.h).

The library is loaded from the package directory's parent
(``stable-diffusion.rs_b200/libsdq.so``), where ``build.py`` writes it.  There
is no fallback: if the library is missing or the device is not an sm_100 part,
every call raises :class:`SdqError`.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("SDQ_LIB", os.path.join(os.path.dirname(HERE), "libsdq.so"))

SDQ_OK = 0
SDQ_ERR_INVALID = 1
SDQ_ERR_UNSUPPORTED = 2
SDQ_ERR_CUDA = 3
SDQ_ERR_TIMEOUT = 4
SDQ_ERR_NCCL = 5

SDQ_F32 = 0
SDQ_BF16 = 1
SDQ_F16 = 2

#: Every symbol include/sdq.h declares, with (restype, argtypes).
_p, _i64, _i32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t
SIGNATURES = {
    "sdq_last_error": (ctypes.c_char_p, []),
    "sdq_abi_version": (_i32, []),
    "sdq_quantize": (_i32, [_p, _i32, _i64, _i64, _i32, _i32, ctypes.c_char_p, _p, _p, _p, _i32, _p]),
    "sdq_dequantize": (_i32, [_p, _p, _p, _i32, _i64, _i64, _i32, _i32, ctypes.c_char_p, _p, _i32, _p]),
    "sdq_quantized_matmul": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _i32, _i64, _i32, _i32, _i32,
                                    ctypes.c_char_p, _p, _p, _i32, _p]),
    "sdq_quantized_matmul_host": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _i32, _i64, _i32, _i32, _p, _p,
                                         _i32, _p, _p, _i64, _p]),
    "sdq_quantized_matmul_epilogue": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _i32, _i64, _i32, _i32,
                                             _p, _i32, _p, _p, _p, _i32, _p]),
    "sdq_resident_bytes": (_sz, [_i64, _i64, _i32, _i32, _i32]),
    "sdq_gguf_bytes": (_sz, [_i32, _i64]),
    "sdq_seeded_normals": (_i32, [ctypes.c_uint64, _i64, _p, _p]),
    "sdq_gguf_quantize": (_i32, [_p, _i32, _i64, _i64, _i32, _i32, _p, _p, _p, _i32, _p]),
    "sdq_gguf_dequantize": (_i32, [_p, _i32, _i64, _p, _i32, _p]),
    "sdq_device_status": (_i32, [_p]),
    "sdq_debug_wait_hook": (_i32, [ctypes.c_uint64, _i32, _p]),
    "sdq_comm_unique_id": (_i32, [_p]),
    "sdq_comm_init": (_i32, [_p, _i32, _i32, ctypes.POINTER(ctypes.c_void_p)]),
    "sdq_comm_destroy": (_i32, [_p]),
    "sdq_comm_output": (_i32, [_p, _i64, _i64, ctypes.POINTER(ctypes.c_void_p)]),
    "sdq_quantized_matmul_sharded": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _i32, _i64, _i32, _i32,
                                            _p, _p, _p, _i32, _p, _p]),
    "sdq_quantized_matmul_sharded_static": (_i32, [_p, _i32, _i64, _i64, _p, _p, _p, _i32, _i64, _i32,
                                                   _i32, _p, _p, _i32, _p, _p]),
}


class SdqError(RuntimeError):
    """A nonzero status from libsdq, with the library's per-thread message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"libsdq error {code}: {message}")
        self.code = code
        self.message = message


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise SdqError(SDQ_ERR_CUDA, f"{LIB_PATH} is missing; build it with "
                                         "`python stable-diffusion.rs_b200/build.py`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    return lib().sdq_last_error().decode("utf-8", "replace")


def check(rc: int) -> None:
    if rc != SDQ_OK:
        raise SdqError(rc, last_error())
