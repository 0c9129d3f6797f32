"""The C ABI without a GPU: the library loads, exports exactly what include/sdq.h
declares, and rejects invalid arguments with the reference-style status + per-thread
message before touching any device.  On a machine with no sm_100 device a valid call
fails loudly (no CPU fallback)."""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT, gpu_available
from sdq import _abi

HEADER = os.path.join(ROOT, "include", "sdq.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sdq_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    declared = declared_symbols()
    assert len(declared) >= 11
    out = subprocess.run(["nm", "-D", "--defined-only", os.path.join(PKG, "libsdq.so")],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\sT\s(sdq_\w+)", out))
    missing = [s for s in declared if s not in exported]
    assert not missing, missing
    # and the Python binding knows every one of them
    assert sorted(_abi.SIGNATURES) == declared


def test_library_loads_and_reports_version():
    L = _abi.lib()
    assert L.sdq_abi_version() == 1
    assert _abi.last_error() == ""


def test_resident_bytes_matches_the_reference_formula():
    L = _abi.lib()
    # packed words + scales + biases, 4 bytes each for scales/biases (mlx.rs:1981-1985)
    assert L.sdq_resident_bytes(1024, 1024, 64, 4, 4) == 1024 * 512 + 2 * 1024 * 16 * 4
    assert L.sdq_resident_bytes(1024, 1024, 64, 8, 2) == 1024 * 1024 + 2 * 1024 * 16 * 2
    assert L.sdq_resident_bytes(10, 100, 64, 4, 4) == 0     # K % 64 != 0
    assert L.sdq_resident_bytes(10, 128, 0, 0, 4) == 10 * 64 + 2 * 10 * 2 * 4  # defaults 64 / 4


def _qmm(x=1, m=4, k=128, n=64, bits=4, group=64, mode=b"affine", transpose=1, xdt=1, y=1):
    L = _abi.lib()
    p = lambda v: ctypes.c_void_p(v) if v else None  # noqa: E731
    return L.sdq_quantized_matmul(p(0x1000 * x), xdt, m, k, p(0x2000), p(0x3000), p(0x4000), 1, n,
                                  transpose, group, bits, mode, None, p(0x5000 * y), 1, None)


@pytest.mark.parametrize("kwargs,code,needle", [
    (dict(bits=3), _abi.SDQ_ERR_UNSUPPORTED, "bits 3"),
    (dict(bits=7), _abi.SDQ_ERR_INVALID, "bits must be"),
    (dict(group=32), _abi.SDQ_ERR_UNSUPPORTED, "group_size 32"),
    (dict(mode=b"mxfp4"), _abi.SDQ_ERR_UNSUPPORTED, "mxfp4"),
    (dict(k=100), _abi.SDQ_ERR_INVALID, "multiple of the group size"),
    (dict(m=0), _abi.SDQ_ERR_INVALID, "m (rows of x)"),
    (dict(n=0), _abi.SDQ_ERR_INVALID, "n (rows"),
    (dict(transpose=0), _abi.SDQ_ERR_UNSUPPORTED, "transpose=false"),
    (dict(x=0), _abi.SDQ_ERR_INVALID, "non-null"),
    (dict(xdt=2), _abi.SDQ_ERR_UNSUPPORTED, "bf16 or f32"),
])
def test_invalid_arguments_are_rejected_with_a_message(kwargs, code, needle):
    assert _qmm(**kwargs) == code
    assert needle in _abi.last_error()


def test_misaligned_pointer_is_rejected():
    L = _abi.lib()
    rc = L.sdq_quantized_matmul(ctypes.c_void_p(0x1002), 1, 4, 128, ctypes.c_void_p(0x2000),
                                ctypes.c_void_p(0x3000), ctypes.c_void_p(0x4000), 1, 64, 1, 64, 4,
                                b"affine", None, ctypes.c_void_p(0x5000), 1, None)
    assert rc == _abi.SDQ_ERR_INVALID and "misaligned" in _abi.last_error()


def test_error_text_is_per_thread_and_cleared_by_success():
    import threading

    assert _qmm(bits=3) == _abi.SDQ_ERR_UNSUPPORTED
    seen = {}

    def other():
        seen["msg"] = _abi.last_error()

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen["msg"] == ""                 # another thread sees no error
    assert "bits 3" in _abi.last_error()     # this one still does
    _abi.lib().sdq_abi_version()
    assert _abi.lib().sdq_resident_bytes(1, 64, 64, 4, 4) > 0


@pytest.mark.skipif(gpu_available(), reason="checks the no-device path")
def test_no_cpu_fallback_without_a_device():
    """A fully valid call on a machine without an sm_100 device fails with SDQ_ERR_CUDA."""
    assert _qmm() == _abi.SDQ_ERR_CUDA
    assert _abi.last_error()


def test_sharded_argument_checks():
    L = _abi.lib()
    rc = L.sdq_quantized_matmul_sharded(None, 1, 4, 128, None, None, None, 1, 64, 64, 4, None, None,
                                        None, 1, None, None)
    assert rc == _abi.SDQ_ERR_INVALID and "non-null" in _abi.last_error()
    h = ctypes.c_void_p()
    assert L.sdq_comm_init(None, 2, 0, ctypes.byref(h)) == _abi.SDQ_ERR_INVALID
    buf = (ctypes.c_uint8 * 128)()
    assert L.sdq_comm_init(buf, 2, 5, ctypes.byref(h)) == _abi.SDQ_ERR_INVALID
    assert "rank" in _abi.last_error()


# ---------------------------------------------------------------- later entry points

def test_gguf_bytes_follow_the_block_table():
    L = _abi.lib()
    table = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 8: (32, 34), 12: (256, 144), 13: (256, 176),
             14: (256, 210)}
    for kind, (per, nb) in table.items():
        assert L.sdq_gguf_bytes(kind, 4 * 256) == 4 * 256 // per * nb
    assert L.sdq_gguf_bytes(12, 100) == 0          # not whole blocks
    assert L.sdq_gguf_bytes(3, 256) == 0           # Q4_1: not supported


@pytest.mark.parametrize("kind,n,k,bits,code,needle", [
    (3, 4, 256, 4, _abi.SDQ_ERR_UNSUPPORTED, "GGML type 3"),
    (12, 4, 320, 4, _abi.SDQ_ERR_INVALID, "whole blocks"),
    (12, 4, 100, 4, _abi.SDQ_ERR_INVALID, "multiple of the group size"),
    (12, 4, 256, 3, _abi.SDQ_ERR_UNSUPPORTED, "bits 3"),
])
def test_gguf_quantize_rejects_bad_arguments(kind, n, k, bits, code, needle):
    L = _abi.lib()
    p = ctypes.c_void_p(0x10000)
    rc = L.sdq_gguf_quantize(p, kind, n, k, 64, bits, p, p, p, _abi.SDQ_BF16, None)
    assert rc == code and needle in _abi.last_error()
    rc = L.sdq_gguf_dequantize(p, 3, 256, p, _abi.SDQ_F32, None)
    assert rc == _abi.SDQ_ERR_UNSUPPORTED


def test_epilogue_rejects_an_unknown_activation_and_a_partial_overlap():
    L = _abi.lib()
    p = ctypes.c_void_p(0x10000)
    rc = L.sdq_quantized_matmul_epilogue(p, 1, 4, 128, p, p, p, 1, 64, 64, 4, None, 9, None, None, p, 1, None)
    assert rc == _abi.SDQ_ERR_INVALID and "act must be" in _abi.last_error()
    rc = L.sdq_quantized_matmul_epilogue(p, 1, 4, 128, p, p, p, 1, 64, 64, 4, None, 0, None,
                                         ctypes.c_void_p(0x10000 + 128), p, 1, None)
    assert rc == _abi.SDQ_ERR_INVALID and "overlaps" in _abi.last_error()


def test_comm_output_and_seeded_normals_check_their_arguments():
    L = _abi.lib()
    out = ctypes.c_void_p()
    assert L.sdq_comm_output(None, 4, 4, ctypes.byref(out)) == _abi.SDQ_ERR_INVALID
    assert L.sdq_seeded_normals(1, -1, None, None) == _abi.SDQ_ERR_INVALID
    assert L.sdq_seeded_normals(1, 0, None, None) == _abi.SDQ_OK
