"""ctypes binding of the sm_100a C-ABI library (``include/ltxfp8.h``).

The library is loaded lazily on first use.  There is no fallback: if the
library is missing, or the device is not an sm_100 part, every op raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "lib", "libltxfp8.so")

# Error codes of include/ltxfp8.h
OK = 0
ERR_INVALID_ARGUMENT = -1
ERR_UNSUPPORTED_SHAPE = -2
ERR_MISALIGNED = -3
ERR_CUDA = -4
ERR_DEVICE = -5
ERR_DEVICE_STATUS = -6

QUANT_TORCH = 0
QUANT_TRITON = 1

GELU_NONE = 0
GELU_TANH = 1       # torch's CUDA GELU-tanh formula (bit-identical bf16 results)
GELU_TANH_FAST = 2  # x / (1 + 2^a) with approximate instructions (within one bf16 ulp)

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2

_lock = threading.Lock()
_lib = None


class LtxFp8Error(RuntimeError):
    """Raised when a C-ABI call returns a non-zero code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"ltxfp8 error {code}: {msg}")
        self.code = code


class Epilogue(ctypes.Structure):
    _fields_ = [
        ("gelu_tanh", ctypes.c_int),
        ("requant_q", ctypes.c_void_p),
        ("requant_scales", ctypes.c_void_p),
        ("requant_ld", ctypes.c_int64),
        ("skip_d", ctypes.c_int),
        ("lora_ax", ctypes.c_void_p),
        ("lora_b", ctypes.c_void_p),
        ("lora_r", ctypes.c_int64),
        ("lora_alpha", ctypes.c_float),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("requant_mode", ctypes.c_int),
    ]


class GemmPlanInfo(ctypes.Structure):
    _fields_ = [
        ("workspace_bytes", ctypes.c_size_t),
        ("launches", ctypes.c_int),
        ("splits", ctypes.c_int),
        ("split_row0", ctypes.c_int64),
    ]


# name -> (restype, argtypes); the exported symbols of include/ltxfp8.h
_vp, _i64, _i32, _f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
SIGNATURES = {
    "ltxfp8_version": (_i32, []),
    "ltxfp8_last_error": (ctypes.c_char_p, []),
    "ltxfp8_quantize_1x128": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i32, _vp]),
    "ltxfp8_quantize_weight_128x128": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _vp]),
    "ltxfp8_dequantize_1x128": (_i32, [_vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp]),
    "ltxfp8_gemm": (_i32, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.POINTER(Epilogue), _vp]),
    "ltxfp8_gemm_fp6w": (_i32, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.POINTER(Epilogue), _vp]),
    "ltxfp8_lora_a": (_i32, [_vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "ltxfp8_gemm_set_variant": (_i32, [_i32]),
    "ltxfp8_gemm_workspace_bytes": (_i32, [_i64, _i64, _i64, ctypes.POINTER(ctypes.c_size_t)]),
    "ltxfp8_gemm_plan": (_i32, [_i64, _i64, _i64, _vp]),
    "ltxfp8_gemm_plan_for_sms": (_i32, [_i64, _i64, _i64, _i32, _vp]),
    "ltxfp8_adanorm_quantize": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _i32,
                                        _vp]),
    "ltxfp8_rms_fma": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _vp, _i64, _vp, _i32, _vp]),
    "ltxfp8_gated_attention": (_i32, [_vp, _vp, _i32, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i32, _vp]),
    "ltxfp8_gelu_quantize_1x128": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i32, _vp]),
    "ltxfp8_gelu_tanh_quantize_1x128": (_i32, [_vp, _i64, _i64, _i64, _vp, _i64, _vp, _i64, _i32, _vp]),
    "ltxfp8_rms_norm_rope": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _vp, _i32, _vp]),
    "ltxfp8_rms_norm_split_rope": (_i32, [_vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
                                          _vp, _vp, _i32, _vp]),
    "ltxfp8_lora_fuse_weight": (_i32, [_vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "ltxfp8_quantize_weight_128x128_scaled": (_i32, [_vp, _i32, _i64, _i64, _f32, _vp, _vp, _vp]),
    "ltxfp8_fp6_pack": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "ltxfp8_fp6_unpack": (_i32, [_vp, _i64, _i64, _vp, _vp]),
    "ltxfp8_fp6_to_tc": (_i32, [_vp, _vp, _i64, _i64, _vp, _vp, _vp]),
    "ltxfp8_gemm_static_scratch": (_i32, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64,
                                           ctypes.POINTER(Epilogue), _vp]),
    "ltxfp8_device_status": (_i32, [ctypes.POINTER(ctypes.c_uint), _i32, _vp]),
    "ltxfp8_selftest_wait_timeout": (_i32, [ctypes.c_ulonglong, ctypes.POINTER(ctypes.c_uint), _vp]),
}


def load(path: str | None = None):
    """Load (once) and return the ctypes handle of libltxfp8.so."""
    global _lib
    with _lock:
        if _lib is None:
            p = path or LIB_PATH
            if not os.path.exists(p):
                raise ImportError(
                    f"{p} is missing: build the sm_100a library first "
                    "(python ltx-2_b200/build.py, or __graft_entry__.build())")
            L = ctypes.CDLL(p)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != OK:
        msg = load().ltxfp8_last_error().decode(errors="replace")
        raise LtxFp8Error(rc, msg)


def device_status(stream: int = 0, clear: bool = True) -> int:
    """Read (and by default clear) the kernels' device status word; 0 = healthy."""
    st = ctypes.c_uint(0)
    check(load().ltxfp8_device_status(ctypes.byref(st), 1 if clear else 0, stream))
    return st.value


SELFTEST_STATUS = 0x5E1F0001


def selftest_wait_timeout(limit_ns: int, stream: int = 0) -> int:
    """Run the bounded-wait failure self-test; returns the status word it left."""
    st = ctypes.c_uint(0)
    check(load().ltxfp8_selftest_wait_timeout(limit_ns, ctypes.byref(st), stream))
    return st.value


GEMM_AUTO = 0
GEMM_ONE_CTA = 1
GEMM_CTA_PAIR = 2


def set_gemm_variant(variant: int) -> None:
    """Force the GEMM kernel (GEMM_AUTO, GEMM_ONE_CTA, GEMM_CTA_PAIR); process-wide."""
    check(load().ltxfp8_gemm_set_variant(variant))
    from .blockwise import ops  # the split-K workspace size and the launch plan depend on the kernel
    ops._WS_CACHE.clear()
    ops._PLAN_CACHE.clear()
