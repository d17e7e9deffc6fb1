"""Loader for the in-tree CUDA library (heatvit_b200/_lib/libheatvit_b200.so).

There is no CPU fallback: every compute entry point of this package goes
through this library, and ``lib()`` raises when the library is missing or no
CUDA device is visible.  Status codes from the C ABI are turned into the
golden model's exception types (ValueError, TypeError, OverflowError).
"""

import ctypes as C
import os
import threading

from . import abi

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libheatvit_b200.so")
_lib = None
_lock = threading.Lock()

P = C.c_void_p
I = C.c_int
I64 = C.c_int64

_SIGNATURES = {
    "hv_version": (C.c_char_p, []),
    "hv_last_error": (C.c_char_p, []),
    "hv_model_create": (I, [P, I, C.POINTER(C.c_void_p)]),
    "hv_model_destroy": (I, [P]),
    "hv_infer_batch": (I, [P, P, I, P, P, P, P, P]),
    "hv_infer_batch_checkpoints": (I, [P, P, I, P, P, P, P, P, P, P]),
    "hv_infer_host": (I, [P, P, I, P, P, P, P]),
    "hv_infer_host_submit": (I, [P, P, I, P, P, P, P]),
    "hv_infer_host_wait": (I, [P]),
    "hv_gemm_i8": (I, [P, P, P, I, I, I, I, I, I, I, I, P, P]),
    "hv_gemm_i8_acc": (I, [P, P, P, I, I, I, I, I, P, P]),
    "hv_gemm_i8_acc_noalloc": (I, [P, P, P, I, I, I, I, I, P, P]),
    "hv_quantize_images": (I, [P, I, I, P, P]),
    "hv_layernorm_i8": (I, [P, P, P, I, I, I, I, I, P, P, P]),
    "hv_softmax_rows": (I, [P, P, I, I, P, P]),
    "hv_shiftgelu": (I, [P, I64, P, P]),
    "hv_plan_sigmoid": (I, [P, I64, P, P]),
    "hv_gelu_requant": (I, [P, I64, I, I, P, P]),
    "hv_transformer_block": (I, [P, I, P, P, I, I, P, P]),
    "hv_patch_embedding": (I, [P, P, I, P, P]),
    "hv_token_selector": (I, [P, I, P, P, P, I, P, P, P, P, P, P, P, P, P, P, P]),
    "hv_writeback_i64": (I, [P, I64, I, I, I, P, P]),
    "hv_profile_start": (I, [P, I, I]),
    "hv_device_error": (I, [P, C.POINTER(C.c_int)]),
    "hv_profile_stop": (I, [P, C.POINTER(C.c_int), C.POINTER(C.c_double), C.POINTER(C.c_longlong)]),
    "hv_graph_kernels": (I, [P, C.POINTER(C.c_int)]),
    "hv_test_gemm_stall": (I, [P, C.c_uint, I]),
    "hv_selector_h2": (I, [P, I, P, P, I, P, P]),
    "hv_align_add_i8": (I, [P, I, P, I, I, I64, P, P]),
}


def build_if_needed():
    from . import build
    return build.build()


def lib():
    """The loaded library; builds it when the sources are newer (this needs
    nvcc) and raises if CUDA is unavailable."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"CUDA library {LIB_PATH} is not built; run heatvit_b200.build.build() "
                    "(this package has no CPU fallback)")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def check(status):
    """Raise the golden model's exception type for a non-zero status."""
    if status == abi.HV_OK:
        return
    msg = lib().hv_last_error().decode(errors="replace")
    if status == abi.HV_ERR_VALUE:
        raise ValueError(msg)
    if status == abi.HV_ERR_TYPE:
        raise TypeError(msg)
    if status == abi.HV_ERR_OVERFLOW:
        raise OverflowError(msg)
    raise RuntimeError(f"heatvit_b200 error {status}: {msg}")
