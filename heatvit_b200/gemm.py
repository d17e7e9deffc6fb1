"""GPU mirror of verification/heatvit_ref/gemm.py (gemm, gemm_numpy, gemm_writeback).

Same signatures, argument meaning and exceptions; the arithmetic runs in the
int8 tensor-core GEMM of the CUDA library (hv_gemm_i8_acc) and the element-wise
writeback kernel (hv_writeback_i64).  Results come back as Python lists, as
in the golden model.
"""

import ctypes as C

import numpy as np

from ._convert import check_int, int_array, to_device, to_list
from ._lib import check, lib
from .engine import _stream, _torch


def _gemm_acc(a, b, bias, transpose_b, a_unsigned):
    torch = _torch()
    lo, hi = (0, 255) if a_unsigned else (-128, 127)
    a = int_array("a", a, lo, hi, ndim=2)
    b = int_array("b", b, -128, 127, ndim=2)
    m = a.shape[0]
    k = a.shape[1] if m else 0
    if transpose_b:
        n, k_b = b.shape[0], (b.shape[1] if b.shape[0] else 0)
    else:
        k_b, n = b.shape[0], (b.shape[1] if b.shape[0] else 0)
    if k != k_b:
        raise ValueError(f"K mismatch: a has {k}, b has {k_b}")
    if bias is not None:
        if not isinstance(bias, (list, tuple, np.ndarray)) or len(bias) != n:
            raise ValueError(f"bias must have length {n}")
        bias = int_array("bias", bias, -(1 << 31), (1 << 31) - 1, ndim=1, dtype=np.int32)
    if m == 0 or n == 0:
        return np.zeros((m, n), np.int64)
    dev = torch.device("cuda", torch.cuda.current_device())
    da = to_device(a.astype(np.uint8 if a_unsigned else np.int8), torch, dev)
    db = to_device(b.astype(np.int8), torch, dev)
    dbias = to_device(bias, torch, dev) if bias is not None else None
    acc = torch.empty((m, n), dtype=torch.int64, device=dev)
    if k == 0:
        acc.zero_()
        if dbias is not None:
            acc += dbias.to(torch.int64)[None, :]
    else:
        check(lib().hv_gemm_i8_acc(C.c_void_p(da.data_ptr()), C.c_void_p(db.data_ptr()),
                                   C.c_void_p(dbias.data_ptr()) if dbias is not None else None,
                                   m, n, k, int(bool(transpose_b)), int(bool(a_unsigned)),
                                   C.c_void_p(acc.data_ptr()), _stream(torch)))
    return acc.cpu().numpy()


def gemm_numpy(a, b, bias, transpose_b, a_unsigned=False):
    """gemm.py:93-120: A[M][K]·B[K][N] (+ bias) as exact integers."""
    return _gemm_acc(a, b, bias, transpose_b, a_unsigned).tolist()


def gemm(a, b, bias, transpose_b, a_unsigned=False):
    """gemm.py:58-90 (proven equal to gemm_numpy by the reference's tests)."""
    return gemm_numpy(a, b, bias, transpose_b, a_unsigned)


def writeback_array(accum, src_exp, dst_exp, output_bits):
    """Array form of gemm_writeback on the GPU; returns numpy int8/int32."""
    torch = _torch()
    src_exp = check_int("src_exp", src_exp)
    dst_exp = check_int("dst_exp", dst_exp)
    output_bits = check_int("output_bits", output_bits)
    if output_bits not in (8, 24, 32):
        raise ValueError("output_bits must be 8 or 32")
    acc = int_array("accum", accum, -(1 << 63), (1 << 63) - 1)
    dev = torch.device("cuda", torch.cuda.current_device())
    dacc = to_device(acc.reshape(-1), torch, dev)
    out = torch.empty(acc.size, dtype=torch.int8 if output_bits == 8 else torch.int32, device=dev)
    check(lib().hv_writeback_i64(C.c_void_p(dacc.data_ptr()), acc.size, src_exp, dst_exp, output_bits,
                                 C.c_void_p(out.data_ptr()), _stream(torch)))
    return out.cpu().numpy().reshape(acc.shape)


def gemm_writeback(accum, src_exp, dst_exp, output_bits):
    """gemm.py:123-139: requant every accumulator to int8 or int32."""
    if isinstance(output_bits, float):
        raise TypeError("output_bits must be an integer, got float")
    if output_bits not in (8, 32):
        raise ValueError("output_bits must be 8 or 32")
    if not isinstance(accum, (list, tuple, np.ndarray)):
        raise TypeError("accum must be a list of rows")
    return to_list(writeback_array(accum, src_exp, dst_exp, output_bits))
