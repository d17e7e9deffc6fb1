"""GPU mirror of verification/heatvit_ref/nonlinear.py.

Scalar golden functions (gelu, plan_sigmoid) keep their signatures; array
forms (gelu_array, plan_array, gelu_requant_array, softmax_rows) are the
batched entry points.  Constants are the golden model's (nonlinear.py:30-55);
the attention softmax delta is 65536 (nonlinear.py:48), not the stale value in
config/heatvit_t.json.
"""

import ctypes as C

import numpy as np

from ._convert import check_int, int_array, to_device
from ._lib import check, lib
from .engine import _stream, _torch

GELU_SLOPE_NUM_Q16 = 11
GELU_SLOPE_SHIFT = 4
GELU_SLOPE_ROUND_ADD = 15
GELU_EXP_NEG_Q_MAX = 16
GELU_EXP_POS_Q_MAX = 7
PLAN_BP_1_Q16 = 65536
PLAN_BP_2_Q16 = 155648
PLAN_BP_3_Q16 = 327680
PLAN_C0_Q16 = 32768
PLAN_C1_Q16 = 40960
PLAN_C2_Q16 = 55296
PLAN_ONE_Q16 = 65536
SOFTMAX_LN2_Q16 = 45426
SOFTMAX_QUAD_Q16 = 23495
SOFTMAX_OFFSET_Q16 = 88670
SOFTMAX_CONST_Q16 = 22544
SOFTMAX_DELTA2_Q16_ATTENTION = 65536
SOFTMAX_DELTA2_Q16_SELECTOR = 65536
LAYERNORM_D = 192
LN_EPS_Q32 = 4295


def _dev(torch):
    return torch.device("cuda", torch.cuda.current_device())


def _elementwise(fn, x):
    torch = _torch()
    a = int_array("x", x, -(1 << 31), (1 << 31) - 1, dtype=np.int32)
    dev = _dev(torch)
    dx = to_device(a.reshape(-1), torch, dev)
    out = torch.empty_like(dx)
    check(fn(C.c_void_p(dx.data_ptr()), dx.numel(), C.c_void_p(out.data_ptr()), _stream(torch)))
    return out.cpu().numpy().reshape(a.shape)


def gelu_array(x):
    """ShiftGELU (nonlinear.py:60-80) on an int32 array of Q8.16 values."""
    return _elementwise(lib().hv_shiftgelu, x)


def plan_array(x):
    """PLAN sigmoid (nonlinear.py:83-95) on an int32 array."""
    return _elementwise(lib().hv_plan_sigmoid, x)


def gelu(x):
    """nonlinear.py:60-80 on one Q8.16 value."""
    x = check_int("x", x)
    if not -(1 << 31) <= x < (1 << 31):
        raise ValueError("x outside int32")
    return int(gelu_array(np.array([x], np.int64))[0])


def plan_sigmoid(x):
    """nonlinear.py:83-95 on one Q8.16 value."""
    x = check_int("x", x)
    if not -(1 << 31) <= x < (1 << 31):
        raise ValueError("x outside int32")
    return int(plan_array(np.array([x], np.int64))[0])


def gelu_requant_array(acc, src_exp, dst_exp):
    """requant(gelu(requant(acc, src, -16, 24)), -16, dst, 8) on int32 accumulators
    (transformer.py:351-356)."""
    torch = _torch()
    a = int_array("acc", acc, -(1 << 31), (1 << 31) - 1, dtype=np.int32)
    dev = _dev(torch)
    da = to_device(a.reshape(-1), torch, dev)
    out = torch.empty(da.numel(), dtype=torch.int8, device=dev)
    check(lib().hv_gelu_requant(C.c_void_p(da.data_ptr()), da.numel(), check_int("src_exp", src_exp),
                                check_int("dst_exp", dst_exp), C.c_void_p(out.data_ptr()), _stream(torch)))
    return out.cpu().numpy().reshape(a.shape)


def softmax_rows(values, lengths, mode):
    """Ragged rows (concatenated ``values`` split by ``lengths``); mode 0 =
    attention (UQ0.8 uint8), 1 = selector (Q0.16 int32)."""
    torch = _torch()
    v = int_array("inputs", values, -(1 << 31), (1 << 31) - 1, dtype=np.int32).reshape(-1)
    lengths = np.asarray(lengths, np.int64)
    if np.any(lengths <= 0):
        raise ValueError("softmax row must not be empty")
    off = np.zeros(lengths.size + 1, np.int32)
    off[1:] = np.cumsum(lengths)
    if off[-1] != v.size:
        raise ValueError("row lengths do not cover the values")
    dev = _dev(torch)
    dv = to_device(v, torch, dev)
    doff = to_device(off, torch, dev)
    out = torch.empty(v.size, dtype=torch.uint8 if mode == 0 else torch.int32, device=dev)
    check(lib().hv_softmax_rows(C.c_void_p(dv.data_ptr()), C.c_void_p(doff.data_ptr()), lengths.size, int(mode),
                                C.c_void_p(out.data_ptr()), _stream(torch)))
    return out.cpu().numpy()


def softmax_selector(inputs):
    """nonlinear.py:124-127: Q0.16 scaled softmax saturated at 65536."""
    if isinstance(inputs, (list, tuple)) and not inputs:
        raise ValueError("softmax row must not be empty")
    v = int_array("inputs", inputs, -(1 << 31), (1 << 31) - 1).reshape(-1)
    if v.size == 0:
        raise ValueError("softmax row must not be empty")
    return softmax_rows(v, [v.size], 1).tolist()


def softmax_attention(inputs):
    """nonlinear.py:130-133: Q0.16 scaled softmax rounded to UQ0.8."""
    if isinstance(inputs, (list, tuple)) and not inputs:
        raise ValueError("softmax row must not be empty")
    v = int_array("inputs", inputs, -(1 << 31), (1 << 31) - 1).reshape(-1)
    if v.size == 0:
        raise ValueError("softmax row must not be empty")
    return softmax_rows(v, [v.size], 0).tolist()


def layernorm_rows(x, gamma, beta, x_scale, gamma_scale, beta_scale, out_scale):
    """LayerNorm over rows of 192 int8 channels on the GPU; returns
    (outputs int8 [rows][192], negative_variance bool [rows])."""
    torch = _torch()
    for name, value in (("x_scale", x_scale), ("gamma_scale", gamma_scale),
                        ("beta_scale", beta_scale), ("out_scale", out_scale)):
        check_int(name, value)
    if not -32 <= x_scale <= 0:
        raise ValueError("layernorm input scale must be in [-32, 0]")
    xa = int_array("channel value", x, -128, 127, dtype=np.int8)
    g = int_array("channel value", gamma, -128, 127, dtype=np.int8).reshape(-1)
    b = int_array("channel value", beta, -128, 127, dtype=np.int8).reshape(-1)
    if xa.shape[-1] != LAYERNORM_D or g.size != LAYERNORM_D or b.size != LAYERNORM_D:
        raise ValueError(f"layernorm rows must have exactly {LAYERNORM_D} channels")
    rows = xa.reshape(-1, LAYERNORM_D)
    dev = _dev(torch)
    dx, dg, dbt = to_device(rows, torch, dev), to_device(g, torch, dev), to_device(b, torch, dev)
    out = torch.empty_like(dx)
    neg = torch.empty(rows.shape[0], dtype=torch.uint8, device=dev)
    check(lib().hv_layernorm_i8(C.c_void_p(dx.data_ptr()), C.c_void_p(dg.data_ptr()), C.c_void_p(dbt.data_ptr()),
                                rows.shape[0], int(x_scale), int(gamma_scale), int(beta_scale), int(out_scale),
                                C.c_void_p(out.data_ptr()), C.c_void_p(neg.data_ptr()), _stream(torch)))
    return out.cpu().numpy().reshape(xa.shape), neg.cpu().numpy().astype(bool)


def layernorm(xs, gammas, betas, x_scale, gamma_scale, beta_scale, out_scale):
    """nonlinear.py:136-186: one D=192 row -> (outputs, negative_variance)."""
    for name, value in (("x_scale", x_scale), ("gamma_scale", gamma_scale),
                        ("beta_scale", beta_scale), ("out_scale", out_scale)):
        check_int(name, value)
    if not -32 <= x_scale <= 0:
        raise ValueError("layernorm input scale must be in [-32, 0]")
    if not (len(xs) == len(gammas) == len(betas) == LAYERNORM_D):
        raise ValueError(f"layernorm rows must have exactly {LAYERNORM_D} channels")
    out, neg = layernorm_rows([list(xs)], gammas, betas, x_scale, gamma_scale, beta_scale, out_scale)
    return out[0].tolist(), bool(neg[0])
