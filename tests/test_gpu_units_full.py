"""Unit configurations at their full sizes, through the C ABI, against the CPU
oracle, bit for bit.

Config 1: the isolated int8 GEMM + requant writeback (gemm.py:93-139) at the
DeiT-T layer shapes stacked over 256 images (M = 256 * 197 = 50,432 rows; the
patch GEMM M = 256 * 196 = 50,176), A int8 in [-128, 127], W in [-127, 127],
bias int32 in [-2^15, 2^15], a and w exponents in [-20, -8], dst = a + w + s
with s = 11 (K = 192) or 12 (K = 768); plus a small-M sweep of s over [0, 31]
and of left shifts for the rounding and saturation paths.  The accumulators of
the check come from a float64 matrix product (exact: every |acc| < 2^53) and the
writeback from the oracle's restatement of gemm_writeback.

Config 2: LayerNorm over [256 * 197][192] rows (nonlinear.py:136-186), the
attention shift-softmax over [256 * 3 * 197] rows of 197 Gaussian scores with
sigma 2^12 at score exponent -17 (nonlinear.py:98-133, transformer.py:240-252),
and the FFN GELU chain over [256 * 197 * 768] int32 accumulators with sigma 2^10
(transformer.py:351-358).
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

B = 256


def _lib():
    from heatvit_b200._lib import lib
    return lib()


def _stream(torch):
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _gemm_i8(torch, a, w, bias, src, dst, bits, transpose_b=False):
    m, k = a.shape
    n = w.shape[0] if transpose_b else w.shape[1]
    da = torch.from_numpy(np.ascontiguousarray(a, np.int8)).cuda()
    dw = torch.from_numpy(np.ascontiguousarray(w, np.int8)).cuda()
    db = torch.from_numpy(np.ascontiguousarray(bias, np.int32)).cuda() if bias is not None else None
    out = torch.empty((m, n), dtype=torch.int8 if bits == 8 else torch.int32, device="cuda")
    L = _lib()
    rc = L.hv_gemm_i8(C.c_void_p(da.data_ptr()), C.c_void_p(dw.data_ptr()),
                      C.c_void_p(db.data_ptr()) if db is not None else None, m, n, k, int(transpose_b), 0,
                      src, dst, bits, C.c_void_p(out.data_ptr()), _stream(torch))
    assert rc == 0, L.hv_last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _acc(a, w, bias, transpose_b=False):
    wm = w.T if transpose_b else w
    acc = a.astype(np.float64) @ wm.astype(np.float64)
    acc = np.rint(acc).astype(np.int64)
    if bias is not None:
        acc += bias.astype(np.int64)[None, :]
    return acc


@pytest.mark.parametrize("name,m,k,n", [("qkv", B * 197, 192, 576), ("proj", B * 197, 192, 192),
                                        ("fc1", B * 197, 192, 768), ("fc2", B * 197, 768, 192),
                                        ("patch", B * 196, 768, 192)])
def test_config1_gemm_requant_full_size(cuda, oracle, name, m, k, n):
    torch = cuda
    rng = np.random.default_rng([20260815, k, n])
    a = rng.integers(-128, 128, (m, k), dtype=np.int64)
    w = rng.integers(-127, 128, (k, n), dtype=np.int64)
    bias = rng.integers(-(1 << 15), (1 << 15) + 1, n, dtype=np.int64)
    a_exp, w_exp = (int(v) for v in rng.integers(-20, -7, 2))
    src = a_exp + w_exp
    dst = src + (11 if k == 192 else 12)
    got = _gemm_i8(torch, a, w, bias, src, dst, 8)
    want = oracle.writeback(_acc(a, w, bias), src, dst, 8)
    np.testing.assert_array_equal(got, want, err_msg=name)
    if name == "qkv":  # the int32 writeback on the same accumulators
        dst32 = src + 5
        got32 = _gemm_i8(torch, a[:4099], w, bias, src, dst32, 32)
        np.testing.assert_array_equal(got32, oracle.writeback(_acc(a[:4099], w, bias), src, dst32, 32))


@pytest.mark.parametrize("k,n", [(192, 192), (192, 64), (96, 100)])
def test_config1_small_m_shift_sweep(cuda, oracle, k, n):
    """Every right shift s in [0, 31] plus left shifts, on small M: the rounding
    (ties away from zero) and int8 / int32 saturation paths of the writeback, for
    the persistent layer-shape kernel (192 x 192) and the tiled kernel."""
    torch = cuda
    rng = np.random.default_rng([7, k, n])
    m = 300
    a = rng.integers(-128, 128, (m, k), dtype=np.int64)
    w = rng.integers(-127, 128, (k, n), dtype=np.int64)
    a[:4] = 127
    w[:, :3] = 127  # saturating corner: large positive accumulators
    bias = rng.integers(-(1 << 15), (1 << 15) + 1, n, dtype=np.int64)
    bias[0] = 1 << 30  # pushes the 64-bit epilogue form
    acc = _acc(a, w, bias)
    for s in list(range(0, 32)) + [-1, -5, -20]:
        for bits in (8, 32):
            got = _gemm_i8(torch, a, w, bias, -30, -30 + s, bits)
            np.testing.assert_array_equal(got, oracle.writeback(acc, -30, -30 + s, bits),
                                          err_msg=f"s={s} bits={bits}")


def test_config2_layernorm_full_size(cuda, oracle):
    from heatvit_b200.nonlinear import layernorm_rows
    rng = np.random.default_rng(20260815)
    x = rng.integers(-128, 128, (B * 197, 192))
    x[::997] = x[::997, :1]  # constant rows: zero variance
    gm, bt = rng.integers(-128, 128, 192), rng.integers(-128, 128, 192)
    xs, gs, bs, os_ = -9, -14, -15, -13
    out, neg = layernorm_rows(x, gm, bt, xs, gs, bs, os_)
    ref, rneg = oracle.layernorm(x, gm, bt, xs, gs, bs, os_)
    np.testing.assert_array_equal(out, ref)
    np.testing.assert_array_equal(neg, rneg)


def test_config2_softmax_full_size(cuda, oracle):
    from heatvit_b200.nonlinear import softmax_rows
    rng = np.random.default_rng(20260815)
    rows = B * 3 * 197
    s = np.clip(np.rint(rng.normal(0, 4096, (rows, 197))), -(1 << 31), (1 << 31) - 1).astype(np.int64)
    # score at exponent -17 -> Q8.16: sat24(rsa(score, -(-17 + 13))), a rounding right
    # shift by 4 (transformer.py:240-252)
    q16 = oracle.requant_array(s, 0, 4, 24).reshape(-1)
    lens = np.full(rows, 197)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    np.testing.assert_array_equal(softmax_rows(q16, lens, 0), oracle.softmax_rows(q16, off, 0))


def test_config2_gelu_chain_full_size(cuda, oracle):
    from heatvit_b200.nonlinear import gelu_requant_array
    rng = np.random.default_rng(20260815)
    acc = np.rint(rng.normal(0, 1024, B * 197 * 768)).astype(np.int64)
    got = gelu_requant_array(acc, -14, -7)
    np.testing.assert_array_equal(np.asarray(got).reshape(-1), oracle.gelu_chain_array(acc, -14, -7))
