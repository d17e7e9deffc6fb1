"""hv_gemm_i8_acc_noalloc, the allocation-free accumulator GEMM, against
hv_gemm_i8_acc through the C ABI.

This file sorts last so it also runs after every other GPU test in the same
process (the per-device scratch address is resolved on the first call; the
test must pass whether or not other work ran on the device before it).
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _lib():
    from heatvit_b200._lib import lib
    return lib()


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _run(fn, a, b, bias, m, n, k, transpose_b, a_unsigned):
    acc = torch.full((m, n), -7, dtype=torch.int64, device="cuda")
    rc = fn(C.c_void_p(a.data_ptr()), C.c_void_p(b.data_ptr()),
            C.c_void_p(bias.data_ptr()) if bias is not None else None,
            m, n, k, transpose_b, a_unsigned, C.c_void_p(acc.data_ptr()), _stream())
    return rc, acc


def _case(seed, m, n, k, transpose_b, a_unsigned, with_bias):
    g = np.random.default_rng(seed)
    a = g.integers(0 if a_unsigned else -128, 256 if a_unsigned else 128, (m, k))
    b = g.integers(-128, 128, (n, k) if transpose_b else (k, n))
    bias = g.integers(-(1 << 31), (1 << 31) - 1, n) if with_bias else None
    da = torch.from_numpy(a.astype(np.uint8 if a_unsigned else np.int8)).cuda()
    db = torch.from_numpy(b.astype(np.int8)).cuda()
    dbias = torch.from_numpy(bias.astype(np.int32)).cuda() if with_bias else None
    bt = b.astype(np.int64) if not transpose_b else b.T.astype(np.int64)
    want = a.astype(np.int64) @ bt + (bias.astype(np.int64)[None, :] if with_bias else 0)
    return da, db, dbias, want


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_noalloc_matches_allocating_gemm_twice_in_a_row():
    L = _lib()
    cases = [
        # (seed, m, n, k, transpose_b, a_unsigned, bias)
        (11, 333, 200, 300, 0, 0, True),    # ragged m, n and k: every padding path
        (12, 197, 64, 100, 1, 1, False),    # smaller k after a larger one: stale pad bytes must not leak
    ]
    for seed, m, n, k, tb, au, wb in cases:
        da, db, dbias, want = _case(seed, m, n, k, tb, au, wb)
        rc_ref, ref = _run(L.hv_gemm_i8_acc, da, db, dbias, m, n, k, tb, au)
        rc_new, got = _run(L.hv_gemm_i8_acc_noalloc, da, db, dbias, m, n, k, tb, au)
        assert rc_ref == 0 and rc_new == 0, L.hv_last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, ref), f"case {seed}: differs from hv_gemm_i8_acc"
        np.testing.assert_array_equal(got.cpu().numpy(), want)


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")
def test_noalloc_rejects_problems_beyond_the_scratch():
    L = _lib()
    limit = 8 << 20
    m, n, k = 50000, 192, 192                 # m * k alone is above the 8 MiB array
    assert m * k > limit
    da = torch.zeros((m, k), dtype=torch.int8, device="cuda")
    db = torch.zeros((k, n), dtype=torch.int8, device="cuda")
    rc, acc = _run(L.hv_gemm_i8_acc_noalloc, da, db, None, m, n, k, 0, 0)
    from heatvit_b200 import abi
    assert rc == abi.HV_ERR_VALUE
    msg = L.hv_last_error().decode()
    assert "HV_NOALLOC_SCRATCH_BYTES" in msg and str(limit) in msg
    torch.cuda.synchronize()
    assert bool((acc == -7).all()), "a rejected call must not write its output"
    # the scratch is still usable afterwards
    da, db, dbias, want = _case(13, 130, 96, 64, 0, 0, True)
    rc, got = _run(L.hv_gemm_i8_acc_noalloc, da, db, dbias, 130, 96, 64, 0, 0)
    assert rc == 0, L.hv_last_error()
    np.testing.assert_array_equal(got.cpu().numpy(), want)
