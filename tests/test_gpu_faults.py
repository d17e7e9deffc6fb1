"""The bounded-wait error path on the GPU, made without a fault.

Every wait of the layer GEMMs on an mbarrier is bounded (a timeout sets the
model's device error word; the reference's RTL reports a watchdog timeout as a
fatal error code, rtl/include/heatvit_pkg.sv:109-118).  The test hook
hv_test_gemm_stall leaves one A tile of every layer-GEMM launch unloaded, so the
waits on it run out; the launch must then drain what it already issued, return,
and report code 3 through hv_device_error, with the context still usable: the
next inference without the hook is bit-exact again."""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_gemm_wait_runs_out_reports_and_recovers(cuda):
    torch = cuda
    from heatvit_b200 import _lib, synth
    from heatvit_b200.engine import Engine
    L = _lib.lib()
    eng = Engine(synth.config3_params(synth.SEED))
    imgs = torch.from_numpy(synth.baseline_images(synth.SEED, 64)).cuda()
    good = eng.infer(imgs)
    torch.cuda.synchronize()
    assert eng.device_error() == 0
    want = {k: good[k].cpu().numpy() for k in ("logits", "token_counts", "warnings")}

    # tile 0 of every layer GEMM never arrives; 2^16 polls per wait
    _lib.check(L.hv_test_gemm_stall(eng.handle, C.c_uint(1 << 16), 0))
    eng.infer(imgs)
    torch.cuda.synchronize()
    assert eng.device_error() == 3
    assert eng.device_error() == 0  # reading clears the word

    _lib.check(L.hv_test_gemm_stall(eng.handle, C.c_uint(0), -1))
    for _ in range(2):
        again = eng.infer(imgs)
        torch.cuda.synchronize()
        assert eng.device_error() == 0
        for k, v in want.items():
            np.testing.assert_array_equal(again[k].cpu().numpy(), v, err_msg=k)


def test_gemm_stall_hook_rejects_bad_tile(cuda):
    from heatvit_b200 import _lib, abi, synth
    from heatvit_b200.engine import Engine
    L = _lib.lib()
    eng = Engine(synth.config3_params(synth.SEED))
    assert L.hv_test_gemm_stall(eng.handle, C.c_uint(0), -2) == abi.HV_ERR_VALUE
