"""Per-operator parity on the GPU: every C-ABI operator against the reference's
KAT vectors, the golden-model fixtures and the CPU oracle.  Integer work, so
the bar is bit-exact everywhere."""

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu


# ---- GEMM -------------------------------------------------------------------------

def test_gemm_kat_scenarios(cuda):
    from heatvit_b200.gemm import gemm_numpy, gemm_writeback
    g = load_golden("kat_gemm.npz")
    for name in g["names"]:
        m, n, k, heads, tr, uns, bits, has_bias, src, dst = (int(v) for v in g[f"{name}_meta"])
        bias = g[f"{name}_bias"].tolist() if has_bias else None
        for h in range(heads):
            acc = gemm_numpy(g[f"{name}_a"][h].tolist(), g[f"{name}_b"][h].tolist(), bias, bool(tr), bool(uns))
            out = gemm_writeback(acc, src, dst, bits)
            np.testing.assert_array_equal(np.array(out), g[f"{name}_expected"][h], err_msg=str(name))


def test_gemm_golden_units(cuda):
    from heatvit_b200.gemm import gemm_numpy, gemm_writeback
    g = load_golden("golden_units.npz")
    i = 0
    while f"gemm{i}_a" in g:
        src, dst = (int(v) for v in g[f"gemm{i}_exps"])
        acc = gemm_numpy(g[f"gemm{i}_a"], g[f"gemm{i}_w"], g[f"gemm{i}_bias"].tolist(), False)
        np.testing.assert_array_equal(np.array(gemm_writeback(acc, src, dst, 8)), g[f"gemm{i}_out8"])
        np.testing.assert_array_equal(np.array(gemm_writeback(acc, src, -14, 32)), g[f"gemm{i}_out32"])
        i += 1


@pytest.mark.parametrize("m,k,n,tr,uns", [(4099, 192, 576, False, False), (2053, 768, 192, False, False),
                                          (1000, 192, 768, True, False), (517, 197, 64, False, True),
                                          (1, 1, 1, False, False), (130, 96, 70, True, True)])
def test_gemm_random_vs_oracle(cuda, oracle, m, k, n, tr, uns):
    from heatvit_b200.gemm import _gemm_acc
    rng = np.random.default_rng(m * 7 + k)
    a = rng.integers(0 if uns else -128, 256 if uns else 128, (m, k))
    b = rng.integers(-128, 128, (n, k) if tr else (k, n))
    bias = rng.integers(-(1 << 31), (1 << 31) - 1, n)
    got = _gemm_acc(a, b, bias, tr, uns)
    np.testing.assert_array_equal(got, oracle.gemm(a, b, bias, tr, uns))


def test_gemm_errors(cuda):
    from heatvit_b200.gemm import gemm_numpy, gemm_writeback
    with pytest.raises(TypeError):
        gemm_numpy([[1.0]], [[1]], None, False)
    with pytest.raises(ValueError):
        gemm_numpy([[128]], [[1]], None, False)
    with pytest.raises(ValueError):
        gemm_numpy([[1, 2]], [[1]], None, False)
    with pytest.raises(ValueError):
        gemm_writeback([[1]], -14, -7, 16)


# ---- element-wise units -------------------------------------------------------------

def test_gelu_plan_exhaustive_q8_16(cuda, oracle):
    """Every Q8.16 input in [-2^23, 2^23): ShiftGELU (incl. its exact integer
    division for every e the argument can produce) and PLAN."""
    from heatvit_b200.nonlinear import gelu_array, plan_array
    x = np.arange(-(1 << 23), 1 << 23, dtype=np.int64)
    np.testing.assert_array_equal(gelu_array(x), oracle.gelu_array(x))
    np.testing.assert_array_equal(plan_array(x), oracle.plan_array(x))


def test_gelu_kat_and_wide_inputs(cuda, oracle):
    from heatvit_b200.nonlinear import gelu, gelu_array, plan_array
    g = load_golden("kat_nonlinear.npz")
    np.testing.assert_array_equal(gelu_array(g["x"]), g["gelu"])
    np.testing.assert_array_equal(plan_array(g["x"]), g["plan"])
    rng = np.random.default_rng(3)
    x = rng.integers(-(1 << 31), (1 << 31) - 1, 100000)
    np.testing.assert_array_equal(gelu_array(x), oracle.gelu_array(x))
    assert gelu(32768) == 22817 and gelu(-163965) == -2404


def test_gelu_requant_chain(cuda, oracle):
    from heatvit_b200.nonlinear import gelu_requant_array
    g = load_golden("golden_units.npz")
    np.testing.assert_array_equal(gelu_requant_array(g["chain_acc"], -14, -7), g["chain_y"])
    rng = np.random.default_rng(11)
    acc = rng.integers(-(1 << 24), 1 << 24, 200000)
    for src, dst in ((-30, -9), (-16, -20), (-40, -8), (-14, -7)):
        np.testing.assert_array_equal(gelu_requant_array(acc, src, dst), oracle.gelu_chain_array(acc, src, dst))


@pytest.mark.parametrize("src,sh_out", [(-17, -7), (-17, -1), (-17, 0), (-17, 1), (-17, 2), (-17, 6), (-17, 8),
                                        (-17, 9), (-17, 12), (-17, 30), (-16, 0), (-16, 7)])
def test_gelu_requant_fma_form_exhaustive(cuda, oracle, src, sh_out):
    """The GELU chain's FMA-pipe form on every Q8.16 input it can see: with
    src = -17 (input shift 1) the values [-2^24, 2^24) cover every q16 with both
    rounding directions; src = -16 (no input shift) covers q16 = v directly.
    Both ends of the range also exercise the exact fallback."""
    from heatvit_b200.nonlinear import gelu_requant_array
    span = 1 << (24 if src == -17 else 23)
    v = np.arange(-span, span, dtype=np.int32)
    dst = sh_out - 16
    np.testing.assert_array_equal(gelu_requant_array(v, src, dst), oracle.gelu_chain_array(v, src, dst))


def test_align_add(cuda, oracle):
    from heatvit_b200.transformer import align_add_array
    rng = np.random.default_rng(5)
    a = rng.integers(-128, 128, 50000)
    b = rng.integers(-128, 128, 50000)
    for ea, eb, eo in ((-7, -7, -7), (-12, -9, -8), (-20, -8, -8), (-8, -20, -19), (-9, -9, -14)):
        np.testing.assert_array_equal(align_add_array(a, ea, b, eb, eo), oracle.align_add_array(a, ea, b, eb, eo))


def test_writeback_kat(cuda):
    from heatvit_b200.gemm import writeback_array
    g = load_golden("kat_requant.npz")
    for suite in ("fixed", "requant"):
        v, s, d, e = (g[f"{suite}_{k}"] for k in ("value", "src", "dst", "expected"))
        got = np.array([writeback_array(np.array([int(v[i])]), int(s[i]), int(d[i]), 8)[0] for i in range(v.size)])
        np.testing.assert_array_equal(got, e)


# ---- softmax ------------------------------------------------------------------------

def test_softmax_kat(cuda):
    from heatvit_b200.nonlinear import softmax_rows
    g = load_golden("kat_softmax.npz")
    np.testing.assert_array_equal(softmax_rows(g["x"], g["lengths"], 0), g["attention"])
    np.testing.assert_array_equal(softmax_rows(g["x"], g["lengths"], 1), g["selector"])


def test_softmax_golden_units_and_api(cuda):
    from heatvit_b200.nonlinear import softmax_attention, softmax_rows, softmax_selector
    g = load_golden("golden_units.npz")
    np.testing.assert_array_equal(softmax_rows(g["sm_x"], g["sm_len"], 0), g["sm_attention"])
    np.testing.assert_array_equal(softmax_rows(g["sm_x"], g["sm_len"], 1), g["sm_selector"])
    assert softmax_attention([0]) == [255]
    assert softmax_selector([12345, 12345]) == [32768, 32768]
    with pytest.raises(ValueError):
        softmax_selector([])
    with pytest.raises(TypeError):
        softmax_selector([0.5, 0.0])


def test_softmax_config2_rows(cuda, oracle):
    """Config-2 style: Gaussian scores sigma 2^12 at score_scale -17 -> Q16, rows of 197."""
    from heatvit_b200.nonlinear import softmax_rows
    rng = np.random.default_rng(2)
    s = np.clip(np.rint(rng.normal(0, 4096, (3 * 197 * 16, 197))), -(1 << 31), (1 << 31) - 1).astype(np.int64)
    q16 = oracle.requant_array(s, 0, 4, 24).reshape(-1)
    lens = np.full(s.shape[0], 197)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    np.testing.assert_array_equal(softmax_rows(q16, lens, 0), oracle.softmax_rows(q16, off, 0))
    np.testing.assert_array_equal(softmax_rows(q16, lens, 1), oracle.softmax_rows(q16, off, 1))


# ---- LayerNorm ----------------------------------------------------------------------

def test_layernorm_kat(cuda):
    from heatvit_b200.nonlinear import layernorm
    g = load_golden("kat_layernorm.npz")
    for i in range(g["x"].shape[0]):
        out, neg = layernorm(g["x"][i].tolist(), g["gamma"][i].tolist(), g["beta"][i].tolist(),
                             *[int(v) for v in g["scales"][i]])
        assert out == g["expected"][i].tolist()
        assert neg == bool(g["warn"][i])


def test_layernorm_units_and_bulk(cuda, oracle):
    from heatvit_b200.nonlinear import layernorm_rows
    g = load_golden("golden_units.npz")
    for i in range(g["ln_inputs"].shape[0]):
        x, gm, bt = g["ln_inputs"][i]
        out, neg = layernorm_rows(x[None, :], gm, bt, *[int(v) for v in g["ln_scales"][i]])
        np.testing.assert_array_equal(out[0], g["ln_expected"][i])
        assert bool(neg[0]) == bool(g["ln_warn"][i])
    rng = np.random.default_rng(9)
    x = rng.integers(-128, 128, (256 * 197 // 8, 192))
    x[::17] = x[::17, :1]  # constant rows
    gm, bt = rng.integers(-128, 128, 192), rng.integers(-128, 128, 192)
    for sc in ((-9, -14, -15, -13), (-20, -8, -20, -12), (-32, 31, -32, 5), (0, -32, 31, -10)):
        out, neg = layernorm_rows(x, gm, bt, *sc)
        ref, rneg = oracle.layernorm(x, gm, bt, *sc)
        np.testing.assert_array_equal(out, ref)
        np.testing.assert_array_equal(neg, rneg)


def test_layernorm_errors(cuda):
    from heatvit_b200.nonlinear import layernorm
    g64, b0 = [64] * 192, [0] * 192
    with pytest.raises(ValueError):
        layernorm([0] * 192, g64, b0, 1, -6, -7, -7)
    with pytest.raises(ValueError):
        layernorm([0] * 191, g64, b0, -7, -6, -7, -7)
    with pytest.raises(ValueError):
        layernorm([128] * 192, g64, b0, -7, -6, -7, -7)
    with pytest.raises(TypeError):
        layernorm([0.5] * 192, g64, b0, -7, -6, -7, -7)
