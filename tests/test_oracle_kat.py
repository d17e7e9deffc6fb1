"""The CPU oracle against the reference's committed known-answer vectors
(sim/vectors, decoded into tests/golden/kat_*.npz by make_golden.py)."""

import numpy as np

from conftest import load_golden


def test_requant_kat(oracle):
    g = load_golden("kat_requant.npz")
    for suite in ("fixed", "requant"):
        got = oracle.requant_array(g[f"{suite}_value"], g[f"{suite}_src"], g[f"{suite}_dst"], 8)
        np.testing.assert_array_equal(got, g[f"{suite}_expected"])


def test_isqrt_and_division_kat(oracle):
    g = load_golden("kat_divsqrt.npz")
    for rad, root, rem in zip(g["isqrt_rad"], g["isqrt_root"], g["isqrt_rem"]):
        assert oracle.isqrt(int(rad)) == (int(root), int(rem))
    # round_div follows divmod: check the quotient/remainder pairs that fit int64
    for n, d, q, r in zip(g["udiv_num"], g["udiv_den"], g["udiv_q"], g["udiv_r"]):
        n, d, q, r = int(n), int(d), int(q), int(r)
        assert (q, r) == divmod(n, d)
        if n < (1 << 63) and d < (1 << 63):
            want = q + (1 if 2 * r >= d else 0)
            assert oracle.round_div(n, d) == want


def test_gelu_plan_kat(oracle):
    g = load_golden("kat_nonlinear.npz")
    np.testing.assert_array_equal(oracle.gelu_array(g["x"]), g["gelu"])
    np.testing.assert_array_equal(oracle.plan_array(g["x"]), g["plan"])


def test_gelu_anchor_values(oracle):
    # verification/tests/test_nonlinear.py:24-37
    for x, y in ((0, 0), (1, 1), (-1, 0), (32768, 22817), (-32768, -9802), (163965, 161556),
                 (-163965, -2404), (8388607, 8323583), (-8388608, 0)):
        assert oracle.gelu(x) == y


def test_softmax_kat(oracle):
    g = load_golden("kat_softmax.npz")
    off = np.concatenate([[0], np.cumsum(g["lengths"])]).astype(np.int32)
    np.testing.assert_array_equal(oracle.softmax_rows(g["x"], off, 0), g["attention"])
    np.testing.assert_array_equal(oracle.softmax_rows(g["x"], off, 1), g["selector"])


def test_layernorm_kat(oracle):
    g = load_golden("kat_layernorm.npz")
    for i in range(g["x"].shape[0]):
        sc = [int(v) for v in g["scales"][i]]
        out, neg = oracle.layernorm(g["x"][i], g["gamma"][i], g["beta"][i], *sc)
        np.testing.assert_array_equal(out, g["expected"][i])
        assert bool(neg[0]) == bool(g["warn"][i])


def test_gemm_kat(oracle):
    g = load_golden("kat_gemm.npz")
    for name in g["names"]:
        m, n, k, heads, tr, uns, bits, has_bias, src, dst = (int(v) for v in g[f"{name}_meta"])
        bias = g[f"{name}_bias"] if has_bias else None
        for h in range(heads):
            acc = oracle.gemm(g[f"{name}_a"][h], g[f"{name}_b"][h], bias, tr, uns)
            np.testing.assert_array_equal(oracle.writeback(acc, src, dst, bits), g[f"{name}_expected"][h])
    for case in g["mac_bank"]:
        a, b = case[0:8], case[8:16]
        rm, cm, uns, k = (int(v) for v in case[16:20])
        acc = case[20:].reshape(8, 8)
        A = np.repeat(a[:, None], k, axis=1)
        if not uns:
            A = np.where(A >= 128, A - 256, A)
        B = np.repeat(b[None, :], k, axis=0)
        got = oracle.gemm(A, B, None, False, bool(uns))
        mask = np.outer([(rm >> r) & 1 for r in range(8)], [(cm >> c) & 1 for c in range(8)])
        np.testing.assert_array_equal(got * mask, acc)


def test_selector_finalize_kat(oracle):
    g = load_golden("kat_selector.npz")
    for name in g["names"]:
        n, pkg, nn, npkg, warn = (int(v) for v in g[f"{name}_meta"])
        tok = g[f"{name}_tokens"]
        scores = g[f"{name}_scores"]
        normals = tok[1:n - 1] if pkg else tok[1:]
        res = oracle.finalize_tokens(tok[0], normals, tok[n - 1] if pkg else None, scores)
        np.testing.assert_array_equal(res["tokens"], g[f"{name}_output"])
        assert res["package_present"] == bool(npkg)
        assert res["warnings"] == warn
    for s, w, want, wb in zip(g["fuse_scores"], g["fuse_weights"], g["fuse_expected"], g["fuse_warn"]):
        fused, warn = oracle.fuse_head_scores(np.array(s)[:, None], np.array(w)[None, :])
        assert int(fused[0]) == int(want)
        assert bool(warn) == bool(wb)
