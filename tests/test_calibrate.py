"""Selector calibration of the reference's seeded model (weights.py:143-251).

CPU: ``synth.calibrate_reference_selectors`` with the oracle as the backend must
reproduce the reference's own calibration outcome, frozen in golden_seeded.npz
(stage attempts 0 / 0 / 12, medians -779 / -420 / 514).
GPU: ``heatvit_b200.calibrate.build_params`` runs the same search with every
model computation on the device and must give the same outcome, token counts and
parameters."""

import hashlib

import numpy as np
import pytest

from conftest import load_golden


def _h2_oracle(oracle, p, tokens):
    """weights.py:143-155 from the oracle's GEMM and GELU-chain primitives."""
    cand = np.asarray(tokens, np.int8)[1:]
    c = cand.shape[0]
    out = np.empty((3, c, 16), np.int64)
    for h in range(3):
        loc = oracle.gelu_chain_array(oracle.gemm(cand[:, 64 * h:64 * (h + 1)], p.local.w[h], p.local.b[h], False),
                                      p.in_scale_exp + p.local_w_scale_exp, p.local_out_scale_exp)
        glob = np.array([max(-128, min(127, oracle.round_div(int(v), c))) for v in loc.astype(np.int64).sum(0)],
                        np.int8)
        lg = np.concatenate([loc, np.tile(glob, (c, 1))], 1)
        h1 = oracle.gelu_chain_array(oracle.gemm(lg, p.score.w1[h], p.score.b1[h], False),
                                     p.concat_out_scale_exp + p.score_w1_scale_exp, p.h1_out_scale_exp)
        out[h] = oracle.gelu_chain_array(oracle.gemm(h1, p.score.w2[h], p.score.b2[h], False),
                                         p.h1_out_scale_exp + p.score_w2_scale_exp, p.h2_out_scale_exp)
    return out


def _run_to_selector(oracle, params, image, stage):
    r = oracle.infer(params, image)
    ck, rows = r["checkpoints"], r["checkpoint_rows"]
    slot = 3 * stage                      # block 3s feeds selector s
    pkg = bool(r["summary"][stage - 2]["package_present"]) if stage > 1 else False
    return ck[slot][:rows[slot]], pkg


def _expected():
    g = load_golden("golden_seeded.npz")
    return [tuple(int(v) for v in row) for row in g["seeded_calibration"]], g


def test_calibration_with_oracle_backend(oracle):
    from heatvit_b200 import synth
    want, _ = _expected()

    def sel(tokens, pkg, params):
        r = oracle.token_selector(tokens, pkg, params)
        return dict(kept_normal=r["kept_normal"], pruned_normal=r["pruned_normal"])

    got = synth.calibrate_reference_selectors(
        synth.reference_seeded_image(), lambda params, image, stage: _run_to_selector(oracle, params, image, stage),
        lambda tokens, params: _h2_oracle(oracle, params, tokens), sel)
    assert got == want


@pytest.mark.gpu
def test_calibration_on_gpu(cuda, oracle):
    from heatvit_b200 import calibrate, synth
    from heatvit_b200.params import PackedParams
    want, g = _expected()
    image = synth.reference_seeded_image()
    params, summary, counts = calibrate.build_params(image)
    assert [(s["attempt"], s["median_logit_diff"]) for s in summary] == want
    assert counts == [197, 100, 55, 28]
    h = hashlib.sha256()
    for a in PackedParams(params)._keep:
        h.update(np.ascontiguousarray(a).tobytes())
    assert h.hexdigest() == str(g["seeded_params_sha256"])
    # the device features against the oracle's, at the first selector's input
    base = synth.reference_seeded_base()
    x, _ = _run_to_selector(oracle, params, image, 1)
    np.testing.assert_array_equal(calibrate.selector_h2(x, base["bases"][0]), _h2_oracle(oracle, base["bases"][0], x))


# What synth.calibrate_keep_bias returns over the current seeded images (the oracle
# as backend, about a minute on 8 host threads); the committed BASELINE_KEEP_BIAS
# came from the first image generator.
KEEP_BIAS_SEARCH = (-23305, -895, 10084)


@pytest.mark.slow
def test_keep_bias_calibration_with_oracle_backend(oracle):
    """The benchmark generator's per-stage keep-bias search (bisection on the mean
    selector output counts of 64 images) with the oracle as the backend."""
    from heatvit_b200 import synth
    got = synth.calibrate_keep_bias(synth.SEED, lambda p, imgs: oracle.infer_batch(p, imgs, threads=0)["counts"])
    assert got == KEEP_BIAS_SEARCH


@pytest.mark.gpu
def test_keep_bias_calibration_on_gpu(cuda):
    """The same search with the CUDA engine as the backend (78 model builds and
    inferences, a few seconds)."""
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine

    def counts(params, imgs):
        return Engine(params).infer(torch.from_numpy(imgs).cuda())["token_counts"].cpu().numpy()

    assert synth.calibrate_keep_bias(synth.SEED, counts) == KEEP_BIAS_SEARCH
