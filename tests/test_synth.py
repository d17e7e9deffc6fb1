"""Parameter generators: the restated reference model and the benchmark model."""

import hashlib

import numpy as np

from conftest import load_golden


def _digest(params):
    from heatvit_b200.params import PackedParams
    h = hashlib.sha256()
    for a in PackedParams(params)._keep:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def test_reference_seeded_params_match_golden():
    from heatvit_b200 import synth
    g = load_golden("golden_seeded.npz")
    calib = [tuple(int(v) for v in row) for row in g["seeded_calibration"]]
    assert _digest(synth.reference_seeded_params(calib)) == str(g["seeded_params_sha256"])


def test_benchmark_params_are_deterministic():
    from heatvit_b200 import synth
    for name, tag in (("golden_baseline.npz", "pruned"), ("golden_unpruned.npz", "unpruned")):
        g = load_golden(name)
        p = synth.config_params(int(g[f"{tag}_seed"]), pruned=bool(g[f"{tag}_pruned"]))
        assert _digest(p) == str(g[f"{tag}_params_sha256"])


def test_config3_params_match_golden():
    from heatvit_b200 import synth
    g = load_golden("golden_config3.npz")
    p = synth.config3_params(int(g["config3_seed"]))
    assert _digest(p) == str(g["config3_params_sha256"])
    sel = p.selectors[0]
    # only the first selector's logits leave [-20, -8]: a zero keep score needs
    # (drop - keep) * 2^(logits_exp + 16) >= 16 * 45426 with |drop - keep| <= 255
    assert sel.logits_out_scale_exp == synth.ZERO_DEN_LOGITS_EXP
    assert 255 << (sel.logits_out_scale_exp + 16) >= 16 * 45426
    assert 255 << (-8 + 16) < 16 * 45426


def test_benchmark_exponents_in_range():
    from heatvit_b200 import synth
    p = synth.config_params(20260815)
    exps = []
    for b in p.blocks:
        for obj in (b.mhsa, b.ffn):
            for k, v in vars(obj).items():
                if k.endswith("_exp") and k not in ("score_scale_exp", "prob_scale_exp"):
                    exps.append(v)
        assert b.mhsa.score_scale_exp == 2 * b.mhsa.qkv_out_scale_exp - 3
    assert min(exps) >= -20 and max(exps) <= -8


def test_images_depend_only_on_seed_and_index():
    from heatvit_b200 import synth
    a = synth.baseline_images(7, 3)
    b = synth.baseline_images(7, 2, first=1)
    np.testing.assert_array_equal(a[1:], b)
    assert a.dtype == np.int8 and a.shape == (3, 150528)
