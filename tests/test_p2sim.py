"""Batched pruned P2-simulator inference (heatvit_b200.p2sim) against the
reference's P2 simulator (tools/p2/p2_sim.py forward_image, pruned and
unpruned) on the config-3 model and seeded float images with rounding ties and
out-of-range values, frozen by tests/golden/make_golden.py (golden_p2sim.npz).

CPU: the QuantDeiT -> parameter mapping, and the oracle on the quantised images
(which pins the oracle to the P2 simulator).  GPU: the quantisation kernel and
the batched engine path."""

import hashlib
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import load_golden


def _digest(params):
    from heatvit_b200.params import PackedParams
    h = hashlib.sha256()
    for a in PackedParams(params)._keep:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _quant_deit(params):
    """A QuantDeiT-shaped object (p2_sim.py:291-304) holding a model's tensors."""
    from heatvit_b200 import memimage
    from heatvit_b200.p2sim import _BLOCK_FIELDS, _SEL_FIELDS
    t = memimage._tensors(params)
    table = memimage.scale_table(params)
    return SimpleNamespace(
        scales=SimpleNamespace(weights=table["weights"], activations=table["activations"]),
        blocks=[SimpleNamespace(**{f: t[f"b{n}_{f}"] for f in _BLOCK_FIELDS}) for n in range(1, 13)],
        selectors=[SimpleNamespace(**{f: t[f"s{s}_{f}"] for f in _SEL_FIELDS}) for s in range(1, 4)],
        **{k: t[k] for k in ("patch_w", "patch_b", "cls", "pos", "final_gamma", "final_beta", "head_w", "head_b")})


def _setup():
    from heatvit_b200 import synth
    g = load_golden("golden_p2sim.npz")
    params = synth.config3_params(int(g["p2_seed"]))
    imgs = synth.p2_float_images(int(g["p2_seed"]), int(g["p2_count"]), params.patch.image_scale_exp)
    return g, params, imgs


def _quantize_np(imgs, e):
    """p2_sim.py:536-541 in numpy: round half to even, clamp, CHW -> HWC."""
    q = np.clip(np.rint(imgs / np.float32(2.0 ** e)), -128, 127).astype(np.int8)
    return q.transpose(0, 2, 3, 1).reshape(q.shape[0], -1)


def test_params_from_quant_deit():
    from heatvit_b200 import p2sim
    from heatvit_b200.params import with_selectors
    _, params, _ = _setup()
    model = _quant_deit(params)
    assert _digest(p2sim.params_from_quant_deit(model)) == _digest(params)
    assert _digest(p2sim.params_from_quant_deit(model, prune=False)) == _digest(with_selectors(params, (), ()))
    model.selectors = model.selectors[:2]
    with pytest.raises(ValueError):
        p2sim.params_from_quant_deit(model)


def test_oracle_matches_p2_simulator(oracle):
    from heatvit_b200.params import with_selectors
    g, params, imgs = _setup()
    q = _quantize_np(imgs, params.patch.image_scale_exp)
    for tag, p in (("pruned", params), ("unpruned", with_selectors(params, (), ()))):
        for i in range(q.shape[0]):
            r = oracle.infer(p, q[i])
            np.testing.assert_array_equal(r["logits"], g[f"p2_{tag}_logits"][i])
            assert [int(v) for v in r["counts"]] == [int(v) for v in g[f"p2_{tag}_counts"][i]]


@pytest.mark.gpu
def test_quantize_kernel_edges(cuda):
    from heatvit_b200 import p2sim
    torch = cuda
    rng = np.random.default_rng(3)
    for e in (-10, -5, 0, 3):
        x = rng.normal(0, 60, (2, 3, 224, 224)).astype(np.float32) * np.float32(2.0 ** e)
        step = np.float32(2.0 ** e)
        special = np.array([0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 126.5, 127.5, -127.5, -128.5, -129.0, 300.0,
                            -1e30, 1e30, np.inf, -np.inf, -0.0, 1e-40], np.float32)
        flat = x.reshape(-1)
        flat[:12] = special[:12] * step
        flat[12:special.size] = special[12:]
        got = p2sim.quantize_images(torch.from_numpy(x).cuda(), e).cpu().numpy()
        np.testing.assert_array_equal(got, _quantize_np(x, e))
    x = np.full((1, 3, 224, 224), np.nan, np.float32)
    assert not p2sim.quantize_images(torch.from_numpy(x).cuda(), -7).cpu().numpy().any()


@pytest.mark.gpu
def test_p2sim_matches_reference_simulator(cuda):
    from heatvit_b200 import p2sim
    torch = cuda
    g, params, imgs = _setup()
    model = _quant_deit(params)
    for tag, prune in (("pruned", True), ("unpruned", False)):
        logits, counts, e = p2sim.forward_batch(model, torch.from_numpy(imgs).cuda(), prune=prune)
        assert e == -14
        np.testing.assert_array_equal(logits.cpu().numpy(), g[f"p2_{tag}_logits"])
        np.testing.assert_array_equal(counts.cpu().numpy(), g[f"p2_{tag}_counts"])
        lg, tc, _ = p2sim.forward_image(model, torch.from_numpy(imgs[2]), prune=prune)
        np.testing.assert_array_equal(lg.cpu().numpy(), g[f"p2_{tag}_logits"][2])
        assert tc == [int(v) for v in g[f"p2_{tag}_counts"][2]]


@pytest.mark.gpu
def test_eval_top1(cuda):
    from heatvit_b200 import p2sim
    torch = cuda
    g, params, imgs = _setup()
    model = _quant_deit(params)
    pred = g["p2_pruned_logits"].argmax(1)
    labels = pred.copy()
    labels[[1, 4]] = (labels[[1, 4]] + 1) % 1000  # two wrong labels
    loader = [(torch.from_numpy(imgs[:4]), torch.from_numpy(labels[:4])),
              (torch.from_numpy(imgs[4:]), torch.from_numpy(labels[4:]))]
    acc, _, correct, total = p2sim.eval_top1(model, loader)
    assert (correct, total) == (4, 6) and abs(acc - 400.0 / 6) < 1e-9
