"""The end-to-end vector set in the RTL's checkpoint order (heatvit_b200.e2evectors)
against the reference generator's own output for its seeded model and image,
frozen by tests/golden/make_golden.py (golden_e2evectors.npz).

CPU: the layout and the files written from the oracle's checkpoints.
GPU: the files written from the CUDA engine's checkpoints (one image through
``HeatViTModel.infer``), and the batched dump of a pruned batch against the
oracle image by image."""

import hashlib
import json

import numpy as np
import pytest

from conftest import load_golden

SEEDED_COUNTS = [197, 100, 55, 28]


def _seeded():
    from heatvit_b200 import synth
    g = load_golden("golden_seeded.npz")
    calib = [tuple(int(v) for v in row) for row in g["seeded_calibration"]]
    return synth.reference_seeded_params(calib), synth.reference_seeded_image(), calib


def _check_files(files):
    g = load_golden("golden_e2evectors.npz")
    for name, digest in zip(g["e2e_files"], g["e2e_sha256"]):
        assert hashlib.sha256(files[str(name)]).hexdigest() == str(digest), name
    assert files["manifest.json"].decode() == str(g["e2e_manifest"])
    assert files["e2e_tb_config.sv"].decode() == str(g["e2e_tb_config_sv"])
    assert set(files) == {str(n) for n in g["e2e_files"]} | {"manifest.json", "e2e_tb_config.sv"}


def test_layout_matches_reference_manifest():
    from heatvit_b200 import e2evectors as E
    g = load_golden("golden_e2evectors.npz")
    assert bool(g["e2e_tb_config_matches_committed"])
    man = json.loads(str(g["e2e_manifest"]))
    assert man["token_counts"] == SEEDED_COUNTS
    want = [{k: v for k, v in c.items() if k != "sha256"} for c in man["checkpoints"]]
    assert E.checkpoint_layout(SEEDED_COUNTS) == want
    assert [c["name"] for c in want] == list(E.CHECKPOINT_NAMES)
    assert E.scratch_layout()["bytes"] == man["regions"]["scratch"]["bytes"]
    assert man["descriptor_rom_sha256"] == E.DESCRIPTOR_ROM_SHA256
    with pytest.raises(ValueError):
        E.checkpoint_layout([197, 100, 55])


def test_mem_text_round_trip():
    from heatvit_b200 import memimage
    rng = np.random.default_rng(5)
    for n in (0, 1, 7, 8, 9, 4000, 37825):
        raw = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        text = memimage.mem_lines(raw)
        assert text.count("\n") == (n + 7) // 8
        want = "".join(f"{int.from_bytes((raw + bytes(8))[i:i + 8], 'little'):016x}\n" for i in range(0, n, 8))
        assert text == want
        assert memimage.parse_mem(text) == raw + bytes((-n) % 8)
        assert memimage.parse_mem(text.replace("\n", "\r\n")) == raw + bytes((-n) % 8)


def test_vector_set_from_oracle(oracle):
    from heatvit_b200 import e2evectors as E
    params, image, calib = _seeded()
    r = oracle.infer(params, image)
    counts = [int(v) for v in r["counts"]]
    assert counts == SEEDED_COUNTS
    ck = E.checkpoint_images_from_slots(r["checkpoints"], r["checkpoint_rows"], r["logits"], counts)
    files = E.vector_files(image, params, ck, counts, E.selector_entries(calib, r["summary"]))
    _check_files(files)


@pytest.mark.gpu
def test_vector_set_from_gpu_model(cuda, tmp_path):
    from heatvit_b200 import e2evectors as E
    from heatvit_b200.model import HeatViTModel
    params, image, calib = _seeded()
    res = HeatViTModel().infer(image.tolist(), params)
    counts = [197] + [s["output_tokens"] for s in res.selector_summary]
    assert counts == SEEDED_COUNTS
    files = E.vector_files(image, params, E.checkpoint_images(res.checkpoints, counts), counts,
                           E.selector_entries(calib, res.selector_summary))
    _check_files(files)
    E.write_vector_files(tmp_path, files)
    assert (tmp_path / "checkpoints" / "selector_03.mem").read_bytes() == files["checkpoints/selector_03.mem"]


@pytest.mark.gpu
def test_batched_checkpoint_dump_matches_oracle(cuda, oracle):
    """A pruned batch (the config-3 model) through one engine launch: each
    image's 18 checkpoint images equal the oracle's."""
    from heatvit_b200 import e2evectors as E
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    params = synth.config3_params(synth.SEED)
    imgs = synth.baseline_images(synth.SEED, 24)
    out = Engine(params).infer(cuda.from_numpy(imgs).cuda(), checkpoints=True)
    dumps = E.checkpoint_images_batch(out)
    assert len(dumps) == imgs.shape[0]
    for i, d in enumerate(dumps):
        r = oracle.infer(params, imgs[i])
        counts, ck = d["token_counts"], d["checkpoints"]
        assert counts == [int(v) for v in r["counts"]], i
        assert d["selector_summary"] == [{k: s[k] for k in d["selector_summary"][0]} for s in r["summary"]], i
        want = E.checkpoint_images_from_slots(r["checkpoints"], r["checkpoint_rows"], r["logits"], counts)
        for e in E.checkpoint_layout(counts):
            assert ck[e["name"]] == want[e["name"]], (i, e["name"])
    # an uncalibrated model's manifest: selector entries without the calibration keys
    files = E.vector_files(imgs[0], params, dumps[0]["checkpoints"], dumps[0]["token_counts"],
                           E.selector_entries(None, dumps[0]["selector_summary"]))
    man = json.loads(files["manifest.json"])
    assert [e["stage"] for e in man["selectors"]] == [1, 2, 3] and "attempt" not in man["selectors"][0]
    assert "SELECTOR_PACKAGE" in files["e2e_tb_config.sv"].decode()
