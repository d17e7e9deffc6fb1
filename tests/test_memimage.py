"""The reference's weight memory image and scale table (heatvit_b200.memimage)
against the reference's own serializer, memory map and ScaleTable, frozen by
tests/golden/make_golden.py (golden_memimage.npz)."""

import hashlib

import numpy as np
import pytest

from conftest import load_golden


def _digest(params):
    from heatvit_b200.params import PackedParams
    h = hashlib.sha256()
    for a in PackedParams(params)._keep:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _models():
    from heatvit_b200 import synth
    g = load_golden("golden_seeded.npz")
    calib = [tuple(int(v) for v in row) for row in g["seeded_calibration"]]
    return {"seeded": synth.reference_seeded_params(calib), "config3": synth.config3_params(synth.SEED)}


def test_weight_image_matches_reference_serializer():
    from heatvit_b200 import memimage
    g = load_golden("golden_memimage.npz")
    for tag, params in _models().items():
        raw = memimage.write_weights(params)
        assert len(raw) == int(g[f"memimage_{tag}_bytes"]) == memimage.weight_bytes()
        assert hashlib.sha256(raw).hexdigest() == str(g[f"memimage_{tag}_sha256"]), tag
        text = memimage.mem_lines(raw).encode()
        assert hashlib.sha256(text).hexdigest() == str(g[f"memimage_{tag}_mem_sha256"]), tag


def test_scale_table_matches_reference_format():
    from heatvit_b200 import memimage, synth
    g = load_golden("golden_memimage.npz")
    text = memimage.scale_table_json(memimage.scale_table(synth.config3_params(synth.SEED)))
    assert text == str(g["memimage_config3_scales_json"])


def test_weight_image_round_trip():
    from heatvit_b200 import memimage
    for tag, params in _models().items():
        raw = memimage.write_weights(params)
        table = memimage.load_scale_table(memimage.scale_table_json(memimage.scale_table(params)))
        back = memimage.read_weights(memimage.parse_mem(memimage.mem_lines(raw)), table)
        assert _digest(back) == _digest(params), tag
        assert memimage.write_weights(back) == raw


def test_layout_is_eight_byte_aligned_and_ordered():
    from heatvit_b200 import memimage
    lay = memimage.weight_layout()
    assert lay[0][:2] == ("patch_w", 0) and lay[-1][0] == "head_b"
    end = 0
    for name, off, shape, esz in lay:
        assert off % 8 == 0 and off >= end, name
        end = off + int(np.prod(shape)) * esz
    assert memimage.weight_bytes() == (end + 7) & ~7


@pytest.mark.gpu
def test_engine_from_reference_memory_image_matches_oracle(cuda, oracle):
    """The engine loaded from the reference's weight memory image (.mem text,
    tools/generate_e2e_vectors.py:87-155) and its ScaleTable JSON
    (tools/p2/scale_table.py:82-98) runs a config-3 batch bit-exactly like the
    oracle on the original parameters.  The image text is the reference
    serializer's, byte for byte (its SHA-256 is the golden one)."""
    import torch
    from heatvit_b200 import memimage, synth
    from heatvit_b200.engine import Engine
    g = load_golden("golden_memimage.npz")
    params = synth.config3_params(synth.SEED)
    text = memimage.mem_lines(memimage.write_weights(params))
    assert hashlib.sha256(text.encode()).hexdigest() == str(g["memimage_config3_mem_sha256"])
    table = memimage.load_scale_table(memimage.scale_table_json(memimage.scale_table(params)))
    loaded = memimage.read_weights(memimage.parse_mem(text), table)
    imgs = synth.baseline_images(synth.SEED, 48)
    got = Engine(loaded).infer(torch.from_numpy(imgs).cuda())
    ref = oracle.infer_batch(params, imgs)
    np.testing.assert_array_equal(got["logits"].cpu().numpy(), ref["logits"])
    np.testing.assert_array_equal(got["token_counts"].cpu().numpy(), ref["counts"])
    np.testing.assert_array_equal(got["warnings"].cpu().numpy(), ref["warnings"])
