"""The reference's weight memory image and scale table (heatvit_b200.memimage)
against the reference's own serializer, memory map and ScaleTable, frozen by
tests/golden/make_golden.py (golden_memimage.npz)."""

import hashlib

import numpy as np

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
