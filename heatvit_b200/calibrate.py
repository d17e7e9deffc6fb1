"""The reference's seeded-model selector calibration, on the GPU.

Restates verification/heatvit_ref/weights.py:143-251 with the same names and
results, but every model computation goes through the CUDA library:

* ``selector_h2`` (weights.py:143-155): the score layer-2 features of a
  selector's candidates, from the selector kernel (``hv_selector_h2``);
* ``calibrate_selector`` (weights.py:158-204): for attempt a = 0, 1, ... the
  last score layer is re-seeded with ``random.Random(20260815 + stage*1000 + a)``,
  the keep bias is set to the negative median of the bias-free keep - drop logit
  differences (h2 · (w3[:, :, 1] - w3[:, :, 0]) over heads and candidates), and
  the first attempt whose selector output keeps at least one and prunes at least
  two normal tokens is accepted;
* ``build_params`` (weights.py:207-251): the seeded parameter stream, with the
  stage inputs produced by the CUDA patch embedding and fused blocks.

The arithmetic of the attempt search (the integer dot products and the median)
runs on the host, as in the reference; each trial selector run, the features
and the block pipeline run on the device.
"""

import ctypes as C

import numpy as np

from . import synth
from ._lib import check, lib
from .engine import _stream, _torch, selector_model_for
from .params import HeatViTParams
from .selector import token_selector_batch
from .transformer import patch_embedding, transformer_block_batch

ATTEMPTS = synth.SELECTOR_ATTEMPTS
SEED = synth.SEED


def selector_h2(tokens, params):
    """weights.py:143-155: per head second hidden layer [3][C][16] of the
    candidates tokens[1:] (int8 values as a numpy array)."""
    torch = _torch()
    x = np.ascontiguousarray(np.asarray(tokens, np.int8))
    if x.ndim != 2 or x.shape[1] != 192 or not 2 <= x.shape[0] <= 197:
        raise ValueError("selector input needs CLS plus 1..196 candidates of 192 values")
    c = x.shape[0] - 1
    dev = torch.device("cuda", torch.cuda.current_device())
    dx = torch.from_numpy(x).to(dev)
    doff = torch.tensor([0, x.shape[0]], dtype=torch.int32, device=dev)
    h2 = torch.zeros((1, 3, 196, 16), dtype=torch.int8, device=dev)
    model = selector_model_for(params)
    check(lib().hv_selector_h2(model.handle, 0, C.c_void_p(dx.data_ptr()), C.c_void_p(doff.data_ptr()), 1,
                               C.c_void_p(h2.data_ptr()), _stream(torch)))
    return h2.cpu().numpy()[0, :, :c]


def calibrate_selector(stage, tokens, package_present, base_params):
    """weights.py:158-204: ``(params, summary)`` for the first accepted attempt;
    RuntimeError after 256 failed attempts."""
    tokens = np.asarray(tokens, np.int8)
    h2 = selector_h2(tokens, base_params).astype(np.int64)
    for attempt in range(ATTEMPTS):
        w3 = np.array(synth._reference_w3(stage, attempt), np.int64)
        diffs = np.einsum("hck,hk->hc", h2, w3[:, :, 1] - w3[:, :, 0]).reshape(-1)
        if np.all(diffs == diffs[0]):
            continue
        median = int(np.sort(diffs)[diffs.size // 2])
        params = synth._calibrated_selector(base_params, stage, attempt, median)
        r = token_selector_batch([tokens], [package_present], params)[0]
        if r["kept_normal_count"] >= 1 and r["pruned_normal_count"] >= 2:
            summary = {
                "stage": stage,
                "attempt": attempt,
                "seed": SEED + stage * 1000 + attempt,
                "median_logit_diff": median,
                "input_tokens": int(tokens.shape[0]),
                "output_tokens": r["token_count"],
                "kept_normal": r["kept_normal_count"],
                "pruned_normal": r["pruned_normal_count"],
                "package_present": int(r["package_present"]),
            }
            return params, summary
    raise RuntimeError(f"selector stage {stage} calibration failed")


def build_params(image):
    """weights.py:207-251: ``(HeatViTParams, selector_summary, token_counts)`` of
    the reference's deterministic model, calibrated on ``image``."""
    base = synth.reference_seeded_base()
    x = np.asarray(patch_embedding(image, base["patch"]), np.int8)
    package_present = False
    summary, selectors, token_counts = [], [], [197]
    stage = 0
    for block_number in range(1, 13):
        if block_number in (4, 7, 10):
            stage += 1
            params, s = calibrate_selector(stage, x, package_present, base["bases"][stage - 1])
            selectors.append(params)
            summary.append(s)
            r = token_selector_batch([x], [package_present], params)[0]
            x = np.asarray(r["tokens"], np.int8)
            package_present = r["package_present"]
            token_counts.append(r["token_count"])
        x = transformer_block_batch([x], base["blocks"][block_number - 1])[0]
    params = HeatViTParams(patch=base["patch"], blocks=base["blocks"], selectors=tuple(selectors),
                           final_gamma=base["final_gamma"], final_beta=base["final_beta"],
                           head_w=base["head_w"], head_b=base["head_b"])
    return params, summary, token_counts
