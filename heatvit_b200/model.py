"""GPU mirror of verification/heatvit_ref/model.py (HeatViTModel, ModelResult).

``HeatViTModel().infer(image, params)`` has the golden signature and return
type and runs the fused CUDA pipeline (``Engine``) with checkpoint capture.
``infer_batch`` is the batched form: images [B, 150528] (numpy or CUDA
tensor) -> logits [B, 1000] int32 at 2^-14 plus token counts, selector
summaries and warning bits, without per-image Python work.
"""

from dataclasses import dataclass

import numpy as np

from . import abi
from .engine import Engine, _torch, engine_for
from .params import HeatViTParams, from_reference  # noqa: F401

LOGIT_SCALE_EXP = abi.LOGIT_SCALE_EXP


@dataclass(frozen=True)
class ModelResult:
    """model.py:49-56."""

    logits: tuple
    output_scale_exp: int
    checkpoints: dict
    selector_summary: tuple


def _golden_checkpoints(ck, rows, num_selectors):
    out = {"patch": ck[abi.CKPT_PATCH][:rows[abi.CKPT_PATCH]].tolist()}
    for s in range(1, num_selectors + 1):
        slot = abi.ckpt_selector(s)
        out[f"selector_{s:02d}"] = ck[slot][:rows[slot]].tolist()
    for b in range(1, 13):
        out[f"block_{b:02d}"] = ck[b][:rows[b]].tolist()
    out["final_ln"] = ck[abi.CKPT_FINAL_LN][:rows[abi.CKPT_FINAL_LN]].tolist()
    return out


class HeatViTModel:
    """Integer HeatViT-T inference on a B200 (model.py:70-123)."""

    def infer(self, image, params):
        if not isinstance(params, HeatViTParams) and not hasattr(params, "blocks"):
            raise TypeError("params must be HeatViTParams")
        torch = _torch()
        if isinstance(image, (bytes, bytearray)) or not isinstance(image, (list, tuple, np.ndarray)):
            raise TypeError("image must be a flat list")
        from ._convert import int_array
        img = int_array("image", image, -128, 127, dtype=np.int8).reshape(-1)
        if img.size != abi.IMAGE_BYTES:
            raise ValueError("image length mismatch")
        eng = engine_for(params)
        dimg = torch.from_numpy(img.reshape(1, -1)).to(eng.device)
        out = eng.infer(dimg, checkpoints=True)
        logits = out["logits"][0].cpu().numpy()
        ck = out["checkpoints"][0].cpu().numpy()
        rows = out["checkpoint_rows"][0].cpu().numpy()
        summ = out["summary"][0].cpu().numpy()
        ns = eng.num_selectors
        checkpoints = _golden_checkpoints(ck, rows, ns)
        checkpoints["logits"] = logits.tolist()
        selector_summary = tuple(
            {"input_tokens": int(s[0]), "output_tokens": int(s[1]), "kept_normal": int(s[2]),
             "pruned_normal": int(s[3]), "package_present": int(s[4])} for s in summ[:ns])
        return ModelResult(logits=tuple(int(v) for v in logits), output_scale_exp=LOGIT_SCALE_EXP,
                           checkpoints=checkpoints, selector_summary=selector_summary)

    def infer_batch(self, images, params, checkpoints=False):
        """Batched inference; returns numpy arrays (logits, token_counts,
        summary [B, S, 6], warnings, and checkpoints when requested)."""
        torch = _torch()
        eng = params if isinstance(params, Engine) else engine_for(params)
        if isinstance(images, np.ndarray):
            if images.dtype != np.int8:
                raise TypeError("images must be int8")
            images = torch.from_numpy(np.ascontiguousarray(images.reshape(images.shape[0], -1))).to(eng.device)
        out = eng.infer(images, checkpoints=checkpoints)
        return {k: v.cpu().numpy() for k, v in out.items()}
