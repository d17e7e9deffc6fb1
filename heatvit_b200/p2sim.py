"""Batched, pruned P2-simulator inference on the GPU, for accuracy evaluation.

The reference's P2 accuracy tooling runs the integer DeiT-T of a ``QuantDeiT``
(int8 / int32 tensors plus a ScaleTable) on normalised float images:
tools/p2/p2_sim.py ``forward_image`` one image at a time (pruned or not),
tools/p2/p2_sim_ivit.py ``forward_batch_cfg`` batched but unpruned, and
tools/p2/p2_ivit.py ``eval_top1`` over a labelled loader.  Here the same
computation runs batched and pruned on the CUDA engine:

* image quantisation (p2_sim.py:536-541): q = clamp(round_half_even(x / 2^e),
  -128, 127) with e the table's "input" exponent, CHW float planes to the
  golden image's HWC int8 order, one kernel (``hv_quantize_images``);
* the model: a ``QuantDeiT``'s tensors through the scale-table mapping of
  tools/p2/p2_export_weights.py (``memimage.params_from_tensors``);
  ``prune=False`` leaves the selectors out (p2_sim.py:571-579);
* the forward pass: ``Engine.infer`` on the whole batch.

The P2 simulator's contract configuration equals the golden model bit for bit
(its LayerNorm square root is a float64 floor that agrees with the integer
square root below 2^40), so the results are the golden model's.
"""

import ctypes as C
import time
from collections import OrderedDict

import numpy as np

from . import abi, memimage
from ._lib import check, lib
from .engine import Engine, _stream, _torch

LOGIT_SCALE_EXP = abi.LOGIT_SCALE_EXP
_BLOCK_FIELDS = ("gamma1", "beta1", "wqkv", "bqkv", "wproj", "bproj", "gamma2", "beta2", "w1", "b1", "w2", "b2")
_SEL_FIELDS = ("local_w", "local_b", "score_w1", "score_b1", "score_w2", "score_b2", "score_w3", "score_b3",
               "hw_w1", "hw_b1", "hw_w2", "hw_b2")


def _np(t):
    if hasattr(t, "detach"):
        t = t.detach().cpu().numpy()
    return np.asarray(t)


def _table(scales):
    if isinstance(scales, dict):
        return {"weights": dict(scales["weights"]), "activations": dict(scales["activations"])}
    return {"weights": dict(scales.weights), "activations": dict(scales.activations)}


def params_from_quant_deit(model, prune=True):
    """HeatViTParams of a ``QuantDeiT`` (p2_sim.py:291-304; any object with its
    fields: ``scales`` with ``weights`` / ``activations`` maps, the tensors as
    torch tensors or arrays).  ``prune=False`` or an empty ``selectors`` list
    gives the unpruned model."""
    t = {k: _np(getattr(model, k)) for k in ("patch_w", "patch_b", "cls", "pos", "final_gamma", "final_beta",
                                              "head_w", "head_b")}
    if len(model.blocks) != 12:
        raise ValueError("the model has 12 blocks")
    for n, b in enumerate(model.blocks, start=1):
        t.update({f"b{n}_{f}": _np(getattr(b, f)) for f in _BLOCK_FIELDS})
    sels = list(model.selectors) if prune else []
    if len(sels) not in (0, 3):
        raise ValueError("a pruned model has three selectors (before blocks 4, 7 and 10)")
    for s, sp in enumerate(sels, start=1):
        t.update({f"s{s}_{f}": _np(getattr(sp, f)) for f in _SEL_FIELDS})
    return memimage.params_from_tensors(t, _table(model.scales), selectors=len(sels))


def quantize_images(images, input_exp):
    """CUDA float32 images [B, 3, 224, 224] -> CUDA int8 [B, 150528] (HWC)."""
    torch = _torch()
    if not images.is_cuda or images.dtype != torch.float32:
        raise TypeError("images must be a CUDA float32 tensor")
    if tuple(images.shape[1:]) != (3, 224, 224):
        raise ValueError("images must be [B, 3, 224, 224]")
    images = images.contiguous()
    out = torch.empty((images.shape[0], abi.IMAGE_BYTES), dtype=torch.int8, device=images.device)
    with torch.cuda.device(images.device):
        check(lib().hv_quantize_images(C.c_void_p(images.data_ptr()), int(images.shape[0]), int(input_exp),
                                       C.c_void_p(out.data_ptr()), _stream(torch)))
    return out


class Simulator:
    """A ``QuantDeiT`` packed on one GPU.  ``forward_batch(images)`` takes float
    images [B, 3, 224, 224] (CUDA or host) and returns CUDA logits [B, 1000]
    int32 at 2^-14 and token counts [B, S+1]."""

    def __init__(self, model, prune=True, device=None):
        self.params = params_from_quant_deit(model, prune)
        self.prune = bool(self.params.selectors)
        self.input_exp = self.params.patch.image_scale_exp
        self.engine = Engine(self.params, device)

    def forward_batch(self, images):
        torch = _torch()
        if not torch.is_tensor(images):
            images = torch.from_numpy(np.ascontiguousarray(images, np.float32))
        images = images.to(self.engine.device, torch.float32)
        if images.dim() == 3:
            images = images.unsqueeze(0)
        q = quantize_images(images, self.input_exp)
        out = self.engine.infer(q)
        return out["logits"], out["token_counts"]

    def forward_image(self, image_float):
        """p2_sim.py:527-581: (logits [1000] int32, token_counts list, -14)."""
        logits, counts = self.forward_batch(image_float)
        return logits[0], [int(v) for v in counts[0].cpu()], LOGIT_SCALE_EXP

    def eval_top1(self, loader):
        """p2_ivit.py:255-265: (top-1 % , seconds, correct, total) over a loader of
        (images [B, 3, 224, 224], labels [B])."""
        torch = _torch()
        correct = total = 0
        t0 = time.time()
        for img, label in loader:
            logits, _ = self.forward_batch(img)
            pred = logits.argmax(dim=1).cpu()
            label = torch.as_tensor(label).reshape(-1).cpu()
            correct += int((pred == label).sum())
            total += int(label.numel())
        elapsed = time.time() - t0
        return (100.0 * correct / total if total else 0.0), elapsed, correct, total


_SIMS = OrderedDict()  # id(model) -> (model, {(prune, device): Simulator}), most recent last
_SIMS_MAX = 4


def simulator_for(model, prune=True):
    """The cached ``Simulator`` of a model object (the four most recently used
    models stay packed; the cache holds a reference to each).  A model's tensors
    are read when it is first used: after changing them in place, build a new
    ``Simulator``."""
    torch = _torch()
    key = (bool(prune), torch.cuda.current_device())
    ent = _SIMS.get(id(model))
    if ent is None or ent[0] is not model:
        ent = (model, {})
        _SIMS[id(model)] = ent
    _SIMS.move_to_end(id(model))
    while len(_SIMS) > _SIMS_MAX:
        _SIMS.popitem(last=False)
    if key not in ent[1]:
        ent[1][key] = Simulator(model, prune)
    return ent[1][key]


def forward_image(model, image_float, rec=None, prune=True):
    """p2_sim.forward_image on the GPU: (logits [1000] int32 CUDA tensor,
    token_counts, -14).  ``rec`` (the reference's activation recorder) is not
    supported."""
    if rec is not None:
        raise NotImplementedError("activation recording is not supported on the GPU path")
    return simulator_for(model, prune).forward_image(image_float)


def forward_batch(model, images, prune=True):
    """Batched pruned (or unpruned) inference: (logits [B, 1000] int32 CUDA
    tensor, token counts [B, S+1], -14)."""
    logits, counts = simulator_for(model, prune).forward_batch(images)
    return logits, counts, LOGIT_SCALE_EXP


def eval_top1(model, loader, prune=True):
    """p2_ivit.eval_top1 over the pruned (default) or unpruned model."""
    return simulator_for(model, prune).eval_top1(loader)
