"""heatvit_b200 — B200-native (sm_100a) batched integer inference for HeatViT-T.

The compute path is the in-tree CUDA library (heatvit_b200/_lib) behind the C
ABI in include/heatvit_b200.h.  The Python modules mirror the reference
golden model's entry points (verification/heatvit_ref): ``model``,
``transformer``, ``selector``, ``nonlinear``, ``gemm``, ``layout``; parameter
dataclasses with the golden field names live in ``params``.
"""

from . import abi  # noqa: F401
from .params import (  # noqa: F401
    BlockParams, FfnParams, HeatViTParams, MhsaParams, PatchParams, SelectorHeadWeightParams,
    SelectorLocalParams, SelectorParams, SelectorScoreParams, from_reference,
)

__version__ = "0.1.0"


def __getattr__(name):
    # Lazy imports keep ``import heatvit_b200`` cheap and torch-free.
    if name in ("Engine",):
        from .engine import Engine
        return Engine
    if name in ("HeatViTModel", "ModelResult"):
        from . import model
        return getattr(model, name)
    raise AttributeError(name)
