"""GPU mirror of verification/heatvit_ref/selector.py (token_selector and its result).

``token_selector`` runs the fused per-image selector kernel (one CTA per
image: local MLP, global mean, score MLP, keep scores, head weights, head
fusion, inclusive threshold, stable compaction, package token) and returns the
golden ``SelectorResult`` with every intermediate.  ``token_selector_batch``
runs many images in one launch over the ragged layout.
"""

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import abi
from ._convert import int_array, to_device
from ._lib import check, lib
from .engine import _stream, _torch, selector_model_for
from .params import (  # noqa: F401  (re-exported golden names)
    SelectorHeadWeightParams, SelectorLocalParams, SelectorParams, SelectorScoreParams, selector_from,
)

WARN_HEAD_DEN_ZERO = 1 << 0
WARN_PACKAGE_DEN_ZERO = 1 << 1
KEEP_THRESHOLD = 32768
Q016_ONE = 65536
MAX_CANDIDATES = 196


@dataclass(frozen=True)
class SelectorResult:
    """selector.py:235-250."""

    tokens: tuple = ()
    token_count: int = 0
    package_present: bool = False
    kept_normal_count: int = 0
    pruned_normal_count: int = 0
    warnings: int = 0
    local: tuple = ()
    global_features: tuple = ()
    head_scores: tuple = ()
    head_stats: tuple = ()
    head_weights: tuple = ()
    fused_scores: tuple = ()


def _tup(a):
    a = np.asarray(a)
    return tuple(_tup(x) for x in a) if a.ndim > 1 else tuple(int(v) for v in a)


def token_selector_batch(token_mats, package_flags, params, intermediates=False):
    """Fused selector over a ragged batch of [n_i][192] token matrices.

    Returns a list of dicts with tokens [n'][192] (numpy), counts, flags,
    warnings and, with ``intermediates``, the SelectorResult fields."""
    torch = _torch()
    sp = selector_from(params)
    mats = []
    for t in token_mats:
        if not isinstance(t, (list, tuple, np.ndarray)) or len(t) < 2:
            raise ValueError("selector input needs CLS plus at least one candidate")
        a = int_array("tokens", t, -128, 127, ndim=2)
        if a.shape[1] != 192:
            raise ValueError("tokens must have 192 elements per row")
        if a.shape[0] > 197:
            raise ValueError("at most 197 tokens per image")
        mats.append(a)
    b = len(mats)
    counts = np.array([m.shape[0] for m in mats], np.int64)
    off = np.zeros(b + 1, np.int32)
    off[1:] = np.cumsum(counts)
    pk = np.array([1 if bool(f) else 0 for f in package_flags], np.uint8)
    dev = torch.device("cuda", torch.cuda.current_device())
    dx = to_device(np.concatenate(mats, axis=0).astype(np.int8), torch, dev)
    doff = to_device(off, torch, dev)
    dpk = to_device(pk, torch, dev)
    dy = torch.empty_like(dx)
    doff_out = torch.empty(b + 1, dtype=torch.int32, device=dev)
    dpk_out = torch.empty(b, dtype=torch.uint8, device=dev)
    dsum = torch.zeros((b, 6), dtype=torch.int32, device=dev)
    C_ = MAX_CANDIDATES
    bufs = {}
    if intermediates:
        bufs = dict(fused=torch.zeros((b, C_), dtype=torch.int32, device=dev),
                    head_scores=torch.zeros((b, 3, C_), dtype=torch.int32, device=dev),
                    head_weights=torch.zeros((b, C_, 3), dtype=torch.int32, device=dev),
                    local=torch.zeros((b, 3, C_, 32), dtype=torch.int8, device=dev),
                    global_=torch.zeros((b, 3, 32), dtype=torch.int8, device=dev),
                    stats=torch.zeros((b, C_, 3), dtype=torch.int8, device=dev))
    ptr = lambda k: C.c_void_p(bufs[k].data_ptr()) if k in bufs else None
    model = selector_model_for(sp)
    check(lib().hv_token_selector(model.handle, 0, C.c_void_p(dx.data_ptr()), C.c_void_p(doff.data_ptr()),
                                  C.c_void_p(dpk.data_ptr()), b, C.c_void_p(dy.data_ptr()),
                                  C.c_void_p(doff_out.data_ptr()), C.c_void_p(dpk_out.data_ptr()),
                                  C.c_void_p(dsum.data_ptr()), ptr("fused"), ptr("head_scores"),
                                  ptr("head_weights"), ptr("local"), ptr("global_"), ptr("stats"), _stream(torch)))
    y = dy.cpu().numpy()
    oo = doff_out.cpu().numpy()
    summ = dsum.cpu().numpy()
    host = {k: v.cpu().numpy() for k, v in bufs.items()}
    results = []
    for i in range(b):
        s = dict(zip(abi.SUMMARY_FIELDS, (int(v) for v in summ[i])))
        r = dict(tokens=y[oo[i]:oo[i + 1]], token_count=int(oo[i + 1] - oo[i]),
                 package_present=bool(s["package_present"]), kept_normal_count=s["kept_normal"],
                 pruned_normal_count=s["pruned_normal"], warnings=s["warnings"])
        if intermediates:
            c = int(counts[i]) - 1
            r.update(local=host["local"][i][:, :c], global_features=host["global_"][i],
                     head_scores=host["head_scores"][i][:, :c], head_stats=host["stats"][i][:c],
                     head_weights=host["head_weights"][i][:c], fused_scores=host["fused"][i][:c])
        results.append(r)
    return results


def token_selector(tokens, package_present, params):
    """selector.py:503-563: returns a SelectorResult."""
    if not isinstance(params, SelectorParams) and not hasattr(params, "head_weight"):
        raise TypeError("params must be SelectorParams")
    if not isinstance(tokens, (list, tuple, np.ndarray)) or len(tokens) < 2:
        raise ValueError("selector input needs CLS plus at least one candidate")
    r = token_selector_batch([tokens], [package_present], params, intermediates=True)[0]
    return SelectorResult(
        tokens=_tup(r["tokens"]), token_count=r["token_count"], package_present=r["package_present"],
        kept_normal_count=r["kept_normal_count"], pruned_normal_count=r["pruned_normal_count"],
        warnings=r["warnings"], local=_tup(r["local"]), global_features=_tup(r["global_features"]),
        head_scores=_tup(r["head_scores"]), head_stats=_tup(r["head_stats"]),
        head_weights=_tup(r["head_weights"]), fused_scores=_tup(r["fused_scores"]))
