"""Input validation and host<->device conversion shared by the golden-API mirror.

Mirrors the golden model's input checks: floats raise TypeError
(verification/heatvit_ref/fixed.py:10-12), ragged or out-of-range values raise
ValueError (gemm.py:19-36, layout.py:7-28).
"""

import numpy as np


def _has_float(value):
    if isinstance(value, float):
        return True
    if isinstance(value, np.ndarray):
        return value.dtype.kind in "fc"
    if isinstance(value, (list, tuple)):
        return any(_has_float(v) for v in value)
    return False


def int_array(name, value, lo, hi, ndim=None, dtype=np.int64):
    """Validated integer numpy array (rectangular, values in [lo, hi])."""
    if hasattr(value, "detach") and hasattr(value, "cpu"):  # torch tensor
        value = value.detach().cpu().numpy()
    if isinstance(value, np.ndarray):
        if value.dtype.kind in "fc":
            raise TypeError(f"{name} must be an integer, got float")
        arr = value
    else:
        if not isinstance(value, (list, tuple)):
            raise TypeError(f"{name} must be a list")
        if _has_float(value):
            raise TypeError(f"{name} must be an integer, got float")
        try:
            arr = np.array(value, dtype=object)
        except ValueError as exc:
            raise ValueError(f"{name} rows must have equal length") from exc
        if arr.dtype == object and arr.size and isinstance(arr.reshape(-1)[0], (list, tuple)):
            raise ValueError(f"{name} rows must have equal length")
        if arr.size and any(not isinstance(v, (int, np.integer, bool)) for v in arr.reshape(-1)):
            raise TypeError(f"{name} must hold integers")
        arr = arr.astype(np.int64) if arr.size else np.zeros(arr.shape, np.int64)
    if ndim is not None and arr.ndim != ndim:
        if arr.size == 0 and ndim == 2:
            arr = arr.reshape(0, 0)
        else:
            raise ValueError(f"{name} must be {ndim}-dimensional")
    if arr.size:
        mn, mx = int(arr.min()), int(arr.max())
        if mn < lo or mx > hi:
            raise ValueError(f"{name} values outside [{lo}, {hi}]")
    return np.ascontiguousarray(arr.astype(dtype))


def check_int(name, value):
    if isinstance(value, float):
        raise TypeError(f"{name} must be an integer, got float")
    return int(value)


def to_device(arr, torch, device):
    return torch.from_numpy(np.ascontiguousarray(arr)).to(device)


def to_list(t):
    if hasattr(t, "detach"):
        t = t.detach().cpu().numpy()
    return np.asarray(t).tolist()
