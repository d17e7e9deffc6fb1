"""Mirror of verification/heatvit_ref/layout.py (pure data movement).

In the fused pipeline these layouts never materialise: patchify is the patch
GEMM's A-operand addressing, qkv_unpack/head_concat are the attention
kernel's load/store addressing.  These functions exist for the per-component
API and return the golden layouts as Python lists.
"""

import numpy as np

from ._convert import check_int, int_array


def patchify(image, width, patch):
    """layout.py:31-72: NHWC -> [patches][patch*patch*3], (in_row, in_col, ch) order."""
    width = check_int("width", width)
    patch = check_int("patch", patch)
    if width <= 0 or patch <= 0 or width % patch != 0:
        raise ValueError("width must be a positive multiple of patch")
    img = int_array("image", image, -128, 127, ndim=1)
    if img.size % (width * 3) != 0:
        raise ValueError("image length is not width*3*height")
    height = img.size // (width * 3)
    if height % patch != 0:
        raise ValueError("height must be a multiple of patch")
    pr, pc = height // patch, width // patch
    t = img.reshape(pr, patch, pc, patch, 3).transpose(0, 2, 1, 3, 4)
    return t.reshape(pr * pc, patch * patch * 3).tolist()


def add_pos(patch_embed, cls, pos):
    """layout.py:75-89: saturating row-wise add of the positional table."""
    cls = int_array("cls", cls, -128, 127, ndim=1)
    pos = int_array("pos", pos, -128, 127, ndim=2)
    pe = int_array("patch_embed", patch_embed, -128, 127, ndim=2)
    if pos.shape[0] != pe.shape[0] + 1:
        raise ValueError("pos must have one more row than patch_embed")
    rows = np.concatenate([cls[None, :], pe], axis=0) + pos
    return np.clip(rows, -128, 127).tolist()


def qkv_unpack(fused_qkv, tokens):
    """layout.py:92-129: [token][Q192,K192,V192] -> [kind][head][token][64]."""
    tokens = check_int("tokens", tokens)
    if tokens < 0:
        raise ValueError("tokens must be non-negative")
    f = int_array("fused_qkv", fused_qkv, -128, 127, ndim=2) if tokens else np.zeros((0, 576), np.int64)
    if f.shape[0] != tokens or (tokens and f.shape[1] != 576):
        raise ValueError("fused_qkv row count must equal tokens")
    return f.reshape(tokens, 3, 3, 64).transpose(1, 2, 0, 3).tolist()


def head_concat(context, tokens):
    """layout.py:132-155: [head][token][64] -> [token][192]."""
    tokens = check_int("tokens", tokens)
    if tokens < 0:
        raise ValueError("tokens must be non-negative")
    if not isinstance(context, (list, tuple, np.ndarray)) or len(context) != 3:
        raise ValueError("context must have 3 heads")
    c = int_array("context", context, -128, 127)
    if c.shape[:2] != (3, tokens):
        raise ValueError("context head row count must equal tokens")
    return c.transpose(1, 0, 2).reshape(tokens, 192).tolist()
