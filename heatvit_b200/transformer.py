"""GPU mirror of verification/heatvit_ref/transformer.py.

``patch_embedding``, ``mhsa``, ``ffn`` and ``transformer_block`` keep the golden
signatures and return the same checkpoint dictionaries; each step runs on the
GPU through the per-operator C ABI (GEMM, writeback, LayerNorm, softmax,
GELU, align-add).  The fused single-kernel-per-stage path used for batched
inference is ``Engine.transformer_block`` / ``transformer_block_batch``.
"""

import ctypes as C

import numpy as np

from ._convert import int_array, to_device
from ._lib import check, lib
from .engine import _stream, _torch, block_model_for
from .gemm import _gemm_acc, writeback_array
from .layout import head_concat, patchify, qkv_unpack
from .nonlinear import gelu_array, layernorm_rows, softmax_rows
from .params import (  # noqa: F401  (re-exported golden names)
    BlockParams, FfnParams, MhsaParams, PatchParams, block_from, ffn_from, mhsa_from, patch_from,
)


def align_add_array(a, a_exp, b, b_exp, out_exp):
    """transformer.py:96-101 _align_add_requant on int8 arrays (GPU)."""
    torch = _torch()
    aa = int_array("main", a, -128, 127, dtype=np.int8)
    bb = int_array("aux", b, -128, 127, dtype=np.int8)
    if aa.shape != bb.shape:
        raise ValueError("align-add operands must have the same shape")
    dev = torch.device("cuda", torch.cuda.current_device())
    da, db = to_device(aa.reshape(-1), torch, dev), to_device(bb.reshape(-1), torch, dev)
    out = torch.empty_like(da)
    check(lib().hv_align_add_i8(C.c_void_p(da.data_ptr()), int(a_exp), C.c_void_p(db.data_ptr()), int(b_exp),
                                int(out_exp), da.numel(), C.c_void_p(out.data_ptr()), _stream(torch)))
    return out.cpu().numpy().reshape(aa.shape)


def _rows8(name, x, cols):
    if not isinstance(x, (list, tuple, np.ndarray)):
        raise ValueError(f"{name} must be a list of rows")
    a = int_array(name, x, -128, 127, dtype=np.int64) if len(x) else np.zeros((0, cols), np.int64)
    if a.ndim != 2 or a.shape[1] != cols:
        raise ValueError(f"{name} rows must have {cols} elements")
    return a


def patch_embedding(image, params):
    """transformer.py:104-145: NHWC image -> [197][192] int8 at tokens_scale_exp."""
    if not isinstance(params, PatchParams) and not hasattr(params, "patch_weight"):
        raise TypeError("params must be PatchParams")
    p = patch_from(params)
    if isinstance(image, (bytes, bytearray)) or not isinstance(image, (list, tuple, np.ndarray)):
        raise TypeError("image must be a flat list")
    if len(image) != p.height * p.width * 3:
        raise ValueError("image length mismatch")
    patches = patchify(list(image) if not isinstance(image, np.ndarray) else image, p.width, p.patch)
    acc = _gemm_acc(patches, p.patch_weight, p.patch_bias, False, False)
    embed = writeback_array(acc, p.image_scale_exp + p.weight_scale_exp, p.activation_scale_exp, 8)
    row0 = align_add_array(p.cls, p.cls_scale_exp, p.pos[0], p.pos_scale_exp, p.tokens_scale_exp)
    rest = align_add_array(embed, p.activation_scale_exp, p.pos[1:], p.pos_scale_exp, p.tokens_scale_exp)
    return np.concatenate([row0[None, :], rest], axis=0).tolist()


def mhsa(x, params):
    """transformer.py:201-284: returns (output, checkpoints)."""
    if not isinstance(params, MhsaParams) and not hasattr(params, "wqkv"):
        raise TypeError("params must be MhsaParams")
    p = mhsa_from(params)
    xa = _rows8("x", x, p.embed_dim)
    n = xa.shape[0]
    ln1, _neg = layernorm_rows(xa, p.ln_gamma, p.ln_beta, p.x_scale_exp, p.gamma1_scale_exp,
                               p.beta1_scale_exp, p.ln1_out_scale_exp)
    fused = writeback_array(_gemm_acc(ln1, p.wqkv, p.bqkv, False, False),
                            p.ln1_out_scale_exp + p.wqkv_scale_exp, p.qkv_out_scale_exp, 8)
    qkv = np.asarray(qkv_unpack(fused, n), np.int64) if n else np.zeros((3, 3, 0, 64), np.int64)
    score, prob, context = [], [], []
    for h in range(p.heads):
        s = writeback_array(_gemm_acc(qkv[0][h], qkv[1][h], None, True, False),
                            2 * p.qkv_out_scale_exp, p.score_scale_exp, 32)
        score.append(s)
        q16 = writeback_array(s.astype(np.int64), 0, -(p.score_scale_exp + 13), 24)
        pr = softmax_rows(q16.reshape(-1), [n] * n, 0).reshape(n, n) if n else np.zeros((0, 0), np.uint8)
        prob.append(pr)
        ctx = writeback_array(_gemm_acc(pr, qkv[2][h], None, False, True),
                              p.prob_scale_exp + p.qkv_out_scale_exp, p.context_out_scale_exp, 8)
        context.append(ctx)
    concat = np.asarray(head_concat([c.tolist() for c in context], n), np.int64).reshape(n, 192)
    out = writeback_array(_gemm_acc(concat, p.wproj, p.bproj, False, False),
                          p.context_out_scale_exp + p.wproj_scale_exp, p.msa_out_scale_exp, 8)
    checkpoints = {
        "ln1": ln1.tolist(),
        "fused_qkv": fused.tolist(),
        "qkv": qkv.tolist(),
        "score": [s.tolist() for s in score],
        "prob": [q.tolist() for q in prob],
        "context": [c.tolist() for c in context],
        "concat": concat.tolist(),
        "msa": out.tolist(),
    }
    return out.tolist(), checkpoints


def ffn(y, params):
    """transformer.py:328-384: returns (z, checkpoints)."""
    if not isinstance(params, FfnParams) and not hasattr(params, "w1"):
        raise TypeError("params must be FfnParams")
    p = ffn_from(params)
    ya = _rows8("y", y, p.embed_dim)
    ln2, _neg = layernorm_rows(ya, p.ln_gamma, p.ln_beta, p.x_scale_exp, p.gamma2_scale_exp,
                               p.beta2_scale_exp, p.ln2_out_scale_exp)
    acc = _gemm_acc(ln2, p.w1, p.b1, False, False)
    q16 = writeback_array(acc, p.ln2_out_scale_exp + p.w1_scale_exp, -16, 24)
    hidden = writeback_array(gelu_array(q16).astype(np.int64), -16, p.hidden_out_scale_exp, 8)
    ffn_out = writeback_array(_gemm_acc(hidden, p.w2, p.b2, False, False),
                              p.hidden_out_scale_exp + p.w2_scale_exp, p.ffn_out_scale_exp, 8)
    z = align_add_array(ya, p.x_scale_exp, ffn_out, p.ffn_out_scale_exp, p.out_scale_exp)
    checkpoints = {"ln2": ln2.tolist(), "hidden": hidden.tolist(), "ffn_out": ffn_out.tolist(), "z": z.tolist()}
    return z.tolist(), checkpoints


def transformer_block(x, params):
    """transformer.py:401-431: Y = X + MSA(LN1(X)); Z = Y + FFN(LN2(Y))."""
    if not isinstance(params, BlockParams) and not hasattr(params, "mhsa"):
        raise TypeError("params must be BlockParams")
    p = block_from(params)
    xa = _rows8("x", x, p.mhsa.embed_dim)
    msa_out, msa_ck = mhsa(xa, p.mhsa)
    y = align_add_array(xa, p.mhsa.x_scale_exp, msa_out, p.mhsa.msa_out_scale_exp, p.ffn.x_scale_exp)
    z, ffn_ck = ffn(y, p.ffn)
    checkpoints = dict(msa_ck)
    checkpoints["y"] = y.tolist()
    checkpoints.update(ffn_ck)
    return z, checkpoints


def transformer_block_batch(xs, params):
    """The fused CUDA block over many token matrices at once (ragged batch).

    ``xs`` is a list of [n_i][192] int8 matrices; returns the list of z_i."""
    torch = _torch()
    p = block_from(params)
    mats = [_rows8("x", x, 192) for x in xs]
    counts = np.array([m.shape[0] for m in mats], np.int64)
    if np.any(counts < 1) or np.any(counts > 197):
        raise ValueError("each token matrix must hold 1..197 rows")
    off = np.zeros(len(mats) + 1, np.int32)
    off[1:] = np.cumsum(counts)
    dev = torch.device("cuda", torch.cuda.current_device())
    dx = to_device(np.concatenate(mats, axis=0).astype(np.int8), torch, dev)
    doff = to_device(off, torch, dev)
    z = torch.empty_like(dx)
    model = block_model_for(p)
    check(lib().hv_transformer_block(model.handle, 0, C.c_void_p(dx.data_ptr()), C.c_void_p(doff.data_ptr()),
                                     len(mats), int(off[-1]), C.c_void_p(z.data_ptr()), _stream(torch)))
    zz = z.cpu().numpy()
    return [zz[off[i]:off[i + 1]] for i in range(len(mats))]
