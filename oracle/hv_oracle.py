"""ctypes wrapper of the CPU oracle (oracle/heatvit_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / --impl reference legs of bench.py, as the checker.  The product
package never imports this module.

Each function mirrors a golden-model function of the reference
(verification/heatvit_ref) with numpy in/out and the same exception types.
"""

import ctypes as C
import os
import subprocess
import threading

import numpy as np

from heatvit_b200 import abi
from heatvit_b200.params import (
    PackedParams, _Keep, pack_block, pack_patch, pack_selector,
)

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libhv_oracle.so")
_lib = None
_lock = threading.Lock()

P = C.c_void_p
i64 = C.c_int64
i32 = C.c_int32


def build(force=False):
    """Compile the oracle with its Makefile (gcc only)."""
    if force or not os.path.exists(_LIB_PATH):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build()
            L = C.CDLL(_LIB_PATH)
            L.hvo_round_shift_away.restype = i64
            L.hvo_round_shift_away.argtypes = [i64, C.c_int]
            L.hvo_requant.restype = i64
            L.hvo_requant.argtypes = [i64, C.c_int, C.c_int, C.c_int]
            L.hvo_round_div.restype = i64
            L.hvo_round_div.argtypes = [i64, i64]
            L.hvo_isqrt.restype = C.c_uint64
            L.hvo_isqrt.argtypes = [C.c_uint64]
            L.hvo_gelu.restype = i32
            L.hvo_gelu.argtypes = [i64]
            L.hvo_plan_sigmoid.restype = i32
            L.hvo_plan_sigmoid.argtypes = [i64]
            L.hvo_softmax_selector.restype = C.c_int
            L.hvo_softmax_selector.argtypes = [P, C.c_int, P]
            L.hvo_softmax_attention.restype = C.c_int
            L.hvo_softmax_attention.argtypes = [P, C.c_int, P]
            L.hvo_softmax_rows.restype = C.c_int
            L.hvo_softmax_rows.argtypes = [P, P, C.c_int, C.c_int, P]
            L.hvo_layernorm.restype = C.c_int
            L.hvo_layernorm.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, P]
            L.hvo_gemm.restype = C.c_int
            L.hvo_gemm.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P]
            L.hvo_writeback.restype = None
            L.hvo_writeback.argtypes = [P, i64, C.c_int, C.c_int, C.c_int, P]
            L.hvo_gelu_chain.restype = C.c_int8
            L.hvo_gelu_chain.argtypes = [i64, C.c_int, C.c_int]
            for name in ("hvo_gelu_array", "hvo_plan_array"):
                getattr(L, name).restype = None
                getattr(L, name).argtypes = [P, i64, P]
            L.hvo_requant_array.restype = None
            L.hvo_requant_array.argtypes = [P, P, P, i64, C.c_int, P]
            L.hvo_gelu_chain_array.restype = None
            L.hvo_gelu_chain_array.argtypes = [P, i64, C.c_int, C.c_int, P]
            L.hvo_patch_embedding.restype = None
            L.hvo_patch_embedding.argtypes = [P, P, P]
            L.hvo_mhsa.restype = C.c_int
            L.hvo_mhsa.argtypes = [P, P, C.c_int, P, P]
            L.hvo_ffn.restype = C.c_int
            L.hvo_ffn.argtypes = [P, P, C.c_int, P, P, P, P]
            L.hvo_transformer_block.restype = C.c_int
            L.hvo_transformer_block.argtypes = [P, P, C.c_int, P, P]
            L.hvo_token_selector.restype = C.c_int
            L.hvo_token_selector.argtypes = [P, P, C.c_int, C.c_int, P, P, P]
            L.hvo_infer.restype = C.c_int
            L.hvo_infer.argtypes = [P, P, P, P, P, P, P]
            L.hvo_infer_batch.restype = C.c_int
            L.hvo_infer_batch.argtypes = [P, P, C.c_int, P, P, P, P, C.c_int]
            L.hvo_fuse_head_scores.restype = C.c_int
            L.hvo_fuse_head_scores.argtypes = [P, P, C.c_int, P]
            L.hvo_finalize_tokens.restype = C.c_int
            L.hvo_finalize_tokens.argtypes = [P, P, C.c_int, P, P, C.c_int, P, P]
            L.hvo_align_add_array.restype = None
            L.hvo_align_add_array.argtypes = [P, C.c_int, P, C.c_int, C.c_int, i64, P]
            L.hvo_num_cpus.restype = C.c_int
            L.hvo_num_cpus.argtypes = []
            _lib = L
    return _lib


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


def _i64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


class _MhsaCkpt(C.Structure):
    _fields_ = [("ln1", P), ("fused", P), ("score", P), ("prob", P), ("context", P), ("msa", P)]


class _SelCkpt(C.Structure):
    _fields_ = [("local", P), ("global_", P), ("head_scores", P), ("head_stats", P),
                ("head_weights", P), ("fused", P)]


# ---- L0 / L1 ---------------------------------------------------------------

def round_shift_away(v, shift):
    return lib().hvo_round_shift_away(int(v), int(shift))


def requant(v, src_exp, dst_exp, bits):
    return lib().hvo_requant(int(v), int(src_exp), int(dst_exp), int(bits))


def requant_array(values, src_exps, dst_exps, bits):
    v = _i64(values)
    s = np.ascontiguousarray(np.broadcast_to(np.asarray(src_exps, np.int32), v.shape))
    d = np.ascontiguousarray(np.broadcast_to(np.asarray(dst_exps, np.int32), v.shape))
    out = np.empty(v.shape, np.int64)
    lib().hvo_requant_array(_p(v), _p(s), _p(d), v.size, int(bits), _p(out))
    return out


def round_div(n, d):
    if d == 0:
        raise ValueError("division by zero")
    return lib().hvo_round_div(int(n), int(d))


def isqrt(x):
    if x < 0:
        raise ValueError("negative radicand")
    r = lib().hvo_isqrt(int(x))
    return r, int(x) - r * r


def gelu(x):
    return lib().hvo_gelu(int(x))


def gelu_array(x):
    x = _i64(x)
    out = np.empty(x.shape, np.int32)
    lib().hvo_gelu_array(_p(x), x.size, _p(out))
    return out


def plan_sigmoid(x):
    return lib().hvo_plan_sigmoid(int(x))


def plan_array(x):
    x = _i64(x)
    out = np.empty(x.shape, np.int32)
    lib().hvo_plan_array(_p(x), x.size, _p(out))
    return out


def gelu_chain_array(acc, src_exp, dst_exp):
    a = _i64(acc)
    out = np.empty(a.shape, np.int8)
    lib().hvo_gelu_chain_array(_p(a), a.size, int(src_exp), int(dst_exp), _p(out))
    return out


def softmax_selector(row):
    x = _i64(row)
    if x.size == 0:
        raise ValueError("softmax row must not be empty")
    out = np.empty(x.size, np.int32)
    if lib().hvo_softmax_selector(_p(x), x.size, _p(out)):
        raise ValueError("softmax row sum is zero")
    return out


def softmax_attention(row):
    x = _i64(row)
    if x.size == 0:
        raise ValueError("softmax row must not be empty")
    out = np.empty(x.size, np.uint8)
    if lib().hvo_softmax_attention(_p(x), x.size, _p(out)):
        raise ValueError("softmax row sum is zero")
    return out


def softmax_rows(x, offsets, mode):
    x = _i64(x)
    off = np.ascontiguousarray(np.asarray(offsets, np.int32))
    out = np.empty(x.size, np.uint8 if mode == 0 else np.int32)
    if lib().hvo_softmax_rows(_p(x), _p(off), off.size - 1, int(mode), _p(out)):
        raise ValueError("softmax row must not be empty")
    return out


def layernorm(x, gamma, beta, x_scale, gamma_scale, beta_scale, out_scale):
    x = np.ascontiguousarray(np.asarray(x, np.int8))
    g = np.ascontiguousarray(np.asarray(gamma, np.int8))
    b = np.ascontiguousarray(np.asarray(beta, np.int8))
    if x.shape[-1] != 192:
        raise ValueError("layernorm rows must have exactly 192 channels")
    rows = x.reshape(-1, 192)
    out = np.empty_like(rows)
    neg = np.zeros(rows.shape[0], bool)
    for r in range(rows.shape[0]):
        rc = lib().hvo_layernorm(_p(rows[r]), _p(g), _p(b), int(x_scale), int(gamma_scale),
                                 int(beta_scale), int(out_scale), _p(out[r]))
        if rc < 0:
            raise ValueError("layernorm input scale must be in [-32, 0]")
        neg[r] = rc > 0
    return out.reshape(x.shape), neg


def gemm(a, b, bias, transpose_b, a_unsigned=False):
    a = np.ascontiguousarray(np.asarray(a, np.uint8 if a_unsigned else np.int8))
    b = np.ascontiguousarray(np.asarray(b, np.int8))
    m, k = a.shape
    n = b.shape[0] if transpose_b else b.shape[1]
    bias_arr = None if bias is None else np.ascontiguousarray(np.asarray(bias, np.int32))
    acc = np.empty((m, n), np.int64)
    ovf = lib().hvo_gemm(_p(a), _p(b), None if bias_arr is None else _p(bias_arr),
                         m, n, k, int(bool(transpose_b)), int(bool(a_unsigned)), _p(acc))
    if ovf:
        raise OverflowError("GEMM accumulator exceeds int32")
    return acc


def writeback(acc, src_exp, dst_exp, bits):
    acc = _i64(acc)
    out = np.empty(acc.shape, np.int8 if bits == 8 else np.int32)
    lib().hvo_writeback(_p(acc), acc.size, int(src_exp), int(dst_exp), int(bits), _p(out))
    return out


# ---- L2 ----------------------------------------------------------------------

def patch_embedding(image, patch_params):
    keep = _Keep()
    s = pack_patch(patch_params, keep)
    img = np.ascontiguousarray(np.asarray(image, np.int8).reshape(-1))
    out = np.empty((197, 192), np.int8)
    lib().hvo_patch_embedding(C.addressof(s), _p(img), _p(out))
    return out


def mhsa(x, block_params, checkpoints=False):
    keep = _Keep()
    s = pack_block(block_params, keep)
    x = np.ascontiguousarray(np.asarray(x, np.int8))
    n = x.shape[0]
    out = np.empty((n, 192), np.int8)
    ck = None
    bufs = {}
    if checkpoints:
        bufs = dict(ln1=np.empty((n, 192), np.int8), fused=np.empty((n, 576), np.int8),
                    score=np.empty((3, n, n), np.int32), prob=np.empty((3, n, n), np.uint8),
                    context=np.empty((3, n, 64), np.int8), msa=np.empty((n, 192), np.int8))
        ck = _MhsaCkpt(*[_p(bufs[k]).value for k in ("ln1", "fused", "score", "prob", "context", "msa")])
    lib().hvo_mhsa(C.addressof(s), _p(x), n, _p(out), C.addressof(ck) if ck else None)
    return out, bufs


def ffn(y, block_params, checkpoints=False):
    keep = _Keep()
    s = pack_block(block_params, keep)
    y = np.ascontiguousarray(np.asarray(y, np.int8))
    n = y.shape[0]
    z = np.empty((n, 192), np.int8)
    bufs = {}
    ptrs = [None, None, None]
    if checkpoints:
        bufs = dict(ln2=np.empty((n, 192), np.int8), hidden=np.empty((n, 768), np.int8),
                    ffn_out=np.empty((n, 192), np.int8))
        ptrs = [_p(bufs["ln2"]), _p(bufs["hidden"]), _p(bufs["ffn_out"])]
    lib().hvo_ffn(C.addressof(s), _p(y), n, _p(z), *ptrs)
    return z, bufs


def transformer_block(x, block_params):
    keep = _Keep()
    s = pack_block(block_params, keep)
    x = np.ascontiguousarray(np.asarray(x, np.int8))
    n = x.shape[0]
    z = np.empty((n, 192), np.int8)
    y = np.empty((n, 192), np.int8)
    negv = lib().hvo_transformer_block(C.addressof(s), _p(x), n, _p(z), _p(y))
    return z, y, bool(negv)


def token_selector(tokens, package_present, selector_params):
    keep = _Keep()
    s = pack_selector(selector_params, keep)
    x = np.ascontiguousarray(np.asarray(tokens, np.int8))
    n = x.shape[0]
    if n < 2:
        raise ValueError("selector input needs CLS plus at least one candidate")
    c = n - 1
    y = np.empty((n, 192), np.int8)
    summ = abi.HvSelectorSummary()
    inter = dict(local=np.empty((3, c, 32), np.int8), global_features=np.empty((3, 32), np.int8),
                 head_scores=np.empty((3, c), np.int32), head_stats=np.empty((c, 3), np.int8),
                 head_weights=np.empty((c, 3), np.int32), fused_scores=np.empty(c, np.int32))
    ck = _SelCkpt(*[_p(inter[k]).value for k in ("local", "global_features", "head_scores",
                                                 "head_stats", "head_weights", "fused_scores")])
    nout = lib().hvo_token_selector(C.addressof(s), _p(x), n, int(bool(package_present)), _p(y),
                                    C.addressof(summ), C.addressof(ck))
    res = dict(tokens=y[:nout].copy(), token_count=nout)
    for f in abi.SUMMARY_FIELDS:
        res[f] = int(getattr(summ, f))
    res["package_present"] = bool(res["package_present"])
    res.update(inter)
    return res


def align_add_array(a, ea, b, eb, eo):
    """transformer.py:96-101 on int8 arrays."""
    a = np.ascontiguousarray(np.asarray(a, np.int8))
    b = np.ascontiguousarray(np.asarray(b, np.int8))
    out = np.empty_like(a)
    lib().hvo_align_add_array(_p(a), int(ea), _p(b), int(eb), int(eo), a.size, _p(out))
    return out


def fuse_head_scores(head_scores, head_weights):
    """selector.py:392-418: head_scores [3][C], head_weights [C][3]."""
    hs = np.ascontiguousarray(np.asarray(head_scores, np.int32))
    hw = np.ascontiguousarray(np.asarray(head_weights, np.int32))
    c = hs.shape[1]
    fused = np.empty(c, np.int32)
    warn = lib().hvo_fuse_head_scores(_p(hs), _p(hw), c, _p(fused))
    return fused, warn


def finalize_tokens(cls, normal, incoming_package, scores):
    """selector.py:421-500."""
    cls = np.ascontiguousarray(np.asarray(cls, np.int8).reshape(-1))
    width = cls.size
    normal = np.ascontiguousarray(np.asarray(normal, np.int8).reshape(-1, width))
    sc = np.ascontiguousarray(np.asarray(scores, np.int32))
    pkg = None if incoming_package is None else np.ascontiguousarray(np.asarray(incoming_package, np.int8))
    out = np.empty((normal.shape[0] + 2, width), np.int8)
    fin = abi.HvSelectorSummary()
    n = lib().hvo_finalize_tokens(_p(cls), _p(normal), normal.shape[0], None if pkg is None else _p(pkg), _p(sc),
                                  width, _p(out), C.addressof(fin))
    res = {f: int(getattr(fin, f)) for f in abi.SUMMARY_FIELDS}
    res["package_present"] = bool(res["package_present"])
    res["tokens"] = out[:n].copy()
    return res


def infer(params, image, checkpoints=True):
    packed = params if isinstance(params, PackedParams) else PackedParams(params)
    img = np.ascontiguousarray(np.asarray(image, np.int8).reshape(-1))
    if img.size != abi.IMAGE_BYTES:
        raise ValueError("image length mismatch")
    ns = packed.num_selectors
    logits = np.empty(1000, np.int32)
    counts = np.zeros(ns + 1, np.int32)
    summ = (abi.HvSelectorSummary * max(ns, 1))()
    ck = np.zeros((abi.CKPT_SLOTS, 197, 192), np.int8) if checkpoints else None
    rows = np.zeros(abi.CKPT_SLOTS, np.int32) if checkpoints else None
    warn = lib().hvo_infer(C.addressof(packed.struct), _p(img), _p(logits), _p(counts),
                           C.addressof(summ), None if ck is None else _p(ck),
                           None if rows is None else _p(rows))
    if warn < 0:
        raise ValueError("selector input needs CLS plus at least one candidate")
    summary = [{f: int(getattr(summ[i], f)) for f in abi.SUMMARY_FIELDS}
               for i in range(packed.used_selectors)]
    return dict(logits=logits, counts=counts[:packed.used_selectors + 1], summary=summary,
                warnings=warn, checkpoints=ck, checkpoint_rows=rows)


def infer_batch(params, images, threads=0):
    """Batched golden inference over host threads; returns a dict with
    logits [B,1000], counts [B,ns+1], summary [B,ns,6], warnings [B], threads."""
    packed = params if isinstance(params, PackedParams) else PackedParams(params)
    imgs = np.ascontiguousarray(np.asarray(images, np.int8).reshape(-1, abi.IMAGE_BYTES))
    b = imgs.shape[0]
    ns = packed.num_selectors
    logits = np.empty((b, 1000), np.int32)
    counts = np.zeros((b, ns + 1), np.int32)
    summ = np.zeros((b, max(ns, 1), 6), np.int32)
    warn = np.zeros(b, np.uint8)
    used = lib().hvo_infer_batch(C.addressof(packed.struct), _p(imgs), b, _p(logits), _p(counts),
                                 _p(summ), _p(warn), int(threads))
    return dict(logits=logits, counts=counts, summary=summ[:, :ns], warnings=warn, threads=used)


def num_cpus():
    return lib().hvo_num_cpus()
