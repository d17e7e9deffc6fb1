"""Frozen parameter dataclasses mirroring the golden model's, stored as numpy.

Field names, defaults and validation follow the reference dataclasses
(verification/heatvit_ref/transformer.py:51-93 PatchParams, :148-198
MhsaParams, :287-325 FfnParams, :387-398 BlockParams; selector.py:111-221
Selector*Params; model.py:24-46 HeatViTParams).  The golden classes hold
tuples of Python ints; these hold contiguous int8/int32 numpy arrays so they
can be handed to the C ABI without copies.  ``from_reference`` accepts any
object with the golden field names (duck typing), so instances of the
reference dataclasses convert directly.

Errors mirror the golden contract: floats raise TypeError, shape and range
violations raise ValueError.
"""

from dataclasses import dataclass, field, fields, replace
import ctypes as C

import numpy as np

from . import abi


def _reject_float(name, arr):
    if arr.dtype.kind == "f" or arr.dtype.kind == "c":
        raise TypeError(f"{name} must be an integer, got float")
    if arr.dtype == object:
        for v in arr.reshape(-1):
            if isinstance(v, float):
                raise TypeError(f"{name} must be an integer, got float")


def as_int_array(name, value, shape, lo, hi, dtype):
    """Validate ``value`` into a contiguous numpy array of ``shape``."""
    if isinstance(value, np.ndarray):
        arr = value
    else:
        if not isinstance(value, (list, tuple)):
            raise ValueError(f"{name} must be a list/tuple/array of shape {shape}")
        try:
            arr = np.asarray(value)
        except ValueError as exc:  # ragged nesting
            raise ValueError(f"{name} rows must have equal length") from exc
    _reject_float(name, arr)
    if tuple(arr.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(arr.shape)}")
    if arr.size:
        a64 = arr.astype(np.int64)
        if a64.min() < lo or a64.max() > hi:
            raise ValueError(f"{name} outside [{lo}, {hi}]")
    return np.ascontiguousarray(arr.astype(dtype))


def i8(name, value, shape):
    return as_int_array(name, value, shape, -128, 127, np.int8)


def i32(name, value, shape):
    return as_int_array(name, value, shape, -(1 << 31), (1 << 31) - 1, np.int32)


def _check_exp(name, value):
    if isinstance(value, float):
        raise TypeError(f"{name} must be an integer, got float")
    return int(value)


class _Frozen:
    def _set(self, name, value):
        object.__setattr__(self, name, value)

    def _ints(self):
        for f in fields(self):
            if f.name.endswith("_exp"):
                self._set(f.name, _check_exp(f.name, getattr(self, f.name)))


@dataclass(frozen=True, eq=False)
class PatchParams(_Frozen):
    """transformer.py:51-93."""

    patch_weight: object = ()
    patch_bias: object = ()
    cls: object = ()
    pos: object = ()
    width: int = 224
    height: int = 224
    patch: int = 16
    embed_dim: int = 192
    tokens: int = 197
    image_scale_exp: int = -7
    weight_scale_exp: int = -7
    activation_scale_exp: int = -7
    tokens_scale_exp: int = -7
    cls_scale_exp: int = -7
    pos_scale_exp: int = -7

    def __post_init__(self):
        if self.embed_dim != 192:
            raise ValueError("embed_dim must be 192")
        if self.tokens != 197:
            raise ValueError("tokens must be 197")
        if (self.width, self.height, self.patch) != (224, 224, 16):
            raise ValueError("this engine implements the 224x224 / 16x16 patch geometry")
        self._ints()
        self._set("patch_weight", i8("patch_weight", self.patch_weight, (768, 192)))
        self._set("patch_bias", i32("patch_bias", self.patch_bias, (192,)))
        self._set("cls", i8("cls", self.cls, (192,)))
        self._set("pos", i8("pos", self.pos, (197, 192)))


@dataclass(frozen=True, eq=False)
class MhsaParams(_Frozen):
    """transformer.py:148-198."""

    ln_gamma: object = ()
    ln_beta: object = ()
    wqkv: object = ()
    bqkv: object = ()
    wproj: object = ()
    bproj: object = ()
    embed_dim: int = 192
    heads: int = 3
    head_dim: int = 64
    x_scale_exp: int = -7
    gamma1_scale_exp: int = -6
    beta1_scale_exp: int = -7
    ln1_out_scale_exp: int = -7
    wqkv_scale_exp: int = -7
    qkv_out_scale_exp: int = -7
    score_scale_exp: int = -17
    prob_scale_exp: int = -8
    context_out_scale_exp: int = -7
    wproj_scale_exp: int = -7
    msa_out_scale_exp: int = -7

    def __post_init__(self):
        if self.embed_dim != 192 or self.heads != 3 or self.head_dim != 64:
            raise ValueError("MHSA dims must be 192/3/64")
        self._ints()
        self._set("ln_gamma", i8("ln_gamma", self.ln_gamma, (192,)))
        self._set("ln_beta", i8("ln_beta", self.ln_beta, (192,)))
        self._set("wqkv", i8("wqkv", self.wqkv, (192, 576)))
        self._set("bqkv", i32("bqkv", self.bqkv, (576,)))
        self._set("wproj", i8("wproj", self.wproj, (192, 192)))
        self._set("bproj", i32("bproj", self.bproj, (192,)))


@dataclass(frozen=True, eq=False)
class FfnParams(_Frozen):
    """transformer.py:287-325."""

    ln_gamma: object = ()
    ln_beta: object = ()
    w1: object = ()
    b1: object = ()
    w2: object = ()
    b2: object = ()
    embed_dim: int = 192
    ffn_dim: int = 768
    x_scale_exp: int = -7
    gamma2_scale_exp: int = -6
    beta2_scale_exp: int = -7
    ln2_out_scale_exp: int = -7
    w1_scale_exp: int = -7
    hidden_out_scale_exp: int = -7
    w2_scale_exp: int = -7
    ffn_out_scale_exp: int = -7
    out_scale_exp: int = -7

    def __post_init__(self):
        if self.embed_dim != 192 or self.ffn_dim != 768:
            raise ValueError("FFN dims must be 192/768")
        self._ints()
        self._set("ln_gamma", i8("ln_gamma", self.ln_gamma, (192,)))
        self._set("ln_beta", i8("ln_beta", self.ln_beta, (192,)))
        self._set("w1", i8("w1", self.w1, (192, 768)))
        self._set("b1", i32("b1", self.b1, (768,)))
        self._set("w2", i8("w2", self.w2, (768, 192)))
        self._set("b2", i32("b2", self.b2, (192,)))


@dataclass(frozen=True, eq=False)
class BlockParams(_Frozen):
    """transformer.py:387-398."""

    mhsa: MhsaParams
    ffn: FfnParams

    def __post_init__(self):
        if not isinstance(self.mhsa, MhsaParams):
            raise TypeError("mhsa must be MhsaParams")
        if not isinstance(self.ffn, FfnParams):
            raise TypeError("ffn must be FfnParams")


@dataclass(frozen=True, eq=False)
class SelectorLocalParams(_Frozen):
    """selector.py:111-126."""

    w: object = ()
    b: object = ()

    def __post_init__(self):
        self._set("w", i8("local w", self.w, (3, 64, 32)))
        self._set("b", i32("local b", self.b, (3, 32)))


@dataclass(frozen=True, eq=False)
class SelectorScoreParams(_Frozen):
    """selector.py:129-156."""

    w1: object = ()
    b1: object = ()
    w2: object = ()
    b2: object = ()
    w3: object = ()
    b3: object = ()

    def __post_init__(self):
        self._set("w1", i8("score w1", self.w1, (3, 64, 32)))
        self._set("b1", i32("score b1", self.b1, (3, 32)))
        self._set("w2", i8("score w2", self.w2, (3, 32, 16)))
        self._set("b2", i32("score b2", self.b2, (3, 16)))
        self._set("w3", i8("score w3", self.w3, (3, 16, 2)))
        self._set("b3", i32("score b3", self.b3, (3, 2)))


@dataclass(frozen=True, eq=False)
class SelectorHeadWeightParams(_Frozen):
    """selector.py:159-174."""

    w1: object = ()
    b1: object = ()
    w2: object = ()
    b2: object = ()

    def __post_init__(self):
        self._set("w1", i8("head w1", self.w1, (3, 3)))
        self._set("b1", i32("head b1", self.b1, (3,)))
        self._set("w2", i8("head w2", self.w2, (3, 3)))
        self._set("b2", i32("head b2", self.b2, (3,)))


@dataclass(frozen=True, eq=False)
class SelectorParams(_Frozen):
    """selector.py:177-221 (activation/weight/logits_scale_exp are carried but,
    as in the golden model, unused by token_selector)."""

    local: SelectorLocalParams
    score: SelectorScoreParams
    head_weight: SelectorHeadWeightParams
    heads: int = 3
    head_dim: int = 64
    local_dim: int = 32
    activation_scale_exp: int = -7
    weight_scale_exp: int = -7
    logits_scale_exp: int = -7
    in_scale_exp: int = -7
    local_w_scale_exp: int = -7
    local_out_scale_exp: int = -7
    concat_out_scale_exp: int = -7
    score_w1_scale_exp: int = -7
    score_w2_scale_exp: int = -7
    score_w3_scale_exp: int = -7
    h1_out_scale_exp: int = -7
    h2_out_scale_exp: int = -7
    logits_out_scale_exp: int = -7
    stats_out_scale_exp: int = -7
    hw_w1_scale_exp: int = -7
    hw_hidden_out_scale_exp: int = -7
    hw_w2_scale_exp: int = -7

    def __post_init__(self):
        if self.heads != 3 or self.head_dim != 64 or self.local_dim != 32:
            raise ValueError("selector dims must be 3 heads / 64 / 32")
        if not isinstance(self.local, SelectorLocalParams):
            raise TypeError("local must be SelectorLocalParams")
        if not isinstance(self.score, SelectorScoreParams):
            raise TypeError("score must be SelectorScoreParams")
        if not isinstance(self.head_weight, SelectorHeadWeightParams):
            raise TypeError("head_weight must be SelectorHeadWeightParams")
        self._ints()


@dataclass(frozen=True, eq=False)
class HeatViTParams(_Frozen):
    """model.py:24-46."""

    patch: PatchParams
    blocks: tuple
    selectors: tuple
    final_gamma: object
    final_beta: object
    head_w: object
    head_b: object
    final_gamma_scale_exp: int = -6
    final_beta_scale_exp: int = -7
    final_ln_out_scale_exp: int = -7
    head_w_scale_exp: int = -7
    selector_blocks: tuple = (4, 7, 10)

    def __post_init__(self):
        if len(self.blocks) != 12:
            raise ValueError("HeatViT-T needs exactly 12 blocks")
        if len(self.selectors) != len(self.selector_blocks):
            raise ValueError("selector count must match selector_blocks")
        self._ints()
        self._set("blocks", tuple(self.blocks))
        self._set("selectors", tuple(self.selectors))
        self._set("selector_blocks", tuple(int(b) for b in self.selector_blocks))
        self._set("final_gamma", i8("final_gamma", self.final_gamma, (192,)))
        self._set("final_beta", i8("final_beta", self.final_beta, (192,)))
        self._set("head_w", i8("head_w", self.head_w, (192, 1000)))
        self._set("head_b", i32("head_b", self.head_b, (1000,)))


# ----------------------------------------------------------------------------
# Conversion from the golden dataclasses (duck typing on field names)
# ----------------------------------------------------------------------------

def _copy_fields(cls, obj, **over):
    kwargs = {}
    for f in fields(cls):
        if f.name in over:
            kwargs[f.name] = over[f.name]
        elif hasattr(obj, f.name):
            kwargs[f.name] = getattr(obj, f.name)
    return cls(**kwargs)


def patch_from(obj):
    return obj if isinstance(obj, PatchParams) else _copy_fields(PatchParams, obj)


def mhsa_from(obj):
    return obj if isinstance(obj, MhsaParams) else _copy_fields(MhsaParams, obj)


def ffn_from(obj):
    return obj if isinstance(obj, FfnParams) else _copy_fields(FfnParams, obj)


def block_from(obj):
    if isinstance(obj, BlockParams):
        return obj
    return BlockParams(mhsa=mhsa_from(obj.mhsa), ffn=ffn_from(obj.ffn))


def selector_from(obj):
    if isinstance(obj, SelectorParams):
        return obj
    return _copy_fields(
        SelectorParams, obj,
        local=_copy_fields(SelectorLocalParams, obj.local),
        score=_copy_fields(SelectorScoreParams, obj.score),
        head_weight=_copy_fields(SelectorHeadWeightParams, obj.head_weight),
    )


def from_reference(obj):
    """Convert a golden ``HeatViTParams`` (or this module's) into this module's."""
    if isinstance(obj, HeatViTParams):
        return obj
    for attr in ("patch", "blocks", "selectors", "head_w"):
        if not hasattr(obj, attr):
            raise TypeError("params must be HeatViTParams")
    return _copy_fields(
        HeatViTParams, obj,
        patch=patch_from(obj.patch),
        blocks=tuple(block_from(b) for b in obj.blocks),
        selectors=tuple(selector_from(s) for s in obj.selectors),
    )


def to_reference(params, ref_module):
    """Build golden dataclasses (tuples of ints) from numpy-backed params.

    ``ref_module`` is a namespace exposing the golden classes; used only by the
    fixture generator and tests that run next to the reference.
    """
    def tl(a):
        a = np.asarray(a)
        return tuple(tl(x) for x in a) if a.ndim > 1 else tuple(int(v) for v in a)

    def conv(obj, cls_name, **over):
        cls = getattr(ref_module, cls_name)
        kwargs = {}
        for f in fields(type(obj)):
            if f.name in over:
                kwargs[f.name] = over[f.name]
                continue
            v = getattr(obj, f.name)
            kwargs[f.name] = tl(v) if isinstance(v, np.ndarray) else v
        return cls(**kwargs)

    patch = conv(params.patch, "PatchParams")
    blocks = tuple(
        ref_module.BlockParams(mhsa=conv(b.mhsa, "MhsaParams"), ffn=conv(b.ffn, "FfnParams"))
        for b in params.blocks)
    selectors = tuple(
        conv(s, "SelectorParams",
             local=conv(s.local, "SelectorLocalParams"),
             score=conv(s.score, "SelectorScoreParams"),
             head_weight=conv(s.head_weight, "SelectorHeadWeightParams"))
        for s in params.selectors)
    return conv(params, "HeatViTParams", patch=patch, blocks=blocks, selectors=selectors)


# ----------------------------------------------------------------------------
# Packing into the C ABI struct
# ----------------------------------------------------------------------------

def _ptr(arr, ctype):
    return arr.ctypes.data_as(C.POINTER(ctype))


def selector_schedule(params):
    """model.py:81-87: the i-th block (in order 1..12) listed in selector_blocks
    runs selectors[i]."""
    sched = [-1] * 12
    wanted = set(params.selector_blocks)
    n = 0
    for b in range(1, 13):
        if b in wanted:
            if n >= len(params.selectors):
                break
            sched[b - 1] = n
            n += 1
    return sched


class _Keep(list):
    """Arrays referenced by a packed struct (kept alive with it)."""

    def p8(self, a):
        a = np.ascontiguousarray(a, dtype=np.int8)
        self.append(a)
        return _ptr(a, C.c_int8)

    def p32(self, a):
        a = np.ascontiguousarray(a, dtype=np.int32)
        self.append(a)
        return _ptr(a, C.c_int32)


def pack_patch(pp, keep):
    pp = patch_from(pp)
    return abi.HvPatchParams(
        keep.p8(pp.patch_weight), keep.p32(pp.patch_bias), keep.p8(pp.cls), keep.p8(pp.pos),
        pp.image_scale_exp, pp.weight_scale_exp, pp.activation_scale_exp,
        pp.tokens_scale_exp, pp.cls_scale_exp, pp.pos_scale_exp)


_MHSA_SCALES = ("x_scale_exp", "gamma1_scale_exp", "beta1_scale_exp", "ln1_out_scale_exp",
                "wqkv_scale_exp", "qkv_out_scale_exp", "score_scale_exp", "prob_scale_exp",
                "context_out_scale_exp", "wproj_scale_exp", "msa_out_scale_exp")
_FFN_SCALES = ("gamma2_scale_exp", "beta2_scale_exp", "ln2_out_scale_exp", "w1_scale_exp",
               "hidden_out_scale_exp", "w2_scale_exp", "ffn_out_scale_exp", "out_scale_exp")


def pack_block(b, keep, sb=None):
    b = block_from(b)
    m, f = b.mhsa, b.ffn
    sb = abi.HvBlockParams() if sb is None else sb
    sb.ln1_gamma, sb.ln1_beta = keep.p8(m.ln_gamma), keep.p8(m.ln_beta)
    sb.wqkv, sb.bqkv = keep.p8(m.wqkv), keep.p32(m.bqkv)
    sb.wproj, sb.bproj = keep.p8(m.wproj), keep.p32(m.bproj)
    sb.ln2_gamma, sb.ln2_beta = keep.p8(f.ln_gamma), keep.p8(f.ln_beta)
    sb.w1, sb.b1 = keep.p8(f.w1), keep.p32(f.b1)
    sb.w2, sb.b2 = keep.p8(f.w2), keep.p32(f.b2)
    for name in _MHSA_SCALES:
        setattr(sb, name, getattr(m, name))
    sb.ffn_x_scale_exp = f.x_scale_exp
    for name in _FFN_SCALES:
        setattr(sb, name, getattr(f, name))
    return sb


def pack_selector(sp, keep, ss=None):
    sp = selector_from(sp)
    ss = abi.HvSelectorParams() if ss is None else ss
    ss.local_w, ss.local_b = keep.p8(sp.local.w), keep.p32(sp.local.b)
    ss.score_w1, ss.score_b1 = keep.p8(sp.score.w1), keep.p32(sp.score.b1)
    ss.score_w2, ss.score_b2 = keep.p8(sp.score.w2), keep.p32(sp.score.b2)
    ss.score_w3, ss.score_b3 = keep.p8(sp.score.w3), keep.p32(sp.score.b3)
    ss.hw_w1, ss.hw_b1 = keep.p8(sp.head_weight.w1), keep.p32(sp.head_weight.b1)
    ss.hw_w2, ss.hw_b2 = keep.p8(sp.head_weight.w2), keep.p32(sp.head_weight.b2)
    for name in abi.SELECTOR_SCALE_FIELDS:
        setattr(ss, name, getattr(sp, name))
    return ss


class PackedParams:
    """An ``abi.HvParams`` struct plus the numpy arrays it points into."""

    def __init__(self, params):
        params = from_reference(params)
        if len(params.selectors) > abi.MAX_SELECTORS:
            raise ValueError("at most 12 selectors")
        self.params = params
        keep = _Keep()
        s = abi.HvParams()
        s.patch = pack_patch(params.patch, keep)
        for i, b in enumerate(params.blocks):
            pack_block(b, keep, s.blocks[i])
        sched = selector_schedule(params)
        for i in range(12):
            s.selector_before[i] = sched[i]
        s.num_selectors = len(params.selectors)
        for i, sp in enumerate(params.selectors):
            pack_selector(sp, keep, s.selectors[i])
        s.final_gamma, s.final_beta = keep.p8(params.final_gamma), keep.p8(params.final_beta)
        s.head_w, s.head_b = keep.p8(params.head_w), keep.p32(params.head_b)
        s.final_gamma_scale_exp = params.final_gamma_scale_exp
        s.final_beta_scale_exp = params.final_beta_scale_exp
        s.final_ln_out_scale_exp = params.final_ln_out_scale_exp
        s.head_w_scale_exp = params.head_w_scale_exp
        self.struct = s
        self._keep = keep
        self.num_selectors = len(params.selectors)
        self.used_selectors = sum(1 for v in sched if v >= 0)


def pack_params(params):
    return PackedParams(params)


def with_selectors(params, selectors, selector_blocks):
    """dataclasses.replace helper that keeps validation (model.py:42-46)."""
    return replace(params, selectors=tuple(selectors), selector_blocks=tuple(selector_blocks))
