"""ctypes mirror of include/heatvit_b200.h (struct layouts and constants).

The C ABI takes plain pointers; this module only describes the structs so the
host wrappers can fill them from numpy arrays.  Field order must match the
header exactly.
"""

import ctypes as C

IMAGE_BYTES = 224 * 224 * 3
TOKENS = 197
EMBED = 192
CLASSES = 1000
BLOCKS = 12
MAX_SELECTORS = 12
LOGIT_SCALE_EXP = -14
CKPT_SLOTS = 26
CKPT_PATCH = 0
CKPT_FINAL_LN = 25


def ckpt_block(b):
    return b


def ckpt_selector(s):
    return 12 + s


HV_OK = 0
HV_ERR_VALUE = 1
HV_ERR_TYPE = 2
HV_ERR_OVERFLOW = 3
HV_ERR_CUDA = 4
HV_ERR_NOMEM = 5
HV_ERR_STATE = 6

WARN_HEAD_DEN_ZERO = 1
WARN_PACKAGE_DEN_ZERO = 2
WARN_LN_NEG_VARIANCE = 4

_p8 = C.POINTER(C.c_int8)
_p32 = C.POINTER(C.c_int32)


class HvPatchParams(C.Structure):
    _fields_ = [
        ("weight", _p8), ("bias", _p32), ("cls", _p8), ("pos", _p8),
        ("image_scale_exp", C.c_int32), ("weight_scale_exp", C.c_int32),
        ("activation_scale_exp", C.c_int32), ("tokens_scale_exp", C.c_int32),
        ("cls_scale_exp", C.c_int32), ("pos_scale_exp", C.c_int32),
    ]


BLOCK_SCALE_FIELDS = (
    "x_scale_exp", "gamma1_scale_exp", "beta1_scale_exp", "ln1_out_scale_exp",
    "wqkv_scale_exp", "qkv_out_scale_exp", "score_scale_exp", "prob_scale_exp",
    "context_out_scale_exp", "wproj_scale_exp", "msa_out_scale_exp",
    "ffn_x_scale_exp", "gamma2_scale_exp", "beta2_scale_exp", "ln2_out_scale_exp",
    "w1_scale_exp", "hidden_out_scale_exp", "w2_scale_exp", "ffn_out_scale_exp",
    "out_scale_exp",
)


class HvBlockParams(C.Structure):
    _fields_ = [
        ("ln1_gamma", _p8), ("ln1_beta", _p8),
        ("wqkv", _p8), ("bqkv", _p32),
        ("wproj", _p8), ("bproj", _p32),
        ("ln2_gamma", _p8), ("ln2_beta", _p8),
        ("w1", _p8), ("b1", _p32),
        ("w2", _p8), ("b2", _p32),
    ] + [(name, C.c_int32) for name in BLOCK_SCALE_FIELDS]


SELECTOR_SCALE_FIELDS = (
    "in_scale_exp", "local_w_scale_exp", "local_out_scale_exp", "concat_out_scale_exp",
    "score_w1_scale_exp", "score_w2_scale_exp", "score_w3_scale_exp",
    "h1_out_scale_exp", "h2_out_scale_exp", "logits_out_scale_exp",
    "stats_out_scale_exp", "hw_w1_scale_exp", "hw_hidden_out_scale_exp", "hw_w2_scale_exp",
)


class HvSelectorParams(C.Structure):
    _fields_ = [
        ("local_w", _p8), ("local_b", _p32),
        ("score_w1", _p8), ("score_b1", _p32),
        ("score_w2", _p8), ("score_b2", _p32),
        ("score_w3", _p8), ("score_b3", _p32),
        ("hw_w1", _p8), ("hw_b1", _p32),
        ("hw_w2", _p8), ("hw_b2", _p32),
    ] + [(name, C.c_int32) for name in SELECTOR_SCALE_FIELDS]


class HvParams(C.Structure):
    _fields_ = [
        ("patch", HvPatchParams),
        ("blocks", HvBlockParams * BLOCKS),
        ("selector_before", C.c_int32 * BLOCKS),
        ("num_selectors", C.c_int32),
        ("selectors", HvSelectorParams * MAX_SELECTORS),
        ("final_gamma", _p8), ("final_beta", _p8),
        ("head_w", _p8), ("head_b", _p32),
        ("final_gamma_scale_exp", C.c_int32), ("final_beta_scale_exp", C.c_int32),
        ("final_ln_out_scale_exp", C.c_int32), ("head_w_scale_exp", C.c_int32),
    ]


class HvSelectorSummary(C.Structure):
    _fields_ = [
        ("input_tokens", C.c_int32), ("output_tokens", C.c_int32),
        ("kept_normal", C.c_int32), ("pruned_normal", C.c_int32),
        ("package_present", C.c_int32), ("warnings", C.c_int32),
    ]


SUMMARY_FIELDS = ("input_tokens", "output_tokens", "kept_normal", "pruned_normal",
                  "package_present", "warnings")
