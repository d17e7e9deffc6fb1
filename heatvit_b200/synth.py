"""Seeded synthetic parameters and images for the benchmark configurations.

Two generators:

* ``reference_seeded_params`` restates the reference's own deterministic
  synthetic model (verification/heatvit_ref/weights.py:167-374): one
  ``random.Random(20260815)`` stream in the fixed order patch -> 12 blocks ->
  3 selector bases -> final LN -> head, then per-stage selector calibration
  that re-seeds ``random.Random(20260815 + stage*1000 + attempt)`` for the
  last score layer and sets the keep/drop bias to the negative median logit
  difference (weights.py:281-327).  The calibration outcome (accepted attempt
  and median per stage) is an input here; ``calibrate_reference_selectors``
  searches for it given any token-selector implementation.

* ``baseline_params`` builds the benchmark model (same architecture, all
  weights int8 uniform in [-127, 127], int32 biases uniform in [-2^15, 2^15],
  per-tensor exponents in [-20, -8]) from ``numpy.random.default_rng(seed)``.
  The exponent of each GEMM/LN output is drawn from the range that keeps its
  int8 outputs unsaturated for these weight statistics, so every tensor in the
  chain carries signal; the chain is consistent (block n input = block n-1
  output, selector input = preceding block output).
"""

import random

import numpy as np

from .params import (
    BlockParams, FfnParams, HeatViTParams, MhsaParams, PatchParams, SelectorHeadWeightParams,
    SelectorLocalParams, SelectorParams, SelectorScoreParams,
)

SEED = 20260815
SELECTOR_ATTEMPTS = 256


# ----------------------------------------------------------------------------
# The reference's deterministic model (weights.py)
# ----------------------------------------------------------------------------

def _ri_matrix(rng, rows, cols, lo=-8, hi=7):
    r = rng.randint
    return [[r(lo, hi) for _ in range(cols)] for _ in range(rows)]


def _ri_vec(rng, cols, lo=-64, hi=63):
    r = rng.randint
    return [r(lo, hi) for _ in range(cols)]


def _gamma(rng, cols):
    return [min(127, max(0, 64 + rng.randint(-24, 24))) for _ in range(cols)]


def _beta(rng, cols):
    return [rng.randint(-4, 4) for _ in range(cols)]


def reference_seeded_image():
    """The reference's end-to-end image: random.Random(20260815), 150528 draws
    in [-128, 127] (verification/tests/test_model.py:14-16)."""
    rng = random.Random(SEED)
    return np.array([rng.randint(-128, 127) for _ in range(224 * 224 * 3)], np.int8)


def _reference_w3(stage, attempt):
    rng = random.Random(SEED + stage * 1000 + attempt)
    return [[[rng.randint(-8, 7) for _ in range(2)] for _ in range(16)] for _ in range(3)]


def reference_seeded_base():
    """All ordinary parameters of weights.build_params in stream order; the
    three selectors come back with b3 = 0 and w3 from the master stream."""
    rng = random.Random(SEED)
    patch = PatchParams(
        patch_weight=np.array(_ri_matrix(rng, 768, 192), np.int8),
        patch_bias=np.array(_ri_vec(rng, 192), np.int32),
        cls=np.array([rng.randint(-128, 127) for _ in range(192)], np.int8),
        pos=np.array([[rng.randint(-128, 127) for _ in range(192)] for _ in range(197)], np.int8),
        image_scale_exp=-7, weight_scale_exp=-7, activation_scale_exp=-7,
        cls_scale_exp=-7, pos_scale_exp=-7)
    blocks = []
    for _ in range(12):
        mhsa = MhsaParams(
            ln_gamma=np.array(_gamma(rng, 192), np.int8), ln_beta=np.array(_beta(rng, 192), np.int8),
            wqkv=np.array(_ri_matrix(rng, 192, 576), np.int8), bqkv=np.array(_ri_vec(rng, 576), np.int32),
            wproj=np.array(_ri_matrix(rng, 192, 192), np.int8), bproj=np.array(_ri_vec(rng, 192), np.int32),
            score_scale_exp=-17, prob_scale_exp=-8)
        ffn = FfnParams(
            ln_gamma=np.array(_gamma(rng, 192), np.int8), ln_beta=np.array(_beta(rng, 192), np.int8),
            w1=np.array(_ri_matrix(rng, 192, 768), np.int8), b1=np.array(_ri_vec(rng, 768), np.int32),
            w2=np.array(_ri_matrix(rng, 768, 192), np.int8), b2=np.array(_ri_vec(rng, 192), np.int32))
        blocks.append(BlockParams(mhsa=mhsa, ffn=ffn))
    bases = []
    for _ in range(3):
        def head_matrix(rows, cols):
            return np.array([_ri_matrix(rng, rows, cols, -64, 63) for _ in range(3)], np.int8)
        local = SelectorLocalParams(w=head_matrix(64, 32),
                                    b=np.array([_ri_vec(rng, 32) for _ in range(3)], np.int32))
        w1 = head_matrix(64, 32)
        b1 = np.array([_ri_vec(rng, 32) for _ in range(3)], np.int32)
        w2 = head_matrix(32, 16)
        b2 = np.array([_ri_vec(rng, 16) for _ in range(3)], np.int32)
        w3 = head_matrix(16, 2)
        score = SelectorScoreParams(w1=w1, b1=b1, w2=w2, b2=b2, w3=w3,
                                    b3=np.zeros((3, 2), np.int32))
        hw = SelectorHeadWeightParams(w1=np.ones((3, 3), np.int8), b1=np.zeros(3, np.int32),
                                      w2=np.eye(3, dtype=np.int8), b2=np.zeros(3, np.int32))
        bases.append(SelectorParams(local=local, score=score, head_weight=hw))
    final_gamma = np.array(_gamma(rng, 192), np.int8)
    final_beta = np.array(_beta(rng, 192), np.int8)
    head_w = np.array(_ri_matrix(rng, 192, 1000), np.int8)
    head_b = np.array(_ri_vec(rng, 1000), np.int32)
    return dict(patch=patch, blocks=tuple(blocks), bases=tuple(bases), final_gamma=final_gamma,
                final_beta=final_beta, head_w=head_w, head_b=head_b)


def _calibrated_selector(base, stage, attempt, median):
    from dataclasses import replace
    w3 = np.array(_reference_w3(stage, attempt), np.int8)
    b3 = np.array([[0, -int(median)] for _ in range(3)], np.int32)
    return replace(base, score=replace(base.score, w3=w3, b3=b3))


def reference_seeded_params(calibration, base=None):
    """weights.build_params with a known calibration outcome.

    ``calibration`` is ``[(attempt, median_logit_diff)] * 3`` (the fields of the
    reference's calibration summary, weights.py:314-324)."""
    base = reference_seeded_base() if base is None else base
    sels = tuple(_calibrated_selector(base["bases"][s], s + 1, a, m)
                 for s, (a, m) in enumerate(calibration))
    return HeatViTParams(patch=base["patch"], blocks=base["blocks"], selectors=sels,
                         final_gamma=base["final_gamma"], final_beta=base["final_beta"],
                         head_w=base["head_w"], head_b=base["head_b"])


def calibrate_reference_selectors(image, run_to_selector, selector_h2, token_selector, base=None):
    """Search the calibration outcome of weights.py:281-327.

    ``run_to_selector(params_so_far, image, stage)`` returns the stage input
    tokens and package flag, ``selector_h2(tokens, selector_params)`` the per
    head second hidden layer [3][C][16], and ``token_selector(tokens, pkg,
    selector_params)`` a dict with kept_normal / pruned_normal.  Any backend
    (the CUDA library, or a CPU implementation in tests) can be plugged in."""
    base = reference_seeded_base() if base is None else base
    outcome = []
    for stage in (1, 2, 3):
        params = reference_seeded_params(outcome + [(0, 0)] * (3 - len(outcome)), base)
        tokens, pkg = run_to_selector(params, image, stage)
        h2 = np.asarray(selector_h2(tokens, base["bases"][stage - 1]), np.int64)
        for attempt in range(SELECTOR_ATTEMPTS):
            w3 = np.array(_reference_w3(stage, attempt), np.int64)
            diffs = np.einsum("hck,hk->hc", h2, w3[:, :, 1] - w3[:, :, 0]).reshape(-1)
            if np.all(diffs == diffs[0]):
                continue
            median = int(np.sort(diffs)[diffs.size // 2])
            sel = _calibrated_selector(base["bases"][stage - 1], stage, attempt, median)
            res = token_selector(tokens, pkg, sel)
            if res["kept_normal"] >= 1 and res["pruned_normal"] >= 2:
                outcome.append((attempt, median))
                break
        else:
            raise RuntimeError(f"selector stage {stage} calibration failed")
    return outcome


# ----------------------------------------------------------------------------
# Benchmark configurations
# ----------------------------------------------------------------------------

EXP_LO, EXP_HI = -20, -8


def _w8(rng, *shape):
    return rng.integers(-127, 128, size=shape, dtype=np.int64).astype(np.int8)


def _b32(rng, *shape):
    return rng.integers(-(1 << 15), (1 << 15) + 1, size=shape, dtype=np.int64).astype(np.int32)


class _Exps:
    """Exponent draws for one parameter set."""

    def __init__(self, rng):
        self.rng = rng

    def free(self):
        return int(self.rng.integers(EXP_LO, EXP_HI + 1))

    def clamp(self, e):
        return int(min(EXP_HI, max(EXP_LO, e)))

    def gemm(self, a_exp, gain):
        """(weight_exp, out_exp) with out = a + w + gain, both inside the range."""
        lo = max(EXP_LO, a_exp + EXP_LO + gain)
        hi = min(EXP_HI, a_exp + EXP_HI + gain)
        if lo > hi:                                 # pick the nearest feasible pair
            w = EXP_HI if a_exp + EXP_HI + gain < EXP_LO else EXP_LO
            return w, self.clamp(a_exp + w + gain)
        out = int(self.rng.integers(lo, hi + 1))
        return out - a_exp - gain, out

    def gelu_gemm(self, a_exp, acc_log2):
        """Exponents for GEMM -> Q16 -> GELU -> int8: put the real GELU input
        near unit scale and the int8 output near 2^5."""
        w = self.clamp(-acc_log2 - a_exp + int(self.rng.integers(-1, 2)))
        real_log2 = acc_log2 + a_exp + w
        out = self.clamp(real_log2 - 1 - 5 + int(self.rng.integers(-1, 2)))
        return w, out

    def ln(self):
        g = int(self.rng.integers(EXP_LO, EXP_HI))
        out = self.clamp(g + 1)
        beta = self.clamp(out - int(self.rng.integers(1, 4)))
        return g, beta, out

    def near(self, a_exp, gain, target):
        """(weight_exp, out_exp) with out = a + w + gain as close to ``target``
        as the weight range allows."""
        w = self.clamp(target - a_exp - gain)
        return w, self.clamp(a_exp + w + gain)

    def join(self, *exps):
        """Residual output exponent: the coarser input, one step coarser when
        both branches sit at the same scale (their sum needs one more bit)."""
        top = max(exps)
        return self.clamp(top + (1 if sum(e == top for e in exps) > 1 else 0))


def baseline_params(seed=SEED, pruned=True, logits_out_exps=(-8, -8, -8), keep_bias=(0, 0, 0)):
    """The benchmark model of configs 0/3/4.

    ``keep_bias[s]`` is added to every head's keep logit bias b3[h][1] of
    selector s (the per-stage bias that sets the keep budget); ``pruned=False``
    gives the unpruned variant (no selectors, model.py:42-46)."""
    rng = np.random.default_rng(seed)
    E = _Exps(rng)
    img_e = E.free()
    pw_e, act_e = E.gemm(img_e, 12)
    pos_e = E.clamp(act_e + int(rng.integers(-1, 2)))
    cls_e = E.clamp(pos_e + int(rng.integers(-1, 2)))
    tok_e = E.join(act_e, pos_e, cls_e)
    patch = PatchParams(patch_weight=_w8(rng, 768, 192), patch_bias=_b32(rng, 192),
                        cls=_w8(rng, 192), pos=_w8(rng, 197, 192),
                        image_scale_exp=img_e, weight_scale_exp=pw_e, activation_scale_exp=act_e,
                        tokens_scale_exp=tok_e, cls_scale_exp=cls_e, pos_scale_exp=pos_e)
    x_e = tok_e
    blocks = []
    block_out_exps = []
    for _ in range(12):
        g1, b1e, l1 = E.ln()
        wq, q = E.gemm(l1, 10)
        ctx = q
        wp, m = E.near(ctx, 10, x_e + int(rng.integers(-1, 1)))
        y = E.join(x_e, m)
        g2, b2e, l2 = E.ln()
        w1e, h = E.gelu_gemm(l2, 15)
        w2e, f = E.near(h, 11, y + int(rng.integers(-1, 1)))
        z = E.join(y, f)
        mhsa = MhsaParams(ln_gamma=_w8(rng, 192), ln_beta=_w8(rng, 192),
                          wqkv=_w8(rng, 192, 576), bqkv=_b32(rng, 576),
                          wproj=_w8(rng, 192, 192), bproj=_b32(rng, 192),
                          x_scale_exp=x_e, gamma1_scale_exp=g1, beta1_scale_exp=b1e,
                          ln1_out_scale_exp=l1, wqkv_scale_exp=wq, qkv_out_scale_exp=q,
                          score_scale_exp=2 * q - 3, prob_scale_exp=-8,
                          context_out_scale_exp=ctx, wproj_scale_exp=wp, msa_out_scale_exp=m)
        ffn = FfnParams(ln_gamma=_w8(rng, 192), ln_beta=_w8(rng, 192),
                        w1=_w8(rng, 192, 768), b1=_b32(rng, 768),
                        w2=_w8(rng, 768, 192), b2=_b32(rng, 192),
                        x_scale_exp=y, gamma2_scale_exp=g2, beta2_scale_exp=b2e,
                        ln2_out_scale_exp=l2, w1_scale_exp=w1e, hidden_out_scale_exp=h,
                        w2_scale_exp=w2e, ffn_out_scale_exp=f, out_scale_exp=z)
        blocks.append(BlockParams(mhsa=mhsa, ffn=ffn))
        block_out_exps.append(z)
        x_e = z
    selectors = []
    for s, blk in enumerate((4, 7, 10)):
        in_e = block_out_exps[blk - 2]
        lw, lo = E.gelu_gemm(in_e, 14)
        s1, h1 = E.gelu_gemm(lo, 15)
        s2, h2 = E.gelu_gemm(h1, 14)
        s3 = E.clamp(logits_out_exps[s] - h2 - 10)
        hw1, hwh = E.gelu_gemm(in_e, 8)
        hw2 = E.free()
        b3 = _b32(rng, 3, 2)
        b3[:, 1] = np.clip(b3[:, 1].astype(np.int64) + int(keep_bias[s]), -(1 << 31), (1 << 31) - 1)
        sel = SelectorParams(
            local=SelectorLocalParams(w=_w8(rng, 3, 64, 32), b=_b32(rng, 3, 32)),
            score=SelectorScoreParams(w1=_w8(rng, 3, 64, 32), b1=_b32(rng, 3, 32),
                                      w2=_w8(rng, 3, 32, 16), b2=_b32(rng, 3, 16),
                                      w3=_w8(rng, 3, 16, 2), b3=b3),
            head_weight=SelectorHeadWeightParams(w1=_w8(rng, 3, 3), b1=_b32(rng, 3),
                                                 w2=_w8(rng, 3, 3), b2=_b32(rng, 3)),
            in_scale_exp=in_e, local_w_scale_exp=lw, local_out_scale_exp=lo,
            concat_out_scale_exp=lo, score_w1_scale_exp=s1, h1_out_scale_exp=h1,
            score_w2_scale_exp=s2, h2_out_scale_exp=h2, score_w3_scale_exp=s3,
            logits_out_scale_exp=logits_out_exps[s], stats_out_scale_exp=in_e,
            hw_w1_scale_exp=hw1, hw_hidden_out_scale_exp=hwh, hw_w2_scale_exp=hw2)
        selectors.append(sel)
    fg, fb, fo = E.ln()
    hw_e = E.clamp(-14 - fo - 2)
    params = HeatViTParams(
        patch=patch, blocks=tuple(blocks), selectors=tuple(selectors),
        final_gamma=_w8(rng, 192), final_beta=_w8(rng, 192),
        head_w=_w8(rng, 192, 1000), head_b=_b32(rng, 1000),
        final_gamma_scale_exp=fg, final_beta_scale_exp=fb, final_ln_out_scale_exp=fo,
        head_w_scale_exp=hw_e)
    if not pruned:
        from .params import with_selectors
        params = with_selectors(params, (), ())
    return params


def baseline_images(seed, count, first=0):
    """Seeded uniform int8 NHWC images.  Image i draws its own value range
    [lo_i, hi_i] (so images differ in brightness and contrast) and then the
    150528 pixels uniformly inside it; image i depends only on (seed, i)."""
    out = np.empty((count, 224 * 224 * 3), np.int8)
    for j in range(count):
        rng = np.random.default_rng([seed, first + j])
        a, b = sorted(int(v) for v in rng.integers(-128, 128, size=2))
        if b - a < 16:
            a, b = max(-128, a - 8), min(127, b + 8)
        out[j] = rng.integers(a, b + 1, size=224 * 224 * 3, dtype=np.int64).astype(np.int8)
    return out


def p2_float_images(seed, count, input_exp, first=0):
    """Seeded float32 images [count, 3, 224, 224] (CHW, the layout of the P2
    tooling's normalised image tensors) for a model whose input exponent is
    ``input_exp``: values mostly inside the int8 range after scaling by
    2^-input_exp, with about 1% exact half-way values (rounding ties) and 0.2%
    values far outside the range (saturation).  Image i depends only on
    (seed, i)."""
    out = np.empty((count, 3, 224, 224), np.float32)
    step = np.float32(2.0 ** input_exp)
    for j in range(count):
        rng = np.random.default_rng([seed, 7, first + j])
        x = rng.normal(0.0, 40.0, (3, 224, 224))
        flat = x.reshape(-1)
        ties = rng.choice(flat.size, flat.size // 100, replace=False)
        flat[ties] = rng.integers(-140, 140, ties.size) + 0.5
        far = rng.choice(flat.size, flat.size // 500, replace=False)
        flat[far] = rng.choice([-1.0, 1.0], far.size) * rng.uniform(130.0, 4000.0, far.size)
        out[j] = (x * step).astype(np.float32)
    return out


# Calibrated per-stage keep-logit biases of ``baseline_params`` (seed ->
# keep_bias): chosen by ``calibrate_keep_bias`` so the mean output token counts
# of the three selectors over ``baseline_images(seed, 64)`` sit at the target
# budget 197 -> 88 -> 45 -> 32.  They come from the first version of the image
# generator; over the current images the same search returns (-23305, -895,
# 10084), a few units away.  The committed values stay: the golden fixtures pin
# the parameters they give.
BASELINE_KEEP_BIAS = {
    20260815: (-23308, -909, 10050),
}

TARGET_COUNTS = (88, 45, 32)


def calibrate_keep_bias(seed, infer_counts, images=64, targets=TARGET_COUNTS, lo=-(1 << 22),
                        hi=(1 << 22), make=None, stages=(0, 1, 2), **kw):
    """Bisect keep_bias stage by stage so the mean selector output count over
    ``baseline_images(seed, images)`` is as close as possible to ``targets``.

    ``infer_counts(params, images) -> counts [B, 4]`` may be any backend;
    ``make(bias) -> params`` builds the model for a bias triple (default:
    ``baseline_params``); only ``stages`` are calibrated."""
    imgs = baseline_images(seed, images)
    if make is None:
        def make(bias):
            return baseline_params(seed, True, keep_bias=bias, **kw)
    bias = [0, 0, 0]
    for s in stages:
        a, b = lo, hi
        best = None
        while a <= b:
            mid = (a + b) // 2
            bias[s] = mid
            mean = float(np.mean(infer_counts(make(bias), imgs)[:, s + 1]))
            if best is None or abs(mean - targets[s]) < abs(best[1] - targets[s]):
                best = (mid, mean)
            if mean < targets[s]:
                a = mid + 1
            else:
                b = mid - 1
        bias[s] = best[0]
    return tuple(bias)


def config_params(seed=SEED, pruned=True):
    """The benchmark model with its calibrated keep biases (config 4)."""
    return baseline_params(seed, pruned=pruned, keep_bias=BASELINE_KEEP_BIAS.get(seed, (0, 0, 0)))


# ----------------------------------------------------------------------------
# Config 3: a ragged batch in which some images have a zero package denominator
# ----------------------------------------------------------------------------
#
# The package denominator of finalize_tokens (selector.py:421-500) is the sum of
# the fused keep scores of the pruned tokens, and it is zero only when every one
# of them scores exactly 0.  A keep score softmax_selector([drop, keep])[1] is 0
# only when the logit gap reaches 16 * 45426 in Q16 (the exp term shifts out),
# i.e. (drop - keep) * 2^(logits_exp + 16) >= 726816.  Int8 logits differ by at
# most 255, so no logits exponent <= -5 (in particular none in [-20, -8]) can
# produce it.  Config 3 therefore gives its first selector logits at 2^-4 and
# lets head 0 alone vote:
#
# * head weights: head_weight.w2 = 0 and b2 = (+2^30, -2^30, -2^30) at
#   exponents -8/-8, so PLAN gives every candidate the weights (1.0, 0, 0) and
#   fuse_head_scores returns head 0's score unchanged;
# * head 0's drop logit saturates at +127 (w3[0, :, 0] = 0, b3[0][0] = 2^30);
# * head 0's keep logit is one seeded int8 column over the 16 h2 features plus a
#   keep bias, at score_w3 exponent logits_exp - h2_exp + shift.
#
# A candidate is kept when its keep logit saturates at +127 too (score 0.5,
# inclusive threshold) and scores exactly 0 when the keep logit is <= -51; an
# image has a zero package denominator when none of its pruned candidates falls
# in between.  The column attempt, shift and bias are searched (seeded, like the
# reference's per-stage calibration, weights.py:281-327) for an output count
# near 88 with the budget's spread and a zero-denominator rate of a few percent;
# selectors 2 and 3 then get keep biases recalibrated for 45 and 32.

ZERO_DEN_LOGITS_EXP = -4


def zero_den_column(seed, attempt):
    """Head 0's keep-logit column (16 int8) for calibration attempt ``attempt``."""
    return np.random.default_rng([seed, 3, attempt]).integers(-127, 128, 16).astype(np.int8)


def zero_den_selector(sel, column, shift, keep_bias):
    """``sel`` rebuilt as config 3's first selector (see above)."""
    from dataclasses import replace
    w3 = np.array(sel.score.w3, np.int8, copy=True)
    b3 = np.array(sel.score.b3, np.int64, copy=True)
    w3[0, :, 0] = 0
    w3[0, :, 1] = column
    b3[0, 0] = 1 << 30
    b3[0, 1] = keep_bias
    hw = replace(sel.head_weight, w2=np.zeros((3, 3), np.int8),
                 b2=np.array([1 << 30, -(1 << 30), -(1 << 30)], np.int32))
    return replace(sel, score=replace(sel.score, w3=w3, b3=b3.astype(np.int32)), head_weight=hw,
                   hw_w2_scale_exp=-8, hw_hidden_out_scale_exp=-8,
                   logits_out_scale_exp=ZERO_DEN_LOGITS_EXP,
                   score_w3_scale_exp=ZERO_DEN_LOGITS_EXP - sel.h2_out_scale_exp + shift)


def config3_from(seed, attempt, shift, keep_bias, later_keep_bias):
    """Config-3 parameters for explicit calibration values."""
    from dataclasses import replace
    base = baseline_params(seed, True, keep_bias=(0,) + tuple(later_keep_bias))
    first = zero_den_selector(base.selectors[0], zero_den_column(seed, attempt), shift, keep_bias)
    return replace(base, selectors=(first,) + tuple(base.selectors[1:]))


# seed -> (attempt, shift, keep_bias of selector 1, keep biases of selectors 2/3),
# found by tests/golden/calibrate_config3.py over baseline_images(seed, 256).
CONFIG3_CALIBRATION = {
    20260815: (172, 1, 5113, (-703, 9635)),
}


def config3_params(seed=SEED):
    """Config 3: the benchmark model with the zero-denominator first selector."""
    if seed not in CONFIG3_CALIBRATION:
        raise KeyError(f"no config-3 calibration for seed {seed}")
    attempt, shift, kb, later = CONFIG3_CALIBRATION[seed]
    return config3_from(seed, attempt, shift, kb, later)
