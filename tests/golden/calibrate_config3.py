#!/usr/bin/env python3
"""Search the config-3 calibration of heatvit_b200.synth (CONFIG3_CALIBRATION).

Config 3's first selector lets head 0 alone vote, with a saturated drop logit
and a seeded keep-logit column at logits exponent -4 (synth.zero_den_selector).
For each seeded column attempt and shift, the keep bias is bisected so the mean
first-selector output count over the first 64 images is 88; the attempt whose
output-count spread over 256 images is closest to the budget's +-20, among
those whose zero-package-denominator rate lies in [4%, 15%], is kept.  Then the
keep biases of selectors 2 and 3 are bisected for 45 and 32, and the whole
model is checked on 256 images.  The oracle (CPU restatement) is the backend.

    python tests/golden/calibrate_config3.py [--seed 20260815]
"""

import argparse
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "oracle"))

import numpy as np  # noqa: E402


def _stage1_inputs(seed, first, count):
    import hv_oracle as O
    from heatvit_b200 import synth
    params = synth.config_params(seed, pruned=True)
    imgs = synth.baseline_images(seed, count, first=first)
    out = []
    for i in range(count):
        x = O.patch_embedding(imgs[i], params.patch)
        for b in range(3):
            x, _, _ = O.transformer_block(x, params.blocks[b])
        out.append(x)
    return out


def head0_h2(p, x):
    """Head 0's 16 score features per candidate (selector.py:253-355)."""
    import hv_oracle as O
    cand = np.asarray(x, np.int8)[1:]
    c = cand.shape[0]
    loc = O.gelu_chain_array(O.gemm(cand[:, :64], p.local.w[0], p.local.b[0], False),
                             p.in_scale_exp + p.local_w_scale_exp, p.local_out_scale_exp)
    glob = np.array([max(-128, min(127, O.round_div(int(v), c))) for v in loc.astype(np.int64).sum(0)], np.int8)
    lg = np.concatenate([loc, np.tile(glob, (c, 1))], 1)
    h1 = O.gelu_chain_array(O.gemm(lg, p.score.w1[0], p.score.b1[0], False),
                            p.concat_out_scale_exp + p.score_w1_scale_exp, p.h1_out_scale_exp)
    h2 = O.gelu_chain_array(O.gemm(h1, p.score.w2[0], p.score.b2[0], False),
                            p.h1_out_scale_exp + p.score_w2_scale_exp, p.h2_out_scale_exp)
    return h2.astype(np.int64)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--seed", type=int, default=20260815)
    ap.add_argument("--attempts", type=int, default=256)
    args = ap.parse_args()
    import multiprocessing as mp
    import hv_oracle as O
    from heatvit_b200 import synth

    seed, n_img = args.seed, 256
    with mp.get_context("spawn").Pool(min(8, os.cpu_count() or 1)) as pool:
        parts = pool.starmap(_stage1_inputs, [(seed, f, 32) for f in range(0, n_img, 32)])
    xs = [x for part in parts for x in part]
    sel0 = synth.config_params(seed, pruned=True).selectors[0]
    feats = [head0_h2(sel0, x) for x in xs]
    L = synth.ZERO_DEN_LOGITS_EXP
    hs = np.array([O.softmax_selector([O.requant(127, L, -16, 24), O.requant(v, L, -16, 24)])[1]
                   for v in range(-128, 128)])
    kept_t, zero_t = hs >= 32768, hs == 0

    def stats(col, shift, kb, images):
        cnt, zd = [], 0
        for h2 in feats[:images]:
            acc = h2 @ col.astype(np.int64) + kb
            l1 = np.clip(acc << shift, -128, 127) + 128
            kept = kept_t[l1]
            pruned = ~kept
            cnt.append(1 + kept.sum() + (1 if pruned.any() else 0))
            zd += bool(pruned.any() and zero_t[l1[pruned]].all())
        return float(np.mean(cnt)), float(np.std(cnt)), zd / images

    best = None
    for attempt in range(args.attempts):
        col = synth.zero_den_column(seed, attempt)
        for shift in (0, 1, 2):
            a, b, fit = -(1 << 20), 1 << 20, None
            while a <= b:
                mid = (a + b) // 2
                m = stats(col, shift, mid, 64)[0]
                if fit is None or abs(m - 88) < abs(fit[1] - 88):
                    fit = (mid, m)
                if m < 88:
                    a = mid + 1
                else:
                    b = mid - 1
            m, sd, zd = stats(col, shift, fit[0], n_img)
            if 0.04 <= zd <= 0.15 and abs(m - 88) <= 2:
                key = (abs(sd - 20), attempt, shift)
                if best is None or key < best[0]:
                    best = (key, attempt, shift, fit[0], m, sd, zd)
    _, attempt, shift, kb, m, sd, zd = best
    print(f"selector 1: attempt {attempt} shift {shift} keep_bias {kb}: mean {m:.1f} sd {sd:.1f} "
          f"zero-den {zd:.3f} (numpy model)", flush=True)

    def counts(params, imgs):
        return O.infer_batch(params, imgs, threads=0)["counts"]

    later = synth.calibrate_keep_bias(
        seed, counts, make=lambda bias: synth.config3_from(seed, attempt, shift, kb, bias[1:]), stages=(1, 2))
    params = synth.config3_from(seed, attempt, shift, kb, later[1:])
    res = O.infer_batch(params, synth.baseline_images(seed, n_img), threads=0)
    c = res["counts"]
    print("counts mean", c.mean(0).round(1).tolist(), "sd", c.std(0).round(1).tolist())
    print("package-denominator-zero images:", int(((res["warnings"] & 2) != 0).sum()), "of", n_img)
    print(f"CONFIG3_CALIBRATION[{seed}] = ({attempt}, {shift}, {kb}, {tuple(later[1:])})")


if __name__ == "__main__":
    main()
