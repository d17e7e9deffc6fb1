"""Model-level parity on the GPU: the fused pipeline (patch, blocks, selectors,
ragged compaction, head) against golden-model fixtures and the CPU oracle,
bit-exact on logits, token counts, selector summaries and checkpoints."""

import numpy as np
import pytest

from conftest import golden_ckpt, load_golden, slot_of

pytestmark = pytest.mark.gpu


def _params_images(tag_file, tag):
    from heatvit_b200 import synth
    g = load_golden(tag_file)
    seed, images, pruned = int(g[f"{tag}_seed"]), int(g[f"{tag}_images"]), bool(g[f"{tag}_pruned"])
    return g, synth.config_params(seed, pruned=pruned), synth.baseline_images(seed, images)


def _check_result(res, g, prefix):
    ck, logits, summ = golden_ckpt(g, prefix)
    assert res.output_scale_exp == -14
    np.testing.assert_array_equal(np.array(res.logits, np.int32), logits)
    for key, rows in ck.items():
        np.testing.assert_array_equal(np.array(res.checkpoints[key], np.int8).reshape(-1, 192), rows, err_msg=key)
    got = np.array([[s[f] for f in ("input_tokens", "output_tokens", "kept_normal", "pruned_normal",
                                    "package_present")] for s in res.selector_summary], np.int32).reshape(-1, 5)
    np.testing.assert_array_equal(got, summ)


def test_seeded_reference_model(cuda):
    from heatvit_b200 import synth
    from heatvit_b200.model import HeatViTModel
    g = load_golden("golden_seeded.npz")
    calib = [tuple(int(v) for v in row) for row in g["seeded_calibration"]]
    res = HeatViTModel().infer(synth.reference_seeded_image(), synth.reference_seeded_params(calib))
    _check_result(res, g, "seeded")
    assert list(res.logits[:8]) == [-762, 1676, -112, -2544, -389, -1228, 2398, 1778]


@pytest.mark.parametrize("name,tag", [("golden_baseline.npz", "pruned"), ("golden_unpruned.npz", "unpruned")])
def test_benchmark_model_vs_golden(cuda, name, tag):
    from heatvit_b200.model import HeatViTModel
    g, params, imgs = _params_images(name, tag)
    for i in range(imgs.shape[0]):
        _check_result(HeatViTModel().infer(imgs[i], params), g, f"{tag}_{i}")


def _oracle_batch(oracle, params, imgs):
    return oracle.infer_batch(params, imgs)


def _compare_batch(out, ref, ns):
    np.testing.assert_array_equal(out["logits"], ref["logits"])
    np.testing.assert_array_equal(out["token_counts"], ref["counts"])
    np.testing.assert_array_equal(out["summary"], ref["summary"])
    np.testing.assert_array_equal(out["warnings"], ref["warnings"])


def test_config3_batch256_bit_exact(cuda, oracle):
    """Config 3: pruned, batch 256 on one GPU, every image against the oracle;
    at least 1% of the images take the zero-package-denominator fallback."""
    from heatvit_b200 import synth
    from heatvit_b200.model import HeatViTModel
    params = synth.config3_params(synth.SEED)
    imgs = synth.baseline_images(synth.SEED, 256)
    out = HeatViTModel().infer_batch(imgs, params)
    ref = _oracle_batch(oracle, params, imgs)
    _compare_batch(out, ref, 3)
    counts = out["token_counts"]
    assert counts[:, 0].min() == 197 and counts[:, 1].std() > 5  # ragged after the selectors
    assert ((np.asarray(out["warnings"]) & 2) != 0).sum() >= 0.01 * 256


def test_config4_pruned_sample_bit_exact(cuda, oracle):
    """The pruned benchmark model without the config-3 selector (calibrated
    keep biases on all three selectors), batch 96."""
    from heatvit_b200 import synth
    from heatvit_b200.model import HeatViTModel
    params = synth.config_params(synth.SEED, pruned=True)
    imgs = synth.baseline_images(synth.SEED, 96)
    out = HeatViTModel().infer_batch(imgs, params)
    _compare_batch(out, _oracle_batch(oracle, params, imgs), 3)


def test_unpruned_batch_bit_exact(cuda, oracle):
    from heatvit_b200 import synth
    from heatvit_b200.model import HeatViTModel
    params = synth.config_params(synth.SEED, pruned=False)
    imgs = synth.baseline_images(synth.SEED, 24, first=1000)
    out = HeatViTModel().infer_batch(imgs, params)
    _compare_batch(out, _oracle_batch(oracle, params, imgs), 0)


def test_checkpoints_batch_vs_oracle(cuda, oracle):
    from heatvit_b200 import synth
    from heatvit_b200.model import HeatViTModel
    params = synth.config_params(synth.SEED, pruned=True)
    imgs = synth.baseline_images(synth.SEED, 6, first=300)
    out = HeatViTModel().infer_batch(imgs, params, checkpoints=True)
    for i in range(imgs.shape[0]):
        r = oracle.infer(params, imgs[i])
        np.testing.assert_array_equal(out["checkpoint_rows"][i], r["checkpoint_rows"])
        for s in range(26):
            n = r["checkpoint_rows"][s]
            np.testing.assert_array_equal(out["checkpoints"][i][s][:n], r["checkpoints"][s][:n], err_msg=f"slot {s}")


def test_batch_invariance_full_size(cuda):
    """Size-independent property at the benchmark's full per-GPU batch (1024):
    the batched result equals the concatenation of sub-batch results."""
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    params = synth.config3_params(synth.SEED)
    eng = Engine(params)
    imgs = torch.from_numpy(synth.baseline_images(synth.SEED, 1024, first=5000)).cuda()
    full = eng.infer(imgs)
    parts = [eng.infer(imgs[a:a + 256]) for a in range(0, 1024, 256)]
    for key in ("logits", "token_counts", "summary", "warnings"):
        assert torch.equal(full[key], torch.cat([p[key] for p in parts]))


def test_full_size_sample_vs_oracle(cuda, oracle):
    """Batch 1024 on the device (the benchmark's per-GPU batch); a seeded sample of
    256 of its images plus every zero-package-denominator image against the oracle."""
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    params = synth.config3_params(synth.SEED)
    imgs = synth.baseline_images(synth.SEED, 1024, first=9000)
    eng = Engine(params)
    out = eng.infer(torch.from_numpy(imgs).cuda())
    assert eng.device_error() == 0
    warn = out["warnings"].cpu().numpy()
    zero_den = np.nonzero(warn & 2)[0]
    assert zero_den.size >= 10                                  # >= 1% of the batch
    idx = np.union1d(np.random.default_rng(1).choice(1024, 256, replace=False), zero_den)
    ref = oracle.infer_batch(params, imgs[idx])
    np.testing.assert_array_equal(out["logits"].cpu().numpy()[idx], ref["logits"])
    np.testing.assert_array_equal(out["token_counts"].cpu().numpy()[idx], ref["counts"])
    np.testing.assert_array_equal(warn[idx], ref["warnings"])


def test_host_entry_matches_device_entry(cuda):
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    params = synth.config3_params(synth.SEED)
    eng = Engine(params)
    n = 1400                                                   # chunks of 512, 512 and 376 images, two workspaces
    imgs = synth.baseline_images(synth.SEED, n, first=77)
    dev = eng.infer(torch.from_numpy(imgs).cuda())
    ns = eng.num_selectors
    pinned = torch.empty(imgs.shape, dtype=torch.int8, pin_memory=True)
    pinned.numpy()[:] = imgs
    pinned_logits = torch.empty((n, 1000), dtype=torch.int32, pin_memory=True).numpy()
    # pageable (staged) and pinned input; pageable (staged) and pinned (direct) logits
    for src, out in ((imgs, None), (pinned.numpy(), None), (pinned.numpy(), pinned_logits)):
        tc = np.empty((n, ns + 1), np.int32)
        warn = np.empty(n, np.uint8)
        if out is not None:
            out[:] = -1
        host = eng.infer_host(src, logits=out, token_counts=tc, warnings=warn)
        np.testing.assert_array_equal(host, dev["logits"].cpu().numpy())
        np.testing.assert_array_equal(tc, dev["token_counts"].cpu().numpy())
        np.testing.assert_array_equal(warn, dev["warnings"].cpu().numpy())


def test_host_submit_wait_pipeline(cuda):
    """Asynchronous host calls: up to two in flight, buffers alternating across
    calls, single- and multi-chunk calls, pageable and pinned arrays; every call's
    outputs equal the device entry's.  Other entry points refuse to run while a
    call is in flight."""
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    params = synth.config3_params(synth.SEED)
    eng = Engine(params)
    ns = eng.num_selectors
    # the first call (nothing in flight) runs 512 + 188 images on two streams; the
    # calls behind it run as 1024-image chunks on one stream: 1024 + 476, 300, 1024,
    # 5 and 513 images (the 1500-image call reuses a workspace that the first call's
    # second chunk may still be using on the other stream)
    sizes = [700, 1500, 300, 1024, 5, 513]
    calls = []
    for i, n in enumerate(sizes):
        imgs = synth.baseline_images(synth.SEED, n, first=3000 + 1000 * i)
        dev = eng.infer(torch.from_numpy(imgs).cuda())
        if i % 2:
            src = torch.empty(imgs.shape, dtype=torch.int8, pin_memory=True).numpy()
            src[:] = imgs
            lg = torch.empty((n, 1000), dtype=torch.int32, pin_memory=True).numpy()
        else:
            src, lg = imgs, np.empty((n, 1000), np.int32)
        calls.append(dict(src=src, logits=lg, tc=np.empty((n, ns + 1), np.int32), warn=np.empty(n, np.uint8),
                          summ=np.empty((n, ns, 6), np.int32), dev=dev))
    def check(c):
        np.testing.assert_array_equal(c["logits"], c["dev"]["logits"].cpu().numpy())
        np.testing.assert_array_equal(c["tc"], c["dev"]["token_counts"].cpu().numpy())
        np.testing.assert_array_equal(c["summ"], c["dev"]["summary"].cpu().numpy())
        np.testing.assert_array_equal(c["warn"], c["dev"]["warnings"].cpu().numpy())

    def submit(c):
        for k in ("logits", "tc", "summ"):
            c[k].fill(-1)
        c["warn"].fill(255)
        eng.infer_host_submit(c["src"], c["logits"], token_counts=c["tc"], summary=c["summ"], warnings=c["warn"])

    # two calls in flight at every submit after the first; waits return in order
    done = []
    for i, c in enumerate(calls):
        submit(c)
        if i == 1:
            with pytest.raises(RuntimeError, match="in flight"):
                eng.infer(torch.zeros((1, 150528), dtype=torch.int8, device="cuda"))
            with pytest.raises(RuntimeError, match="in flight"):
                eng.infer_host(c["src"])
        if len(eng._inflight) == 2:
            done.append(eng.infer_host_wait())
    done.append(eng.infer_host_wait())
    assert [id(a) for a in done] == [id(c["logits"]) for c in calls]
    for c in calls:
        check(c)
    # a third submit waits for the oldest call itself
    for c in calls[:5]:
        submit(c)
    while eng._inflight:
        eng.infer_host_wait()
    for c in calls[:5]:
        check(c)
    eng.infer(torch.zeros((1, 150528), dtype=torch.int8, device="cuda"))  # idle again
    with pytest.raises(RuntimeError, match="no host call"):
        eng.infer_host_wait()


def test_engine_input_errors(cuda):
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    eng = Engine(synth.config_params(synth.SEED, pruned=True))
    with pytest.raises(TypeError):
        eng.infer(torch.zeros((2, 150528), dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        eng.infer(torch.zeros((2, 1000), dtype=torch.int8, device="cuda"))


# ---- component entry points (golden signatures) --------------------------------------

def test_transformer_block_composed_vs_golden(cuda):
    from heatvit_b200 import synth
    from heatvit_b200.transformer import transformer_block
    g = load_golden("golden_units.npz")
    blk = synth.config_params(synth.SEED, pruned=True).blocks[3]
    z, ck = transformer_block(g["block_x"].tolist(), blk)
    np.testing.assert_array_equal(np.array(z), g["block_z"])
    for key in ("ln1", "fused_qkv", "score", "prob", "context", "concat", "msa", "y", "ln2", "hidden", "ffn_out"):
        np.testing.assert_array_equal(np.array(ck[key]), g[f"block_ck_{key}"], err_msg=key)


def test_transformer_block_fused_ragged_vs_oracle(cuda, oracle):
    from heatvit_b200 import synth
    from heatvit_b200.transformer import transformer_block_batch
    params = synth.config_params(synth.SEED, pruned=True)
    rng = np.random.default_rng(4)
    counts = [197, 1, 2, 31, 32, 33, 88, 150, 196, 17]
    xs = [rng.integers(-128, 128, (n, 192)) for n in counts]
    for b in (0, 5, 11):
        zs = transformer_block_batch(xs, params.blocks[b])
        for x, z in zip(xs, zs):
            want, _, _ = oracle.transformer_block(x, params.blocks[b])
            np.testing.assert_array_equal(z, want)


def test_transformer_block_ragged_two_attention_launches_vs_oracle(cuda, oracle):
    """More than 3 images per SM with lengths on both sides of 128: the attention
    stage then runs list A (n <= 128) and list B (n > 128) as two launches of two CTA
    shapes instead of one launch over both lists."""
    import torch
    from heatvit_b200 import synth
    from heatvit_b200.transformer import transformer_block_batch
    params = synth.config_params(synth.SEED, pruned=True)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rng = np.random.default_rng(41)
    counts = rng.integers(1, 198, 3 * sms + 37)
    counts[:4] = [197, 128, 129, 1]
    xs = [rng.integers(-128, 128, (int(n), 192)) for n in counts]
    zs = transformer_block_batch(xs, params.blocks[5])
    for x, z in zip(xs, zs):
        want, _, _ = oracle.transformer_block(x, params.blocks[5])
        np.testing.assert_array_equal(z, want)


@pytest.mark.parametrize("q,k", [(-8, 9), (-5, 12), (-10, 7)])
def test_attention_wide_scores_vs_oracle(cuda, oracle, q, k):
    """Attention rows with wide Q8.16 spreads: qkv_out_scale_exp q (score_scale 2q - 3)
    with the QKV weight exponent raised by k so the scores stay large.  (-8, 9): most
    arguments above the small-argument table, none past ln2; (-5, 12): arguments far
    past ln2 (zero exp terms) through the general (non-FAST) q16 form; (-10, 7): small
    arguments only.  The benchmark model's rows are nearly flat, so these cases carry
    the general exp path of the attention kernel."""
    import dataclasses
    from heatvit_b200 import synth
    from heatvit_b200.transformer import transformer_block_batch
    params = synth.config_params(synth.SEED, pruned=True)
    bp = params.blocks[5]
    m = dataclasses.replace(bp.mhsa, qkv_out_scale_exp=q, score_scale_exp=2 * q - 3,
                            wqkv_scale_exp=bp.mhsa.wqkv_scale_exp + k)
    blk = dataclasses.replace(bp, mhsa=m)
    rng = np.random.default_rng([-q, k])
    counts = [197, 1, 2, 31, 32, 33, 64, 65, 88, 128, 129, 150, 196, 17]
    xs = [rng.integers(-128, 128, (n, 192)) for n in counts]
    zs = transformer_block_batch(xs, blk)
    for x, z in zip(xs, zs):
        want, _, _ = oracle.transformer_block(x, blk)
        np.testing.assert_array_equal(z, want)


def test_patch_embedding_vs_oracle(cuda, oracle):
    from heatvit_b200 import synth
    from heatvit_b200.transformer import patch_embedding
    params = synth.config_params(synth.SEED, pruned=True)
    img = synth.baseline_images(synth.SEED, 1)[0]
    np.testing.assert_array_equal(np.array(patch_embedding(img, params.patch)),
                                  oracle.patch_embedding(img, params.patch))


def test_token_selector_vs_golden(cuda):
    from heatvit_b200 import synth
    from heatvit_b200.selector import token_selector
    g = load_golden("golden_units.npz")
    params = synth.config_params(synth.SEED, pruned=True)
    i = 0
    while f"sel{i}_in" in g:
        n, pkg, stage = (int(v) for v in g[f"sel{i}_cfg"])
        r = token_selector(g[f"sel{i}_in"].tolist(), pkg, params.selectors[stage])
        np.testing.assert_array_equal(np.array(r.tokens), g[f"sel{i}_out"])
        assert (r.token_count, int(r.package_present), r.kept_normal_count, r.pruned_normal_count,
                r.warnings) == tuple(int(v) for v in g[f"sel{i}_state"])
        np.testing.assert_array_equal(np.array(r.fused_scores), g[f"sel{i}_fused"])
        np.testing.assert_array_equal(np.array(r.head_scores), g[f"sel{i}_head_scores"])
        np.testing.assert_array_equal(np.array(r.head_weights), g[f"sel{i}_head_weights"])
        np.testing.assert_array_equal(np.array(r.local), g[f"sel{i}_local"])
        np.testing.assert_array_equal(np.array(r.global_features), g[f"sel{i}_global"])
        np.testing.assert_array_equal(np.array(r.head_stats), g[f"sel{i}_stats"])
        i += 1


def _zero_den_selector(params, head_zero):
    """Selector parameters that force every keep score to 0 (package
    denominator zero) or every head weight to 0 (head denominator zero)."""
    from dataclasses import replace
    s = params.selectors[0]
    w3 = np.zeros((3, 16, 2), np.int8)
    b3 = np.tile(np.array([[1 << 30, -(1 << 30)]], np.int32), (3, 1))
    score = replace(s.score, w3=w3, b3=b3)
    s = replace(s, score=score, logits_out_scale_exp=-2, score_w3_scale_exp=-2 - s.h2_out_scale_exp)
    if head_zero:
        hw = replace(s.head_weight, w2=np.zeros((3, 3), np.int8), b2=np.full(3, -(1 << 30), np.int32))
        s = replace(s, head_weight=hw, hw_w2_scale_exp=-8, hw_hidden_out_scale_exp=-8)
    return s


@pytest.mark.parametrize("head_zero", [False, True])
def test_selector_zero_denominators_vs_oracle(cuda, oracle, head_zero):
    from heatvit_b200 import synth
    from heatvit_b200.selector import token_selector_batch
    params = synth.config_params(synth.SEED, pruned=True)
    sel = _zero_den_selector(params, head_zero)
    rng = np.random.default_rng(8)
    mats = [rng.integers(-128, 128, (n, 192)) for n in (197, 88, 2, 45)]
    pk = [0, 1, 1, 0]
    res = token_selector_batch(mats, pk, sel, intermediates=True)
    for m, p, r in zip(mats, pk, res):
        o = oracle.token_selector(m, p, sel)
        np.testing.assert_array_equal(r["tokens"], o["tokens"])
        assert r["warnings"] == o["warnings"]
        assert r["warnings"] & 2  # package fallback to the arithmetic mean
        if head_zero:
            assert r["warnings"] & 1
        np.testing.assert_array_equal(r["fused_scores"], o["fused_scores"])


def test_selector_ragged_batch_vs_oracle(cuda, oracle):
    from heatvit_b200 import synth
    from heatvit_b200.selector import token_selector_batch
    params = synth.config_params(synth.SEED, pruned=True)
    rng = np.random.default_rng(12)
    # random counts plus the edges of the selector's 128-row tensor-core tiles (one
    # full tile, a second tile holding one row) and the smallest selectable image
    counts = list(rng.integers(2, 198, 40)) + [2, 3, 127, 128, 129, 130, 196, 197]
    mats = [rng.integers(-128, 128, (n, 192)) for n in counts]
    pk = list(rng.integers(0, 2, len(counts)))
    for stage in range(3):
        res = token_selector_batch(mats, pk, params.selectors[stage], intermediates=True)
        for m, p, r in zip(mats, pk, res):
            o = oracle.token_selector(m, p, params.selectors[stage])
            np.testing.assert_array_equal(r["tokens"], o["tokens"])
            assert (r["kept_normal_count"], r["pruned_normal_count"], r["warnings"]) == \
                (o["kept_normal"], o["pruned_normal"], o["warnings"])
            np.testing.assert_array_equal(r["head_weights"], o["head_weights"])


def test_model_parameter_errors(cuda):
    from dataclasses import replace
    from heatvit_b200 import synth
    from heatvit_b200.engine import Engine
    params = synth.config_params(synth.SEED, pruned=True)
    bad = replace(params, blocks=(replace(params.blocks[0], mhsa=replace(params.blocks[0].mhsa, x_scale_exp=3)),)
                  + params.blocks[1:])
    with pytest.raises(ValueError):
        Engine(bad)


@pytest.mark.parametrize("l2,w1,hid", [(-12, -8, -11), (-20, -20, -8), (-9, -8, -20), (-8, -8, -9), (-14, -2, -5),
                                       (-7, -10, -13),
                                       # short output windows: the exact table form
                                       (-13, -10, -15), (-14, -13, -18), (-12, -12, -16), (-12, -14, -14),
                                       # central tables with FMA-form escapes: often / seldom taken
                                       (-8, -8, -11), (-9, -8, -11),
                                       # two-level bucket tables over 300k+ input windows
                                       (-8, -8, -8), (-9, -8, -10)])
def test_ffn_gelu_epilogue_exponents(cuda, oracle, l2, w1, hid):
    """FC1's fused GELU epilogue (table, FMA-pipe and 64-bit forms) across
    input/output exponents, through the fused block kernel."""
    from dataclasses import replace
    from heatvit_b200 import synth
    from heatvit_b200.transformer import transformer_block_batch
    blk = synth.config_params(synth.SEED, pruned=True).blocks[2]
    blk = replace(blk, ffn=replace(blk.ffn, ln2_out_scale_exp=l2, w1_scale_exp=w1, hidden_out_scale_exp=hid))
    rng = np.random.default_rng(abs(l2 * 31 + hid))
    xs = [rng.integers(-128, 128, (n, 192)) for n in (197, 64, 5)]
    for x, z in zip(xs, transformer_block_batch(xs, blk)):
        want, _, _ = oracle.transformer_block(x, blk)
        np.testing.assert_array_equal(z, want)
