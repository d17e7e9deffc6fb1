#!/usr/bin/env python3
"""Generate the committed golden fixtures under tests/golden/.

Run next to the reference checkout (it is not available on the GPU box):

    python tests/golden/make_golden.py --reference /path/to/HeatViT

Two kinds of fixtures:

* ``kat_*.npz`` decode the reference's own committed known-answer vectors
  (sim/vectors/*: requant, divsqrt, nonlinear, softmax, layernorm, gemm,
  selector), whose record layouts are defined by tools/generate_unit_vectors.py,
  tools/generate_gemm_vectors.py and tools/generate_selector_vectors.py.
* ``golden_*.npz`` hold outputs of the reference golden model
  (verification/heatvit_ref) imported and run here on seeded inputs: the
  reference's own seeded model (weights.build_params), benchmark-generator
  models, and per-operator cases.

The reference tree is read-only; bytecode writing is disabled.
"""

import argparse
import hashlib
import json
import os
import random
import sys
import time

sys.dont_write_bytecode = True
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402


def read_mem(path):
    with open(path) as f:
        return [int(line, 16) for line in f if line.strip()]


def sx(v, bits):
    v &= (1 << bits) - 1
    return v - (1 << bits) if v >> (bits - 1) else v


def bytes_of(words, count):
    out = []
    for w in words:
        out += [(w >> (8 * j)) & 0xFF for j in range(8)]
    return out[:count]


def i8(b):
    return [x - 256 if x >= 128 else x for x in b]


def i32(b):
    vals = []
    for i in range(0, len(b) - 3, 4):
        v = b[i] | (b[i + 1] << 8) | (b[i + 2] << 16) | (b[i + 3] << 24)
        vals.append(v - (1 << 32) if v >> 31 else v)
    return vals


# ---------------------------------------------------------------------------
# KAT decoders
# ---------------------------------------------------------------------------

def kat_requant(ref):
    out = {}
    for suite, header in (("fixed", False), ("requant", True)):
        words = read_mem(os.path.join(ref, "sim/vectors", suite, "requant.mem"))
        if header:
            words = words[1:1 + words[0]]
        # tools/generate_unit_vectors.py:58-64: value48 | src6<<48 | dst6<<54 | exp8<<60
        out[f"{suite}_value"] = np.array([sx(w, 48) for w in words], np.int64)
        out[f"{suite}_src"] = np.array([sx(w >> 48, 6) for w in words], np.int32)
        out[f"{suite}_dst"] = np.array([sx(w >> 54, 6) for w in words], np.int32)
        out[f"{suite}_expected"] = np.array([sx(w >> 60, 8) for w in words], np.int32)
    return out


def kat_divsqrt(ref):
    u = read_mem(os.path.join(ref, "sim/vectors/divsqrt/udiv.mem"))
    u = u[1:1 + u[0]]
    s = read_mem(os.path.join(ref, "sim/vectors/divsqrt/isqrt.mem"))
    s = s[1:1 + s[0]]
    m64 = (1 << 64) - 1
    return dict(
        udiv_num=np.array([w & m64 for w in u], np.uint64), udiv_den=np.array([(w >> 64) & m64 for w in u], np.uint64),
        udiv_q=np.array([(w >> 128) & m64 for w in u], np.uint64),
        udiv_r=np.array([(w >> 192) & m64 for w in u], np.uint64),
        isqrt_rad=np.array([w & ((1 << 48) - 1) for w in s], np.uint64),
        isqrt_root=np.array([(w >> 48) & 0xFFFFFFFF for w in s], np.uint64),
        isqrt_rem=np.array([(w >> 80) & ((1 << 48) - 1) for w in s], np.uint64))


def kat_nonlinear(ref):
    w = read_mem(os.path.join(ref, "sim/vectors/nonlinear/nonlinear.mem"))
    w = w[1:1 + w[0]]
    # tools/generate_unit_vectors.py:238-245: x24 | gelu24<<24 | plan17<<48
    return dict(x=np.array([sx(v, 24) for v in w], np.int64),
                gelu=np.array([sx(v >> 24, 24) for v in w], np.int64),
                plan=np.array([(v >> 48) & ((1 << 17) - 1) for v in w], np.int64))


def kat_softmax(ref):
    w = read_mem(os.path.join(ref, "sim/vectors/softmax/softmax.mem"))
    w = w[1:1 + w[0]]
    # tools/generate_unit_vectors.py:290-299: len8 | x24<<8 | attn8<<32 | sel17<<40
    x, attn, sel, lengths = [], [], [], []
    i = 0
    while i < len(w):
        n = w[i] & 0xFF or 256
        # rows of length 256 never occur; a length field of 0 would mean 256
        for j in range(n):
            v = w[i + j]
            x.append(sx(v >> 8, 24))
            attn.append((v >> 32) & 0xFF)
            sel.append((v >> 40) & ((1 << 17) - 1))
        lengths.append(n)
        i += n
    return dict(x=np.array(x, np.int64), attention=np.array(attn, np.int64), selector=np.array(sel, np.int64),
                lengths=np.array(lengths, np.int64))


def kat_layernorm(ref):
    w = read_mem(os.path.join(ref, "sim/vectors/layernorm/layernorm.mem"))
    count = w[0]
    w = w[1:]
    xs, gs, bs, ex, scales, warn = [], [], [], [], [], []
    for t in range(count):
        cfg = w[t * 193]
        scales.append([sx(cfg, 6), sx(cfg >> 6, 6), sx(cfg >> 12, 6), sx(cfg >> 18, 6)])
        warn.append((cfg >> 24) & 1)
        rec = w[t * 193 + 1:t * 193 + 193]
        xs.append([sx(v, 8) for v in rec])
        gs.append([sx(v >> 8, 8) for v in rec])
        bs.append([sx(v >> 16, 8) for v in rec])
        ex.append([sx(v >> 24, 8) for v in rec])
    return dict(x=np.array(xs, np.int8), gamma=np.array(gs, np.int8), beta=np.array(bs, np.int8),
                expected=np.array(ex, np.int8), scales=np.array(scales, np.int32), warn=np.array(warn, np.int32))


# tools/generate_gemm_vectors.py:395-416 scenario scales (src0, src1, dst)
GEMM_SCALES = {"mini": (-7, -7, -7), "ordinary": (-7, -7, -7), "full": (-7, -7, -7), "tail": (-7, -7, -14),
               "large": (-7, -7, -7), "head": (-7, -7, -7), "transpose": (-7, -7, -7), "unsigned": (-8, -7, -15)}


def kat_gemm(ref):
    d = os.path.join(ref, "sim/vectors/gemm")
    man = json.load(open(os.path.join(d, "manifest.json")))
    out = {"names": np.array([s["name"] for s in man["scenarios"]])}
    for s in man["scenarios"]:
        name, m, n, k = s["name"], s["m"], s["n"], s["k"]
        heads = s["heads"] or 1
        a_bytes = bytes_of(read_mem(os.path.join(d, f"{name}_a.mem")), heads * m * k)
        w = read_mem(os.path.join(d, f"{name}_w.mem"))
        b_count = heads * n * k
        wb = bytes_of(w, len(w) * 8)
        b_vals = i8(wb[:b_count])
        pad = (-b_count) % 8
        bias = i32(wb[b_count + pad:b_count + pad + 4 * n]) if s["bias"] else []
        esize = 4 if s["output_bits"] == 32 else 1
        e = bytes_of(read_mem(os.path.join(d, f"{name}_expected.mem")), heads * m * n * esize)
        expected = i32(e) if esize == 4 else i8(e)
        a_vals = a_bytes if s["unsigned"] else i8(a_bytes)
        bshape = (heads, n, k) if s["transpose"] else (heads, k, n)
        src0, src1, dst = GEMM_SCALES[name]
        out[f"{name}_a"] = np.array(a_vals, np.int64).reshape(heads, m, k)
        out[f"{name}_b"] = np.array(b_vals, np.int64).reshape(bshape)
        out[f"{name}_bias"] = np.array(bias, np.int64)
        out[f"{name}_expected"] = np.array(expected, np.int64).reshape(heads, m, n)
        out[f"{name}_meta"] = np.array([m, n, k, heads, int(s["transpose"]), int(s["unsigned"]),
                                        s["output_bits"], int(s["bias"]), src0 + src1, dst], np.int64)
    # MAC-bank cases (35 words each): acc[r][c] = k * a[r] * b[c] for masked rows/cols.
    mb = read_mem(os.path.join(d, "mac_bank.mem"))
    mb = mb[1:1 + mb[0]]
    cases = []
    for c in range(len(mb) // 35):
        w0, w1, w2 = mb[c * 35:c * 35 + 3]
        acc = []
        for wd in mb[c * 35 + 3:c * 35 + 35]:
            acc += [sx(wd, 32), sx(wd >> 32, 32)]
        a = [(w0 >> (8 * j)) & 0xFF for j in range(8)]
        b = [sx(w1 >> (8 * j), 8) for j in range(8)]
        cases.append(a + b + [w2 & 0xFF, (w2 >> 8) & 0xFF, (w2 >> 16) & 1, (w2 >> 17) & 0x3FFF] + acc)
    out["mac_bank"] = np.array(cases, np.int64)
    return out


def kat_selector(ref):
    d = os.path.join(ref, "sim/vectors/selector")
    man = json.load(open(os.path.join(d, "manifest.json")))
    out = {"names": np.array(sorted(man["cases"]))}
    for name, meta in sorted(man["cases"].items()):
        n = meta["tokens"]
        tok = i8(bytes_of(read_mem(os.path.join(d, name, "tokens.mem")), n * 192))
        sc = i32(bytes_of(read_mem(os.path.join(d, name, "scores.mem")), meta["candidates"] * 4))
        nn = meta["next_token_count"]
        o = i8(bytes_of(read_mem(os.path.join(d, name, "output.mem")), nn * 192))
        out[f"{name}_tokens"] = np.array(tok, np.int8).reshape(n, 192)
        out[f"{name}_scores"] = np.array(sc, np.int32)
        out[f"{name}_output"] = np.array(o, np.int8).reshape(nn, 192)
        out[f"{name}_meta"] = np.array([n, meta["input_package_present"], nn, meta["next_package_present"],
                                        meta["warning_flags"]], np.int32)
    zd = os.path.join(d, "zero_den")
    nf = man["cases"]["zero_den"]["fuse_candidates"]
    out["fuse_scores"] = np.array(i32(bytes_of(read_mem(os.path.join(zd, "fuse_scores.mem")), nf * 12)),
                                  np.int32).reshape(nf, 3)
    out["fuse_weights"] = np.array(i32(bytes_of(read_mem(os.path.join(zd, "fuse_weights.mem")), nf * 12)),
                                   np.int32).reshape(nf, 3)
    out["fuse_expected"] = np.array(i32(bytes_of(read_mem(os.path.join(zd, "fuse_expected.mem")), nf * 4)), np.int32)
    out["fuse_warn"] = np.array(bytes_of(read_mem(os.path.join(zd, "fuse_warn.mem")), nf), np.int32)
    return out


# ---------------------------------------------------------------------------
# Golden-model runs
# ---------------------------------------------------------------------------

def ragged(rows_list):
    rows_list = [np.asarray(r, np.int8).reshape(-1, 192) for r in rows_list]
    off = np.zeros(len(rows_list) + 1, np.int32)
    off[1:] = np.cumsum([r.shape[0] for r in rows_list])
    return np.concatenate(rows_list, axis=0), off


CKPT_ORDER = ["patch"] + [f"block_{b:02d}" for b in range(1, 13)] + [f"selector_{s:02d}" for s in range(1, 4)] + \
    ["final_ln"]


def pack_result(res, prefix):
    keys = [k for k in CKPT_ORDER if k in res.checkpoints]
    data, off = ragged([res.checkpoints[k] for k in keys])
    summ = np.array([[s["input_tokens"], s["output_tokens"], s["kept_normal"], s["pruned_normal"],
                      s["package_present"]] for s in res.selector_summary], np.int32).reshape(-1, 5)
    return {f"{prefix}_logits": np.array(res.logits, np.int32), f"{prefix}_ckpt": data,
            f"{prefix}_ckpt_off": off, f"{prefix}_ckpt_keys": np.array(keys), f"{prefix}_summary": summ}


def params_digest(params):
    from heatvit_b200.params import PackedParams
    h = hashlib.sha256()
    for a in PackedParams(params)._keep:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def golden_seeded(R):
    from verification.heatvit_ref import weights as W
    from verification.heatvit_ref.model import HeatViTModel
    rng = random.Random(W.SEED)
    image = [rng.randint(-128, 127) for _ in range(224 * 224 * 3)]
    params, summary, counts = W.build_params(image)
    res = HeatViTModel().infer(image, params)
    out = pack_result(res, "seeded")
    out["seeded_calibration"] = np.array([[s["attempt"], s["median_logit_diff"]] for s in summary], np.int64)
    out["seeded_counts"] = np.array(counts, np.int32)
    out["seeded_params_sha256"] = np.array(params_digest(params))
    return out


def ref_namespace():
    """The golden dataclasses in one namespace (for params.to_reference)."""
    from verification.heatvit_ref import model as M
    from verification.heatvit_ref import selector as S
    from verification.heatvit_ref import transformer as T
    ns = type("ns", (), {})()
    for mod in (M, S, T):
        for k in dir(mod):
            setattr(ns, k, getattr(mod, k))
    return ns


def golden_baseline(R, seed, images, pruned, tag):
    from heatvit_b200 import synth
    from heatvit_b200.params import to_reference
    from verification.heatvit_ref import model as M
    params = synth.config_params(seed, pruned=pruned)
    gparams = to_reference(params, ref_namespace())
    imgs = synth.baseline_images(seed, images)
    out = {f"{tag}_seed": np.array(seed), f"{tag}_images": np.array(images), f"{tag}_pruned": np.array(int(pruned)),
           f"{tag}_params_sha256": np.array(params_digest(params))}
    for i in range(images):
        res = M.HeatViTModel().infer([int(v) for v in imgs[i]], gparams)
        out.update(pack_result(res, f"{tag}_{i}"))
    return out


def golden_config3(R, seed, indices):
    """Config-3 model (zero-denominator first selector) on chosen images of
    baseline_images(seed, .): a zero-package-denominator image and a regular one."""
    from heatvit_b200 import synth
    from heatvit_b200.params import to_reference
    from verification.heatvit_ref import model as M
    params = synth.config3_params(seed)
    gparams = to_reference(params, ref_namespace())
    imgs = synth.baseline_images(seed, max(indices) + 1)
    out = {"config3_seed": np.array(seed), "config3_indices": np.array(indices),
           "config3_params_sha256": np.array(params_digest(params))}
    from verification.heatvit_ref import selector as S
    for j, i in enumerate(indices):
        res = M.HeatViTModel().infer([int(v) for v in imgs[i]], gparams)
        out.update(pack_result(res, f"config3_{j}"))
        # the first selector again on its input, for its warning bits and scores
        r = S.token_selector(res.checkpoints["block_03"], 0, gparams.selectors[0])
        out[f"config3_{j}_sel1_warnings"] = np.array(r.warnings)
        out[f"config3_{j}_sel1_fused"] = np.array(r.fused_scores)
        out[f"config3_{j}_sel1_head_weights"] = np.array(r.head_weights)
    return out


def golden_memimage(R, seed):
    """Digests of the reference's weight image (serialize_weights at
    build_memory_map's weight offsets, and its .mem text) for the seeded model and
    the config-3 model, and the reference ScaleTable's saved text for config 3."""
    import tempfile
    from pathlib import Path
    from heatvit_b200 import synth
    from heatvit_b200 import memimage
    from heatvit_b200.params import to_reference
    from tools.generate_descriptors import build_memory_map
    from tools.generate_e2e_vectors import serialize_weights, write_mem_lines
    from tools.p2.scale_table import ScaleTable
    from verification.heatvit_ref import weights as W
    rng = random.Random(W.SEED)
    image = [rng.randint(-128, 127) for _ in range(224 * 224 * 3)]
    seeded, _, _ = W.build_params(image)
    mm = build_memory_map()[0]["weight"]
    out = {"memimage_seed": np.array(seed)}
    with tempfile.TemporaryDirectory() as td:
        for tag, gp in (("seeded", seeded), ("config3", to_reference(synth.config3_params(seed), ref_namespace()))):
            raw = serialize_weights(gp, mm)
            out[f"memimage_{tag}_bytes"] = np.array(len(raw))
            out[f"memimage_{tag}_sha256"] = np.array(hashlib.sha256(raw).hexdigest())
            path = Path(td) / f"{tag}.mem"
            write_mem_lines(path, raw)
            out[f"memimage_{tag}_mem_sha256"] = np.array(hashlib.sha256(path.read_bytes()).hexdigest())
        table = memimage.scale_table(synth.config3_params(seed))
        st = ScaleTable(weights=table["weights"], activations=table["activations"]).validate()
        path = Path(td) / "scales.json"
        st.save(path)
        out["memimage_config3_scales_json"] = np.array(path.read_text())
    return out


def golden_e2evectors(R):
    """The reference's end-to-end vector set for its seeded model and image
    (tools/generate_e2e_vectors.py ``generate``), written into a temporary
    folder: the SHA-256 of every region image and checkpoint file, and the full
    text of manifest.json and e2e_tb_config.sv.  The testbench package, which
    ``generate`` writes into the reference's sim/generated/, is redirected to the
    temporary folder and compared with the committed copy there."""
    import tempfile
    from pathlib import Path
    import tools.generate_e2e_vectors as G
    from verification.heatvit_ref import weights as W
    orig = G.write_e2e_tb_config
    with tempfile.TemporaryDirectory() as td:
        sv = Path(td) / "e2e_tb_config.sv"
        G.write_e2e_tb_config = lambda mm, manifest, layout, tc, cfg_path=None: orig(mm, manifest, layout, tc, sv)
        try:
            G.generate(W.SEED, Path(td) / "e2e")
        finally:
            G.write_e2e_tb_config = orig
        base = Path(td) / "e2e"
        names = ["input.mem", "weights.mem", "scratch_init.mem", "output_init.mem"]
        names += sorted(f"checkpoints/{p.name}" for p in (base / "checkpoints").iterdir())
        committed = (Path(R) / "sim" / "generated" / "e2e_tb_config.sv").read_text()
        return {
            "e2e_files": np.array(names),
            "e2e_sha256": np.array([hashlib.sha256((base / n).read_bytes()).hexdigest() for n in names]),
            "e2e_manifest": np.array((base / "manifest.json").read_text()),
            "e2e_tb_config_sv": np.array(sv.read_text()),
            "e2e_tb_config_matches_committed": np.array(sv.read_text() == committed),
        }


def _quant_deit(params, table, pruned):
    """The reference P2 simulator's QuantDeiT holding a model's integer tensors."""
    import torch
    from heatvit_b200 import memimage
    from tools.p2 import p2_sim as P
    from tools.p2.scale_table import ScaleTable
    t = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in memimage._tensors(params).items()}
    blocks = [P.BlockP(**{f: t[f"b{n}_{f}"] for f in P.BlockP.__dataclass_fields__}) for n in range(1, 13)]
    sels = [P.SelectorP(**{f: t[f"s{s}_{f}"] for f in P.SelectorP.__dataclass_fields__})
            for s in range(1, 4)] if pruned else []
    return P.QuantDeiT(scales=ScaleTable(weights=dict(table["weights"]), activations=dict(table["activations"])),
                       patch_w=t["patch_w"], patch_b=t["patch_b"], cls=t["cls"], pos=t["pos"], blocks=blocks,
                       selectors=sels, final_gamma=t["final_gamma"], final_beta=t["final_beta"],
                       head_w=t["head_w"], head_b=t["head_b"])


def golden_p2sim(R, seed, count=6):
    """The reference P2 simulator (tools/p2/p2_sim.py forward_image, pruned and
    unpruned) on the config-3 model and seeded float images
    (synth.p2_float_images): logits and token counts."""
    import torch
    from heatvit_b200 import memimage, synth
    from tools.p2 import p2_sim as P
    params = synth.config3_params(seed)
    table = memimage.scale_table(params)
    imgs = synth.p2_float_images(seed, count, params.patch.image_scale_exp)
    out = {"p2_seed": np.array(seed), "p2_count": np.array(count)}
    for tag, pruned in (("pruned", True), ("unpruned", False)):
        model = _quant_deit(params, table, pruned)
        logits, counts = [], []
        for i in range(count):
            lg, tc, e = P.forward_image(model, torch.from_numpy(imgs[i]), prune=pruned)
            assert e == -14
            logits.append(lg.numpy().astype(np.int32))
            counts.append(tc)
        out[f"p2_{tag}_logits"] = np.stack(logits)
        out[f"p2_{tag}_counts"] = np.array(counts, np.int32)
    return out


def golden_units(R, seed):
    """Per-operator golden outputs on seeded random inputs."""
    from verification.heatvit_ref import fixed as F
    from verification.heatvit_ref import gemm as G
    from verification.heatvit_ref import nonlinear as N
    from verification.heatvit_ref import selector as S
    from verification.heatvit_ref import transformer as T
    from heatvit_b200 import synth
    from heatvit_b200.params import to_reference
    rng = np.random.default_rng(seed)
    out = {}
    # LayerNorm with scales in the benchmark range and in the full 6-bit range.
    rows, scales, exp, warn = [], [], [], []
    for i in range(96):
        x = rng.integers(-128, 128, 192)
        if i % 8 == 0:
            x = np.full(192, rng.integers(-128, 128)) + rng.integers(-1, 2, 192)
            x = np.clip(x, -128, 127)
        g = rng.integers(-128, 128, 192)
        b = rng.integers(-128, 128, 192)
        if i < 48:
            sc = [int(rng.integers(-20, -7)), int(rng.integers(-20, -7)), int(rng.integers(-20, -7)),
                  int(rng.integers(-20, -7))]
        else:
            sc = [int(rng.integers(-32, 1)), int(rng.integers(-32, 32)), int(rng.integers(-32, 32)),
                  int(rng.integers(-32, 32))]
        o, w = N.layernorm([int(v) for v in x], [int(v) for v in g], [int(v) for v in b], *sc)
        rows.append(np.stack([x, g, b]))
        scales.append(sc)
        exp.append(o)
        warn.append(int(w))
    out["ln_inputs"] = np.array(rows, np.int8)
    out["ln_scales"] = np.array(scales, np.int32)
    out["ln_expected"] = np.array(exp, np.int8)
    out["ln_warn"] = np.array(warn, np.int32)
    # Softmax rows: config-2 style Gaussian scores (sigma 2^12) converted to Q16
    # at score_scale -17, plus wide uniform rows.
    lens = list(rng.integers(1, 198, 48)) + [197] * 8
    vals, att, sel = [], [], []
    for i, n in enumerate(lens):
        if i % 2:
            row = rng.integers(-(1 << 23), 1 << 23, n)
        else:
            s = np.clip(np.rint(rng.normal(0, 4096, n)), -(1 << 31), (1 << 31) - 1).astype(np.int64)
            row = np.array([F.sat_signed(F.round_shift_away(int(v), 4), 24) for v in s])
        vals += [int(v) for v in row]
        att += N.softmax_attention([int(v) for v in row])
        sel += N.softmax_selector([int(v) for v in row])
    out["sm_x"] = np.array(vals, np.int64)
    out["sm_len"] = np.array(lens, np.int64)
    out["sm_attention"] = np.array(att, np.int64)
    out["sm_selector"] = np.array(sel, np.int64)
    # GELU / PLAN on random Q8.16 values and the FFN chain on int32 accumulators.
    gx = rng.integers(-(1 << 23), 1 << 23, 4096)
    out["gelu_x"] = gx
    out["gelu_y"] = np.array([N.gelu(int(v)) for v in gx], np.int64)
    out["plan_y"] = np.array([N.plan_sigmoid(int(v)) for v in gx], np.int64)
    acc = np.clip(np.rint(rng.normal(0, 1024, 4096)), -(1 << 31), (1 << 31) - 1).astype(np.int64)
    out["chain_acc"] = acc
    out["chain_y"] = np.array([F.requant(N.gelu(F.requant(int(v), -14, -16, 24)), -16, -7, 8) for v in acc], np.int64)
    # GEMM + writeback over the model's shapes (small M) and random exponents.
    gem = []
    for i, (m, k, n) in enumerate([(37, 192, 576), (29, 192, 192), (33, 192, 768), (21, 768, 192), (5, 768, 192),
                                   (17, 64, 32), (9, 32, 16), (7, 16, 2), (13, 3, 3)]):
        a = rng.integers(-128, 128, (m, k))
        w = rng.integers(-127, 128, (k, n))
        bias = rng.integers(-(1 << 15), (1 << 15) + 1, n)
        src = int(rng.integers(-40, -15))
        dst = src + (11 if k == 192 else 12) + int(rng.integers(-3, 4))
        accm = G.gemm_numpy(a.tolist(), w.tolist(), bias.tolist(), False)
        gem.append((a, w, bias, src, dst, np.array(G.gemm_writeback(accm, src, dst, 8)),
                    np.array(G.gemm_writeback(accm, src, -14, 32))))
    for i, (a, w, bias, src, dst, o8, o32) in enumerate(gem):
        out[f"gemm{i}_a"], out[f"gemm{i}_w"], out[f"gemm{i}_bias"] = a, w, bias
        out[f"gemm{i}_exps"] = np.array([src, dst])
        out[f"gemm{i}_out8"], out[f"gemm{i}_out32"] = o8, o32
    # Transformer block, MHSA, FFN on a small token count with a benchmark block.
    gparams = to_reference(synth.config_params(seed, pruned=True), ref_namespace())
    block = gparams.blocks[3]
    x = rng.integers(-128, 128, (23, 192))
    z, ck = T.transformer_block(x.tolist(), block)
    out["block_x"] = x
    out["block_z"] = np.array(z)
    for key in ("ln1", "fused_qkv", "score", "prob", "context", "concat", "msa", "y", "ln2", "hidden", "ffn_out"):
        out[f"block_ck_{key}"] = np.array(ck[key])
    # Token selector with the benchmark selector parameters on random tokens.
    sel_params = gparams.selectors
    cases = []
    for i, (n, pkg, stage) in enumerate([(197, 0, 0), (88, 1, 1), (45, 1, 2), (2, 0, 0), (3, 1, 1), (12, 0, 2)]):
        t = rng.integers(-128, 128, (n, 192))
        r = S.token_selector(t.tolist(), pkg, sel_params[stage])
        out[f"sel{i}_in"] = t
        out[f"sel{i}_cfg"] = np.array([n, pkg, stage])
        out[f"sel{i}_out"] = np.array(r.tokens)
        out[f"sel{i}_state"] = np.array([r.token_count, int(r.package_present), r.kept_normal_count,
                                         r.pruned_normal_count, r.warnings])
        out[f"sel{i}_fused"] = np.array(r.fused_scores)
        out[f"sel{i}_head_scores"] = np.array(r.head_scores)
        out[f"sel{i}_head_weights"] = np.array(r.head_weights)
        out[f"sel{i}_local"] = np.array(r.local)
        out[f"sel{i}_global"] = np.array(r.global_features)
        out[f"sel{i}_stats"] = np.array(r.head_stats)
    return out


def _narrow(a):
    a = np.asarray(a)
    if a.dtype.kind in "iu" and a.size:
        lo, hi = int(a.min()), int(a.max())
        for dt in (np.int8, np.int16, np.int32):
            if np.iinfo(dt).min <= lo and hi <= np.iinfo(dt).max:
                return a.astype(dt)
    return a


def save(name, data):
    data = {k: _narrow(v) for k, v in data.items()}
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **data)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)", flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    ref = os.path.abspath(args.reference)
    sys.path.insert(0, ref)
    want = set(args.only.split(",")) if args.only else None

    def on(name):
        return want is None or name in want

    t0 = time.time()
    if on("kat"):
        save("kat_requant.npz", kat_requant(ref))
        save("kat_divsqrt.npz", kat_divsqrt(ref))
        save("kat_nonlinear.npz", kat_nonlinear(ref))
        save("kat_softmax.npz", kat_softmax(ref))
        save("kat_layernorm.npz", kat_layernorm(ref))
        save("kat_gemm.npz", kat_gemm(ref))
        save("kat_selector.npz", kat_selector(ref))
    if on("units"):
        save("golden_units.npz", golden_units(ref, 20260815))
    if on("seeded"):
        save("golden_seeded.npz", golden_seeded(ref))
    if on("baseline"):
        save("golden_baseline.npz", golden_baseline(ref, 20260815, 2, True, "pruned"))
    if on("memimage"):
        save("golden_memimage.npz", golden_memimage(ref, 20260815))
    if on("e2evectors"):
        save("golden_e2evectors.npz", golden_e2evectors(ref))
    if on("p2sim"):
        save("golden_p2sim.npz", golden_p2sim(ref, 20260815))
    if on("config3"):
        save("golden_config3.npz", golden_config3(ref, 20260815, (2, 0)))
    if on("unpruned"):
        save("golden_unpruned.npz", golden_baseline(ref, 20260815, 1, False, "unpruned"))
    print(f"done in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
