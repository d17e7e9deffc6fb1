"""The reference's weight memory image and per-tensor scale table.

* Weight region layout (tools/generate_descriptors.py:154-196 ``build_memory_map``):
  the tensors of patch, 12 blocks, 3 selectors, final LN and head, each placed at
  the next 8-byte boundary in a fixed order.  int8 tensors are stored row-major
  as the golden dataclasses hold them; int32 biases are little-endian.  Selector
  tensors hold their three heads back to back.
* Serialisation (tools/generate_e2e_vectors.py:87-155 ``serialize_weights``) and
  the ``.mem`` text form: one 64-bit little-endian beat per line, 16 hex digits,
  the last beat zero-padded (tools/generate_e2e_vectors.py:66-81).
* The scale table (tools/p2/scale_table.py): JSON with "weights" and
  "activations" maps of tensor name to exponent, keys sorted, two-space indent;
  its mapping onto the golden dataclasses follows tools/p2/p2_export_weights.py:
  86-94, 115-241 (block n reads ``act_tokens`` or ``b<n-1>_out``, selector s
  reads ``b<3s>_out``; score = 2 * qkv_out - 3, prob = -8; bias exponents are
  derived).

``read_weights(raw, table)`` and ``write_weights(params)`` convert between the
image and ``HeatViTParams``, so an engine can load the reference's exported
weights unchanged.
"""

import json

import numpy as np

from .params import (
    BlockParams, FfnParams, HeatViTParams, MhsaParams, PatchParams, SelectorHeadWeightParams,
    SelectorLocalParams, SelectorParams, SelectorScoreParams,
)

_BLOCK = (("wqkv", (192, 576), 1), ("bqkv", (576,), 4), ("wproj", (192, 192), 1), ("bproj", (192,), 4),
          ("gamma1", (192,), 1), ("beta1", (192,), 1), ("w1", (192, 768), 1), ("b1", (768,), 4),
          ("w2", (768, 192), 1), ("b2", (192,), 4), ("gamma2", (192,), 1), ("beta2", (192,), 1))
_SEL = (("local_w", (3, 64, 32), 1), ("local_b", (3, 32), 4), ("score_w1", (3, 64, 32), 1),
        ("score_b1", (3, 32), 4), ("score_w2", (3, 32, 16), 1), ("score_b2", (3, 16), 4),
        ("score_w3", (3, 16, 2), 1), ("score_b3", (3, 2), 4), ("hw_w1", (3, 3), 1), ("hw_b1", (3,), 4),
        ("hw_w2", (3, 3), 1), ("hw_b2", (3,), 4))


def weight_layout():
    """[(name, offset, shape, element bytes)] of the weight region, in order."""
    entries = [("patch_w", (768, 192), 1), ("patch_b", (192,), 4), ("cls", (192,), 1), ("pos", (197, 192), 1)]
    entries += [(f"b{n}_{k}", s, e) for n in range(1, 13) for k, s, e in _BLOCK]
    entries += [(f"s{n}_{k}", s, e) for n in range(1, 4) for k, s, e in _SEL]
    entries += [("final_gamma", (192,), 1), ("final_beta", (192,), 1), ("head_w", (192, 1000), 1),
                ("head_b", (1000,), 4)]
    out, cur = [], 0
    for name, shape, esz in entries:
        off = (cur + 7) & ~7
        out.append((name, off, shape, esz))
        cur = off + int(np.prod(shape)) * esz
    return out


def weight_bytes():
    """Size of the weight region (8-byte aligned)."""
    name, off, shape, esz = weight_layout()[-1]
    return (off + int(np.prod(shape)) * esz + 7) & ~7


def _tensors(params):
    p = params
    t = {"patch_w": p.patch.patch_weight, "patch_b": p.patch.patch_bias, "cls": p.patch.cls, "pos": p.patch.pos}
    for n, b in enumerate(p.blocks, start=1):
        m, f = b.mhsa, b.ffn
        t.update({f"b{n}_wqkv": m.wqkv, f"b{n}_bqkv": m.bqkv, f"b{n}_wproj": m.wproj, f"b{n}_bproj": m.bproj,
                  f"b{n}_gamma1": m.ln_gamma, f"b{n}_beta1": m.ln_beta, f"b{n}_w1": f.w1, f"b{n}_b1": f.b1,
                  f"b{n}_w2": f.w2, f"b{n}_b2": f.b2, f"b{n}_gamma2": f.ln_gamma, f"b{n}_beta2": f.ln_beta})
    for n, s in enumerate(p.selectors, start=1):
        t.update({f"s{n}_local_w": s.local.w, f"s{n}_local_b": s.local.b, f"s{n}_score_w1": s.score.w1,
                  f"s{n}_score_b1": s.score.b1, f"s{n}_score_w2": s.score.w2, f"s{n}_score_b2": s.score.b2,
                  f"s{n}_score_w3": s.score.w3, f"s{n}_score_b3": s.score.b3, f"s{n}_hw_w1": s.head_weight.w1,
                  f"s{n}_hw_b1": s.head_weight.b1, f"s{n}_hw_w2": s.head_weight.w2,
                  f"s{n}_hw_b2": s.head_weight.b2})
    t.update({"final_gamma": p.final_gamma, "final_beta": p.final_beta, "head_w": p.head_w, "head_b": p.head_b})
    return t


def write_weights(params):
    """serialize_weights: the weight region image (bytes) of a pruned model."""
    if len(params.selectors) != 3:
        raise ValueError("the weight image holds exactly three selectors")
    t = _tensors(params)
    buf = bytearray(weight_bytes())
    for name, off, shape, esz in weight_layout():
        a = np.asarray(t[name], np.int64).reshape(shape)
        raw = a.astype("<i4" if esz == 4 else np.int8).tobytes()
        buf[off:off + len(raw)] = raw
    return bytes(buf)


def mem_lines(raw):
    """.mem text: one 64-bit little-endian beat per line (16 hex digits)."""
    raw = bytes(raw) + b"\0" * ((-len(raw)) % 8)
    beats = np.frombuffer(raw, np.uint8).reshape(-1, 8)[:, ::-1]  # most significant byte first
    digits = np.frombuffer(beats.tobytes().hex().encode(), np.uint8).reshape(-1, 16)
    return np.concatenate([digits, np.full((digits.shape[0], 1), ord("\n"), np.uint8)], 1).tobytes().decode()


def parse_mem(text):
    """Bytes of a .mem text (inverse of mem_lines; the padding stays)."""
    lines = text.split()
    if all(len(v) == 16 for v in lines):
        return np.frombuffer(bytes.fromhex("".join(lines)), np.uint8).reshape(-1, 8)[:, ::-1].tobytes()
    return b"".join(int(v, 16).to_bytes(8, "little") for v in lines)


def _arrays(raw):
    if len(raw) < weight_bytes():
        raise ValueError(f"weight image too short: {len(raw)} < {weight_bytes()} bytes")
    out = {}
    for name, off, shape, esz in weight_layout():
        n = int(np.prod(shape))
        dt = np.dtype("<i4") if esz == 4 else np.dtype(np.int8)
        out[name] = np.frombuffer(raw, dt, n, off).reshape(shape).astype(np.int32 if esz == 4 else np.int8)
    return out


# ---- scale table --------------------------------------------------------------------

def scale_table(params):
    """The scale-table maps ({"weights": ..., "activations": ...}) of a pruned model."""
    p = params
    w = {"patch_w": p.patch.weight_scale_exp, "cls": p.patch.cls_scale_exp, "pos": p.patch.pos_scale_exp,
         "final_gamma": p.final_gamma_scale_exp, "final_beta": p.final_beta_scale_exp,
         "head_w": p.head_w_scale_exp}
    a = {"input": p.patch.image_scale_exp, "act_patch_matrix": p.patch.image_scale_exp,
         "act_patch_embed": p.patch.activation_scale_exp, "act_tokens": p.patch.tokens_scale_exp,
         "final_ln_out": p.final_ln_out_scale_exp}
    for n, b in enumerate(p.blocks, start=1):
        m, f = b.mhsa, b.ffn
        w.update({f"b{n}_wqkv": m.wqkv_scale_exp, f"b{n}_wproj": m.wproj_scale_exp,
                  f"b{n}_gamma1": m.gamma1_scale_exp, f"b{n}_beta1": m.beta1_scale_exp, f"b{n}_w1": f.w1_scale_exp,
                  f"b{n}_w2": f.w2_scale_exp, f"b{n}_gamma2": f.gamma2_scale_exp, f"b{n}_beta2": f.beta2_scale_exp})
        a.update({f"b{n}_ln1_out": m.ln1_out_scale_exp, f"b{n}_qkv_out": m.qkv_out_scale_exp,
                  f"b{n}_context_out": m.context_out_scale_exp, f"b{n}_msa_out": m.msa_out_scale_exp,
                  f"b{n}_y": f.x_scale_exp, f"b{n}_ln2_out": f.ln2_out_scale_exp,
                  f"b{n}_hidden": f.hidden_out_scale_exp, f"b{n}_ffn_out": f.ffn_out_scale_exp,
                  f"b{n}_out": f.out_scale_exp})
    for n, s in enumerate(p.selectors, start=1):
        w.update({f"s{n}_local_w": s.local_w_scale_exp, f"s{n}_score_w1": s.score_w1_scale_exp,
                  f"s{n}_score_w2": s.score_w2_scale_exp, f"s{n}_score_w3": s.score_w3_scale_exp,
                  f"s{n}_hw_w1": s.hw_w1_scale_exp, f"s{n}_hw_w2": s.hw_w2_scale_exp})
        a.update({f"s{n}_local_out": s.local_out_scale_exp, f"s{n}_concat_out": s.concat_out_scale_exp,
                  f"s{n}_h1_out": s.h1_out_scale_exp, f"s{n}_h2_out": s.h2_out_scale_exp,
                  f"s{n}_logits_out": s.logits_out_scale_exp, f"s{n}_stats_out": s.stats_out_scale_exp,
                  f"s{n}_hw_hidden_out": s.hw_hidden_out_scale_exp})
    return {"weights": w, "activations": a}


def scale_table_json(table):
    """ScaleTable.save text: sorted keys, two-space indent, trailing newline."""
    payload = {"weights": {k: table["weights"][k] for k in sorted(table["weights"])},
               "activations": {k: table["activations"][k] for k in sorted(table["activations"])}}
    return json.dumps(payload, indent=2) + "\n"


def load_scale_table(text):
    raw = json.loads(text)
    if not isinstance(raw, dict):
        raise ValueError("scale table root must be an object")
    return {"weights": dict(raw.get("weights") or {}), "activations": dict(raw.get("activations") or {})}


def read_weights(raw, table):
    """A pruned HeatViTParams from a weight image and its scale table
    (p2_export_weights.golden_params_from_real with integer tensors)."""
    return params_from_tensors(_arrays(raw), table)


def params_from_tensors(tensors, table, selectors=3):
    """HeatViTParams from named integer tensors (the weight layout's names:
    patch_w, b<n>_wqkv, s<s>_local_w, ...) and a scale table; ``selectors=0``
    gives the unpruned model and needs no selector tensors or exponents."""
    t = {}
    for name, off, shape, esz in weight_layout():
        if name.startswith("s") and name[1].isdigit() and int(name[1]) > selectors:
            continue
        a = np.asarray(tensors[name])
        if a.size != int(np.prod(shape)):
            raise ValueError(f"{name}: {a.size} values, the layout holds {int(np.prod(shape))}")
        lo, hi = (-(1 << 31), (1 << 31) - 1) if esz == 4 else (-128, 127)
        if a.size and (int(a.min()) < lo or int(a.max()) > hi):
            raise ValueError(f"{name}: values outside the int{8 * esz} range")
        t[name] = a.reshape(shape).astype(np.int32 if esz == 4 else np.int8)
    wt, act = table["weights"], table["activations"]

    def block_in(n):
        return act["act_tokens"] if n == 1 else act[f"b{n - 1}_out"]

    patch = PatchParams(patch_weight=t["patch_w"], patch_bias=t["patch_b"], cls=t["cls"], pos=t["pos"],
                        image_scale_exp=act["input"], weight_scale_exp=wt["patch_w"],
                        activation_scale_exp=act["act_patch_embed"], tokens_scale_exp=act["act_tokens"],
                        cls_scale_exp=wt["cls"], pos_scale_exp=wt["pos"])
    blocks = []
    for n in range(1, 13):
        mhsa = MhsaParams(ln_gamma=t[f"b{n}_gamma1"], ln_beta=t[f"b{n}_beta1"], wqkv=t[f"b{n}_wqkv"],
                          bqkv=t[f"b{n}_bqkv"], wproj=t[f"b{n}_wproj"], bproj=t[f"b{n}_bproj"],
                          x_scale_exp=block_in(n), gamma1_scale_exp=wt[f"b{n}_gamma1"],
                          beta1_scale_exp=wt[f"b{n}_beta1"], ln1_out_scale_exp=act[f"b{n}_ln1_out"],
                          wqkv_scale_exp=wt[f"b{n}_wqkv"], qkv_out_scale_exp=act[f"b{n}_qkv_out"],
                          score_scale_exp=2 * act[f"b{n}_qkv_out"] - 3, prob_scale_exp=-8,
                          context_out_scale_exp=act[f"b{n}_context_out"], wproj_scale_exp=wt[f"b{n}_wproj"],
                          msa_out_scale_exp=act[f"b{n}_msa_out"])
        ffn = FfnParams(ln_gamma=t[f"b{n}_gamma2"], ln_beta=t[f"b{n}_beta2"], w1=t[f"b{n}_w1"], b1=t[f"b{n}_b1"],
                        w2=t[f"b{n}_w2"], b2=t[f"b{n}_b2"], x_scale_exp=act[f"b{n}_y"],
                        gamma2_scale_exp=wt[f"b{n}_gamma2"], beta2_scale_exp=wt[f"b{n}_beta2"],
                        ln2_out_scale_exp=act[f"b{n}_ln2_out"], w1_scale_exp=wt[f"b{n}_w1"],
                        hidden_out_scale_exp=act[f"b{n}_hidden"], w2_scale_exp=wt[f"b{n}_w2"],
                        ffn_out_scale_exp=act[f"b{n}_ffn_out"], out_scale_exp=act[f"b{n}_out"])
        blocks.append(BlockParams(mhsa=mhsa, ffn=ffn))
    sels = []
    for s in range(1, selectors + 1):
        sels.append(SelectorParams(
            local=SelectorLocalParams(w=t[f"s{s}_local_w"], b=t[f"s{s}_local_b"]),
            score=SelectorScoreParams(w1=t[f"s{s}_score_w1"], b1=t[f"s{s}_score_b1"], w2=t[f"s{s}_score_w2"],
                                      b2=t[f"s{s}_score_b2"], w3=t[f"s{s}_score_w3"], b3=t[f"s{s}_score_b3"]),
            head_weight=SelectorHeadWeightParams(w1=t[f"s{s}_hw_w1"], b1=t[f"s{s}_hw_b1"], w2=t[f"s{s}_hw_w2"],
                                                 b2=t[f"s{s}_hw_b2"]),
            in_scale_exp=act[f"b{3 * s}_out"], local_w_scale_exp=wt[f"s{s}_local_w"],
            local_out_scale_exp=act[f"s{s}_local_out"], concat_out_scale_exp=act[f"s{s}_concat_out"],
            score_w1_scale_exp=wt[f"s{s}_score_w1"], score_w2_scale_exp=wt[f"s{s}_score_w2"],
            score_w3_scale_exp=wt[f"s{s}_score_w3"], h1_out_scale_exp=act[f"s{s}_h1_out"],
            h2_out_scale_exp=act[f"s{s}_h2_out"], logits_out_scale_exp=act[f"s{s}_logits_out"],
            stats_out_scale_exp=act[f"s{s}_stats_out"], hw_w1_scale_exp=wt[f"s{s}_hw_w1"],
            hw_hidden_out_scale_exp=act[f"s{s}_hw_hidden_out"], hw_w2_scale_exp=wt[f"s{s}_hw_w2"]))
    return HeatViTParams(patch=patch, blocks=tuple(blocks), selectors=tuple(sels),
                         selector_blocks=(4, 7, 10)[:selectors],
                         final_gamma=t["final_gamma"], final_beta=t["final_beta"], head_w=t["head_w"],
                         head_b=t["head_b"], final_gamma_scale_exp=wt["final_gamma"],
                         final_beta_scale_exp=wt["final_beta"], final_ln_out_scale_exp=act["final_ln_out"],
                         head_w_scale_exp=wt["head_w"])
