"""The reference's end-to-end vector set, written from a CUDA inference.

tools/generate_e2e_vectors.py freezes, for one image, what the RTL testbench
checks a run against: four region images (input, weights, zeroed scratch and
output), the 18 golden checkpoints in descriptor order with the address each
one is found at, a JSON manifest and a SystemVerilog constants package.  This
module produces the same files, byte for byte, from a ``ModelResult`` (one image)
or from the batched engine's checkpoint tensors, so every image of a CUDA batch
can be cross-checked against an XSim log.

* Regions (tools/generate_e2e_vectors.py:31-34): input at 0, weights at
  0x01000000, scratch at 0x02000000, output at 0x03000000 (1000 int32 logits).
* Scratch (tools/generate_descriptors.py:104-152 ``build_memory_map``): two
  activation slots of 197 x 192 bytes (BUF0 at 0, BUF1 after it), then each
  operator buffer at the next 8-byte boundary; the final LayerNorm output is the
  last of them.
* Checkpoints (tools/generate_e2e_vectors.py:189-227 ``checkpoint_layout``): the
  patch embedding in BUF0; in each stage of three blocks the first and third
  block write BUF1 and the second BUF0; selector outputs in BUF0; the final LN in
  its own buffer; the logits at the start of the output region.  A checkpoint's
  descriptor index is the last descriptor of its stage in the schedule: the
  patch stage ends at descriptor 2, a block takes 13 descriptors, a selector 12,
  the final LN and the head one each.
* Files (tools/generate_e2e_vectors.py:318-420 ``generate``): ``.mem`` text of
  each image and checkpoint (int8 rows, int32 little-endian logits), the manifest
  (``json.dump`` with two-space indent and a trailing newline; checkpoint
  entries ascending by descriptor index, each with the SHA-256 of its ``.mem``
  file) and ``e2e_tb_config.sv`` (:423-488).

The descriptor ROM and the error-injection ROMs belong to the accelerator's
control schedule and are not written; the manifest carries the ROM's digest.
"""

import hashlib
import json
import os

import numpy as np

from . import abi, memimage

INPUT_BASE = 0x00000000
WEIGHT_BASE = 0x01000000
SCRATCH_BASE = 0x02000000
OUTPUT_BASE = 0x03000000
OUTPUT_BYTES = abi.CLASSES * 4
PART = "xc7k325tfbg900-3"
GENERATOR = "tools/generate_e2e_vectors.py"
# rtl/generated/heatvit_descriptors.mem of the reference: the descriptor
# schedule the vectors are run with (the manifest records its digest).
DESCRIPTOR_ROM_SHA256 = "fb82d49c25b82764e45e9750c1dd7a8b3461dcc22aa83d7a8691254073633509"
# The testbench's hang bound, a calibrated constant of the reference
# (4x the worst measured end-to-end cycle count, rounded up).
WATCHDOG_CYCLES = 850_000_000

ACT_SLOT = abi.TOKENS * abi.EMBED
_N = abi.TOKENS
_C = abi.TOKENS - 1

# Operator buffers after the two activation slots, in allocation order.
_SCRATCH_BUFFERS = (
    ("patch_matrix", 196 * 768), ("patch_embed", 196 * 192),
    ("block_ln1", _N * 192), ("block_fused", _N * 576), ("block_qkv", 3 * 3 * _N * 64),
    ("block_score", 3 * _N * _N * 4), ("block_prob", 3 * _N * _N), ("block_context", 3 * _N * 64),
    ("block_concat", _N * 192), ("block_msa", _N * 192), ("block_y", _N * 192), ("block_ln2", _N * 192),
    ("block_hidden", _N * 768), ("block_ffn_out", _N * 192),
    ("sel_local", 3 * _C * 32), ("sel_global", 96), ("sel_concat", 3 * _C * 64), ("sel_h1", 3 * _C * 32),
    ("sel_h2", 3 * _C * 16), ("sel_logits", 3 * _C * 2), ("sel_keep", 3 * _C * 4), ("sel_stats", _C * 3),
    ("sel_hw_hidden", _C * 3), ("sel_hw", _C * 12), ("sel_fused", _C * 4),
    ("final_ln", _N * 192),
)

# Descriptors per schedule stage: the patch stage ends at index 2.
_PATCH_LAST_DESC = 2
_BLOCK_DESCS = 13
_SELECTOR_DESCS = 12

CHECKPOINT_NAMES = (
    "patch", "block_01", "block_02", "block_03", "selector_01", "block_04", "block_05", "block_06",
    "selector_02", "block_07", "block_08", "block_09", "selector_03", "block_10", "block_11", "block_12",
    "final_ln", "logits",
)


def _align8(v):
    return (v + 7) & ~7


def scratch_layout():
    """{buffer name: offset} of the scratch region plus its 8-byte aligned size
    under ``"bytes"``."""
    out = {"buf0": 0, "buf1": ACT_SLOT}
    cur = 2 * ACT_SLOT
    for name, size in _SCRATCH_BUFFERS:
        out[name] = _align8(cur)
        cur = out[name] + size
    out["bytes"] = _align8(cur)
    return out


def checkpoint_layout(token_counts):
    """The 18 checkpoints in descriptor order: dicts with name, desc_index,
    region, offset (within the region), bytes and scale_exp.

    ``token_counts`` = [197, n1, n2, n3], the rows entering each stage."""
    tc = [int(v) for v in token_counts]
    if len(tc) != 4:
        raise ValueError("the vector set describes the three-selector model: token_counts = [197, n1, n2, n3]")
    scr = scratch_layout()
    out = []
    idx = _PATCH_LAST_DESC

    def add(name, region, offset, nbytes, scale):
        out.append({"name": name, "desc_index": idx, "region": region, "offset": offset, "bytes": nbytes,
                    "scale_exp": scale})

    add("patch", "scratch", scr["buf0"], tc[0] * 192, -7)
    for stage in range(4):
        if stage:
            idx += _SELECTOR_DESCS
            add(f"selector_{stage:02d}", "scratch", scr["buf0"], tc[stage] * 192, -7)
        for j in range(3):
            b = 3 * stage + j + 1
            idx += _BLOCK_DESCS
            add(f"block_{b:02d}", "scratch", scr["buf0"] if j == 1 else scr["buf1"], tc[stage] * 192, -7)
    idx += 1
    add("final_ln", "scratch", scr["final_ln"], tc[3] * 192, -7)
    idx += 1
    add("logits", "output", 0, OUTPUT_BYTES, abi.LOGIT_SCALE_EXP)
    return out


def _ck_bytes(entry, data):
    raw = np.ascontiguousarray(data).tobytes()
    if len(raw) > entry["bytes"]:
        raise ValueError(f"checkpoint {entry['name']} holds {len(raw)} bytes, its slot {entry['bytes']}")
    return raw + b"\0" * (entry["bytes"] - len(raw))


def checkpoint_images(checkpoints, token_counts):
    """{name: bytes} of the 18 checkpoints from golden-form checkpoints
    (``ModelResult.checkpoints``: name -> rows of 192 int8 values, "logits" ->
    1000 int32 values)."""
    out = {}
    for e in checkpoint_layout(token_counts):
        v = checkpoints[e["name"]]
        a = np.asarray(v, "<i4") if e["name"] == "logits" else np.asarray(v, np.int64).astype(np.int8)
        out[e["name"]] = _ck_bytes(e, a)
    return out


def checkpoint_images_from_slots(ck, rows, logits, token_counts):
    """{name: bytes} from one image's checkpoint slots (the [26, 197, 192] int8
    array and [26] row counts of include/heatvit_b200.h) and its logits."""
    ck = np.asarray(ck)
    rows = np.asarray(rows)
    slot = {"patch": abi.CKPT_PATCH, "final_ln": abi.CKPT_FINAL_LN}
    slot.update({f"block_{b:02d}": abi.ckpt_block(b) for b in range(1, 13)})
    slot.update({f"selector_{s:02d}": abi.ckpt_selector(s) for s in range(1, 4)})
    out = {}
    for e in checkpoint_layout(token_counts):
        if e["name"] == "logits":
            out["logits"] = _ck_bytes(e, np.asarray(logits, "<i4"))
            continue
        k = slot[e["name"]]
        r = int(rows[k])
        if r * 192 != e["bytes"]:
            raise ValueError(f"checkpoint {e['name']} has {r} rows, the token counts give {e['bytes'] // 192}")
        out[e["name"]] = _ck_bytes(e, ck[k, :r])
    return out


def checkpoint_images_batch(out):
    """Per-image dicts {"token_counts", "checkpoints": {name: bytes},
    "selector_summary": [dict] * 3} from the output of
    ``Engine.infer(images, checkpoints=True)`` on a three-selector model (one
    device-to-host copy of the checkpoint tensors for the batch)."""
    ck = out["checkpoints"].cpu().numpy()
    rows = out["checkpoint_rows"].cpu().numpy()
    logits = out["logits"].cpu().numpy()
    counts = out["token_counts"].cpu().numpy()
    summ = out["summary"].cpu().numpy()
    if counts.shape[1] != 4:
        raise ValueError("the vector set describes the three-selector model")
    res = []
    for i in range(ck.shape[0]):
        tc = [int(v) for v in counts[i]]
        res.append({"token_counts": tc, "checkpoints": checkpoint_images_from_slots(ck[i], rows[i], logits[i], tc),
                    "selector_summary": [dict(zip(abi.SUMMARY_FIELDS[:5], (int(v) for v in s[:5])))
                                         for s in summ[i]]})
    return res


def selector_entries(calibration, selector_summary, seed=20260815):
    """The manifest's "selectors" list (weights.py:191-201 key order) from a
    run's selector summaries (input_tokens, output_tokens, kept_normal,
    pruned_normal, package_present) and, for a calibrated model, the calibration
    outcome [(attempt, median_logit_diff)] * 3; ``calibration=None`` leaves out
    the attempt, seed and median keys."""
    out = []
    for stage, s in enumerate(selector_summary, 1):
        e = {"stage": stage}
        if calibration is not None:
            attempt, median = calibration[stage - 1]
            e.update(attempt=int(attempt), seed=seed + stage * 1000 + int(attempt), median_logit_diff=int(median))
        e.update({k: int(s[k]) for k in ("input_tokens", "output_tokens", "kept_normal", "pruned_normal",
                                         "package_present")})
        out.append(e)
    return out


def _sha(b):
    return hashlib.sha256(b).hexdigest()


def vector_files(image, params, ck_images, token_counts, selectors, seed=20260815,
                 descriptor_rom_sha256=DESCRIPTOR_ROM_SHA256, generator=GENERATOR):
    """{relative path: bytes} of the vector set: input.mem, weights.mem,
    scratch_init.mem, output_init.mem, checkpoints/<name>.mem, manifest.json and
    e2e_tb_config.sv.  ``ck_images`` comes from one of the ``checkpoint_images``
    functions; ``selectors`` from ``selector_entries``."""
    img = np.asarray(image, np.int64).astype(np.int8).reshape(-1)
    if img.size != abi.IMAGE_BYTES:
        raise ValueError("image length mismatch")
    wbytes = memimage.weight_bytes()
    scr = scratch_layout()
    files = {
        "input.mem": memimage.mem_lines(img.tobytes()).encode(),
        "weights.mem": memimage.mem_lines(memimage.write_weights(params)).encode(),
        "scratch_init.mem": memimage.mem_lines(bytes(scr["bytes"])).encode(),
        "output_init.mem": memimage.mem_lines(bytes(OUTPUT_BYTES)).encode(),
    }
    entries = []
    for e in checkpoint_layout(token_counts):
        data = memimage.mem_lines(ck_images[e["name"]]).encode()
        files[f"checkpoints/{e['name']}.mem"] = data
        entries.append(dict(e, sha256=_sha(data)))
    entries.sort(key=lambda c: c["desc_index"])
    manifest = {
        "seed": seed,
        "part": PART,
        "generator": generator,
        "descriptor_rom_sha256": descriptor_rom_sha256,
        "regions": {
            "input": {"base": INPUT_BASE, "bytes": _align8(img.size), "valid_bytes": img.size},
            "weight": {"base": WEIGHT_BASE, "bytes": _align8(wbytes), "valid_bytes": wbytes},
            "scratch": {"base": SCRATCH_BASE, "bytes": scr["bytes"], "valid_bytes": scr["bytes"]},
            "output": {"base": OUTPUT_BASE, "bytes": OUTPUT_BYTES, "valid_bytes": OUTPUT_BYTES},
        },
        "checkpoints": entries,
        "selectors": list(selectors),
        "token_counts": [int(v) for v in token_counts],
        "output_scale_exp": abi.LOGIT_SCALE_EXP,
        "watchdog_cycles": WATCHDOG_CYCLES,
        "files": {k: _sha(files[k]) for k in ("input.mem", "weights.mem", "scratch_init.mem", "output_init.mem")},
    }
    files["manifest.json"] = (json.dumps(manifest, indent=2) + "\n").encode()
    files["e2e_tb_config.sv"] = tb_config_sv(manifest).encode()
    return files


def tb_config_sv(manifest):
    """The SystemVerilog constants package of a manifest
    (tools/generate_e2e_vectors.py:423-488)."""
    reg, tc, cps = manifest["regions"], manifest["token_counts"], manifest["checkpoints"]
    last = len(cps) - 1

    lines = ["`ifndef E2E_TB_CONFIG_PKG_SV", "`define E2E_TB_CONFIG_PKG_SV", "",
             f"// Generated by {GENERATOR}; do not edit.", "package e2e_tb_config_pkg;", ""]
    for name, label in (("input", "INPUT"), ("weight", "WEIGHT"), ("scratch", "SCRATCH"), ("output", "OUTPUT")):
        lines += [f"  localparam logic [31:0] {label + '_BASE':<12} = 32'h{reg[name]['base']:08x};",
                  f"  localparam int          {label + '_BYTES':<12} = {reg[name]['bytes']};"]
    lines += [f"  localparam int WATCHDOG_CYCLES = {manifest['watchdog_cycles']};",
              f"  localparam int OUTPUT_SCALE_EXP = {manifest['output_scale_exp']};", "",
              f"  localparam int SELECTOR_IN_N [0:2] = '{{{tc[0]}, {tc[1]}, {tc[2]}}};",
              f"  localparam int SELECTOR_OUT_N [0:2] = '{{{tc[1]}, {tc[2]}, {tc[3]}}};"]
    pk = [e["package_present"] for e in manifest["selectors"]]
    lines += [f"  localparam int SELECTOR_PACKAGE [0:2] = '{{{pk[0]}, {pk[1]}, {pk[2]}}};", "",
              f"  localparam int CHECKPOINT_DESC_INDEX [0:{last}] = '{{"
              + ", ".join(str(c["desc_index"]) for c in cps) + "};",
              f"  localparam logic [31:0] CHECKPOINT_OFFSET [0:{last}] = '{{"]
    addrs = [f"      32'h{reg[c['region']]['base'] + c['offset']:08x}" for c in cps]
    lines += [a + "," for a in addrs[:-1]] + [addrs[-1], "  };"]
    lines += [f"  localparam int CHECKPOINT_BYTES [0:{last}] = '{{" + ", ".join(str(c["bytes"]) for c in cps) + "};",
              f"  localparam logic signed [5:0] CHECKPOINT_SCALE [0:{last}] = '{{"]
    scales = [f"      -6'sd{-c['scale_exp']}" for c in cps]
    lines += [s + "," for s in scales[:-1]] + [scales[-1], "  };", "", "endpackage", "", "`endif"]
    return "\n".join(lines) + "\n"


def write_vector_files(outdir, files):
    """Write ``vector_files`` output under ``outdir``."""
    for rel, data in files.items():
        path = os.path.join(outdir, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "wb") as f:
            f.write(data)
