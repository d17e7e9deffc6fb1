#!/usr/bin/env python3
"""Throughput benchmark: batched pruned int8 DeiT-T (HeatViT) on B200.

One step = the full fused pipeline (patch embedding, 12 blocks, 3 token
selectors with ragged compaction, final LN, head) over one per-GPU batch of
seeded synthetic images already resident in HBM, followed (N > 1) by the
gather of logits, token counts and warnings to rank 0 (on a side stream,
overlapped with the next step).  Weak scaling: every rank processes
``--batch`` images per step (default 1024).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  Besides the config-4 headline it carries:
  * ``config3``: the north-star configuration (pruned, 256 images, 1 GPU);
  * ``parity``: the timed step's outputs against the CPU oracle, bit for bit;
  * ``roofline`` (dominant kernel) and ``stages`` (every kernel of a step);
  * ``e2e``: the same metric through the host-buffer API, plus the ceiling of
    plain pinned host-to-device copies run at the same time on every rank.
``--impl reference`` times the reference algorithm's CPU implementation (the
C restatement in oracle/, since the reference is a Python golden model that
cannot travel) on the host cores.
"""

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "images/sec pruned int8 DeiT-T @1/2/4/8 B200, bit-exact logits; % int8 roofline"
INT8_SPEC_TOPS = 4500.0      # B200 dense int8 (NVIDIA datasheet, non-sparse)
HBM_SPEC_GBS = 8000.0
WEIGHT_BYTES = 5_830_000     # int8 weights + biases + LN + pos + selectors
STAGES = {"ln1": 1, "qkv": 2, "attn": 3, "proj": 4, "ln2": 5, "fc1": 6, "fc2": 7, "selector": 8, "patch": 9,
          "head": 10, "ffn": 11}
# GEMM stages: (K, N, residual bytes per row).  Algorithmic ops per row 2*K*N; HBM
# bytes per row K (A) + N (output) + residual, plus the weights once per launch.
GEMM_SHAPES = {"qkv": (192, 576, 0), "proj": (192, 192, 192), "fc1": (192, 768, 0), "fc2": (768, 192, 192),
               "patch": (768, 192, 192), "head": (192, 1000, 0)}
# DRAM bytes (read + write) per live row of one launch, from full-size ncu captures
# (profiles/): block 1 of a 1024-image step, 201,728 rows (dram__bytes_read.sum +
# dram__bytes_write.sum).  Traffic grows with the rows of a launch.
STAGE_TRAFFIC_PER_ROW = {"ffn": (77_869_824 + 11_407_360) / 201_728,
                         "attn": (116_336_896 + 17_401_088) / 201_728,
                         "ln1": (38_799_616 + 1_387_776) / 201_728}


# The reference's own implementation is the pure-Python golden model.  Its sources are
# not part of this repository and are not present where the benchmark runs, so the
# timed CPU legs run the C restatement; the golden model's single-core rate was
# measured where the reference is installed.
GOLDEN_PYTHON_NOTE = ("not timed here: verification/heatvit_ref is not present on the benchmark host (its "
                      "sources are not copied into this repository); measured where it is installed: "
                      "13.6 s per pruned image on one core (HeatViTModel.infer)")


def algorithmic_macs(counts):
    """Reference MAC convention (tools/p8/_perf_common.py:88-123): patch +
    per block 442368*N + 384*N^2 + selectors 13938*C + head, per image."""
    counts = np.asarray(counts, np.int64)
    macs = np.full(counts.shape[0], 28_901_376 + 192_000, np.int64)
    for b, col, sel in block_columns(counts.shape[1] - 1):
        if sel is not None:
            macs += 13_938 * (counts[:, sel] - 1)
        n = counts[:, col]
        macs += 442_368 * n + 384 * n * n
    return macs


def block_columns(ns):
    """(block, token-count column, column of the selector input or None) per block."""
    sel_before = {4: 1, 7: 2, 10: 3} if ns == 3 else {}
    out, col = [], 0
    for b in range(1, 13):
        sel = None
        if b in sel_before:
            sel = col
            col = sel_before[b]
        out.append((b, col, sel))
    return out


def stage_work(stage, counts, launches_per_step):
    """Algorithmic (ops, bytes) of the first ``launches_per_step`` launches of a
    stage in one step over images with these token counts."""
    counts = np.asarray(counts, np.int64)
    b = counts.shape[0]
    cols = block_columns(counts.shape[1] - 1)
    if stage == "patch":
        k, n, r = GEMM_SHAPES["patch"]
        return 2.0 * b * 196 * k * n, float(b * (150528 + 197 * 192) + k * n)
    if stage == "head":
        k, n, _ = GEMM_SHAPES["head"]
        return 2.0 * b * k * n, float(b * (192 + 4 * n) + k * n)
    if stage == "selector":
        sels = [(s, c) for _, c, s in cols if s is not None][:launches_per_step]
        ops = sum(2.0 * 13_938 * float((counts[:, s] - 1).sum()) for s, _ in sels)
        byt = sum(float(counts[:, s].sum() + counts[:, c].sum()) * 192 for s, c in sels)
        return ops, byt
    ops = byt = 0.0
    for _, col, _ in cols[:launches_per_step]:
        n = counts[:, col]
        rows = float(n.sum())
        if stage in GEMM_SHAPES:
            k, nn, r = GEMM_SHAPES[stage]
            ops += 2.0 * rows * k * nn
            byt += rows * (k + nn + r) + k * nn
        elif stage == "ffn":  # FC1 + FC2 fused: LN2 rows and the residual in, block output out
            ops += 2.0 * rows * 2 * 192 * 768
            byt += rows * (192 + 192 + 192) + 2 * 192 * 768
        elif stage == "attn":
            ops += float((3 * 4 * 64 * n * n).sum())   # QK^T and P.V per head
            byt += rows * (576 + 192)                   # Q, K, V in; context out
        else:  # ln1 / ln2
            byt += rows * 384
    return ops, byt


def roofline_of(stage, ms, ops, byt, int8_tops, hbm, traffic_rows=None):
    """The slower of ops at the int8 peak and bytes at HBM bandwidth binds."""
    t_tensor = ops / (int8_tops * 1e12) if ops else 0.0
    t_hbm = byt / (hbm * 1e9)
    sec = ms * 1e-3
    tensor = {"achieved": ops / sec / 1e12 if ops else 0.0, "peak": int8_tops, "unit": "TOPS",
              "frac": t_tensor / sec, "frac_of_spec": (ops / (INT8_SPEC_TOPS * 1e12)) / sec}
    mem = {"achieved": byt / sec / 1e9, "peak": hbm, "unit": "GB/s", "frac": t_hbm / sec,
           "frac_of_spec": (byt / (HBM_SPEC_GBS * 1e9)) / sec}
    bound = "tensor" if t_tensor > t_hbm else "hbm"
    main = tensor if bound == "tensor" else mem
    out = {"bound": bound, "achieved": main["achieved"], "peak": main["peak"], "unit": main["unit"],
           "frac": main["frac"], "frac_of_spec": main["frac_of_spec"],
           "traffic": traffic_rows, "ms": ms, "tensor": tensor, "hbm": mem}
    return out


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


def measure_int8_tops(torch):
    """Dense int8 tensor throughput of this GPU via cuBLASLt (torch._int_mm)."""
    try:
        n = 8192
        a = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
        b = torch.randint(-128, 127, (n, n), dtype=torch.int8, device="cuda")
        for _ in range(3):
            torch._int_mm(a, b)
        torch.cuda.synchronize()
        best = 1e9
        for _ in range(10):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch._int_mm(a, b)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12, "measured torch._int_mm 8192^3 (cuBLASLt), best of 10"
    except Exception as exc:  # pragma: no cover - depends on the box
        return INT8_SPEC_TOPS, f"spec (int8 measurement failed: {type(exc).__name__})"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.lines = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def physical_gpu_index(torch, local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import hv_oracle
    hv_oracle.build()
    return hv_oracle


def cpu_oracle_rate(params, images, target_s=15.0, max_images=4096):
    """Images/s of the oracle (C restatement of the golden model) on all host
    threads over a bounded sample sized for about ``target_s`` seconds.  The
    sample is the step's own images, cycled when it needs more than one batch.
    Also returns the oracle's outputs for the first min(sample, batch) images."""
    hv_oracle = _oracle()
    threads = hv_oracle.num_cpus()
    probe = min(images.shape[0], max(2 * threads, 8))
    t0 = time.perf_counter()
    hv_oracle.infer_batch(params, images[:probe], threads=threads)
    dt = time.perf_counter() - t0
    rate = probe / dt
    n = int(min(max_images, max(probe, rate * target_s)))
    sample = images[np.arange(n) % images.shape[0]]
    t0 = time.perf_counter()
    ref = hv_oracle.infer_batch(params, sample, threads=threads)
    dt = time.perf_counter() - t0
    k = min(n, images.shape[0])
    ref = {key: ref[key][:k] for key in ("logits", "counts", "warnings")}
    return n / dt, threads, n, dt, ref


def parity_check(params, seed, logits, counts, warnings, ref=None, sample=256, rng_seed=7):
    """Bit-exact comparison of a step's outputs (all images of the job, in image
    order) with the CPU oracle.  ``ref`` holds oracle outputs for the first
    images already; the rest of the check covers a seeded sample of ``sample``
    images plus every image whose package denominator was zero (warning bit 1)."""
    from heatvit_b200 import synth
    total = logits.shape[0]
    covered = 0 if ref is None else ref["logits"].shape[0]
    idx = set()
    if covered < total:
        rng = np.random.default_rng(rng_seed)
        pool = np.arange(covered, total)
        idx.update(int(i) for i in rng.choice(pool, size=min(sample, pool.size), replace=False))
        idx.update(int(i) for i in np.nonzero(warnings[covered:] & 2)[0] + covered)
    idx = sorted(idx)
    mism = 0
    checked = covered
    zero_den = 0
    if covered:
        g = slice(0, covered)
        bad = (np.any(logits[g] != ref["logits"], axis=1) | np.any(counts[g] != ref["counts"], axis=1) |
               (warnings[g] != ref["warnings"]))
        mism += int(bad.sum())
        zero_den += int(((ref["warnings"] & 2) != 0).sum())
    if idx:
        hv_oracle = _oracle()
        imgs = np.concatenate([synth.baseline_images(seed, 1, first=i) for i in idx])
        r = hv_oracle.infer_batch(params, imgs, threads=hv_oracle.num_cpus())
        bad = (np.any(logits[idx] != r["logits"], axis=1) | np.any(counts[idx] != r["counts"], axis=1) |
               (warnings[idx] != r["warnings"]))
        mism += int(bad.sum())
        checked += len(idx)
        zero_den += int(((r["warnings"] & 2) != 0).sum())
    return {"checked": checked, "mismatches": mism, "zero_den_images_checked": zero_den,
            "of": int(total), "fields": "logits, token counts, warning bits",
            "oracle": "C restatement of verification/heatvit_ref (oracle/)"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from heatvit_b200 import synth
    hv_oracle = _oracle()
    params = bench_params(synth, args.variant)
    threads = hv_oracle.num_cpus()
    per_step = max(4 * threads, 16)
    imgs = synth.baseline_images(synth.SEED, per_step)
    for _ in range(args.warmup):
        hv_oracle.infer_batch(params, imgs[:threads], threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        hv_oracle.infer_batch(params, imgs, threads=threads)
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt
    line = {
        "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8/int32", "data": "synthetic",
        "config": {"workload": f"config4-{args.variant}: batch {args.batch}/GPU, 224x224x3 int8 images, "
                               "seeded benchmark DeiT-T (heatvit_b200.synth." + PARAMS_FN[args.variant] + ")",
                   "per_step_sample_images": per_step,
                   "note": "a bounded per-step sample (the first images of the batch) on the host cores; "
                           "images/s is independent of the sample size"},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} seeded images per step, {args.steps} steps, C restatement of "
                                   "verification/heatvit_ref on all host threads",
                         "golden_python": GOLDEN_PYTHON_NOTE},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Config 4 runs the benchmark model unpruned, or pruned with config 3's selectors.
PARAMS_FN = {"pruned": "config3_params", "unpruned": "config_params(pruned=False)"}


def bench_params(synth, variant):
    if variant == "pruned":
        return synth.config3_params(synth.SEED)
    return synth.config_params(synth.SEED, pruned=False)


def _lib_call(fn, *a):
    from heatvit_b200 import _lib
    _lib.check(fn(*a))


def time_steps(torch, step, steps, world, barrier=None):
    """Device time of ``steps`` calls of ``step`` on the current stream (CUDA
    events, synchronised on both sides), max over ranks."""
    import torch.distributed as dist
    stream = torch.cuda.current_stream()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    if barrier is not None:
        barrier()
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def stage_breakdown(torch, eng, step, counts, int8_tops, hbm, launches_of):
    """Per-kernel time of one step: for each stage, a short run with CUDA events
    around every launch of that stage, then the algorithmic roofline of those
    launches (the slower of ops at the int8 peak and bytes at HBM)."""
    from heatvit_b200 import _lib
    L = _lib.lib()
    out = {}
    for name, sid in STAGES.items():
        n = launches_of[name]
        if n == 0:
            continue
        _lib.check(L.hv_profile_start(eng.handle, sid, n))
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        launches, kms, krows = C.c_int(), C.c_double(), C.c_longlong()
        _lib.check(L.hv_profile_stop(eng.handle, C.byref(launches), C.byref(kms), C.byref(krows)))
        if launches.value == 0:
            continue
        ops, byt = stage_work(name, counts, launches.value)
        r = roofline_of(name, kms.value, ops, byt, int8_tops, hbm)
        out[name] = {"ms_per_step": kms.value, "launches": launches.value, "bound": r["bound"],
                     "frac": r["frac"], "frac_of_spec": r["frac_of_spec"],
                     "tensor_frac": r["tensor"]["frac"], "hbm_frac": r["hbm"]["frac"],
                     "achieved": r["achieved"], "unit": r["unit"]}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1024, help="images per GPU per step")
    ap.add_argument("--variant", default="pruned", choices=["pruned", "unpruned"])
    ap.add_argument("--profile-stage", default="ffn", choices=sorted(STAGES))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the config-3 leg, the stage breakdown and the parity check")
    ap.add_argument("--e2e-steps", type=int, default=None, help="end-to-end steps (default: --steps)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.e2e_steps is None:
        args.e2e_steps = max(args.steps, 1)

    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist
    from heatvit_b200 import _lib, synth
    from heatvit_b200.engine import Engine
    from heatvit_b200.shard import RootGather, shard_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    L = _lib.lib()

    params = bench_params(synth, args.variant)
    eng = Engine(params)
    b = args.batch
    first, _ = shard_range(rank, world, b)
    host_imgs = synth.baseline_images(synth.SEED, b, first=first)
    imgs = torch.from_numpy(host_imgs).cuda()
    ns = eng.num_selectors
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)

    # Two output sets: step i writes set i % 2 while the gather of step i - 1 still
    # reads the other one; fence() orders a set's reuse after its gather.
    outs = [eng.alloc_outputs(b) for _ in range(2)]
    gat = RootGather(world, rank, outs[0]["packed"].numel(), torch.int32, torch.device("cuda", local))
    st = {"i": 0, "res": None, "buf": None}

    def step():
        o = outs[st["i"] % 2]
        st["i"] += 1
        gat.fence(o["packed"])
        eng.infer(imgs, out=o)
        st["res"] = gat.submit(o["packed"])
        st["buf"] = o

    # Block 1's launch of the profiled stage (the largest) is bracketed by CUDA
    # events inside the replayed graph; the warm-up captures that graph, so the
    # timed steps only replay it.  One bracketed launch per step keeps the events
    # from breaking more than one programmatic-launch edge.
    _lib.check(L.hv_profile_start(eng.handle, STAGES[args.profile_stage], 1))
    for _ in range(args.warmup):
        step()
    gat.flush()
    torch.cuda.synchronize()
    counts_local = st["buf"]["token_counts"].cpu().numpy()

    sampler = ClockSampler(physical_gpu_index(torch, local)) if rank == 0 else None
    time.sleep(0.3 if sampler else 0)
    _lib.check(L.hv_profile_start(eng.handle, STAGES[args.profile_stage], 1))
    elapsed_ms = time_steps(torch, step, args.steps, world, barrier=gat.flush)
    launches, kms, krows = C.c_int(), C.c_double(), C.c_longlong()
    _lib.check(L.hv_profile_stop(eng.handle, C.byref(launches), C.byref(kms), C.byref(krows)))
    graph_kernels = C.c_int()
    _lib.check(L.hv_graph_kernels(eng.handle, C.byref(graph_kernels)))
    clocks = sampler.stop() if sampler else None
    ms_per_step = elapsed_ms / args.steps
    value = world * b / (ms_per_step * 1e-3)

    # The last timed step's outputs, gathered on rank 0 in image order.
    if rank == 0:
        if world > 1:
            rows = st["res"].cpu().numpy()
            parts = [Engine.unpack_outputs(rows[r], b, ns) for r in range(world)]
            g_logits = np.concatenate([p[0] for p in parts])
            g_counts = np.concatenate([p[1] for p in parts])
            g_warn = np.concatenate([p[2] for p in parts])
        else:
            g_logits = st["buf"]["logits"].cpu().numpy()
            g_counts = st["buf"]["token_counts"].cpu().numpy()
            g_warn = st["buf"]["warnings"].cpu().numpy()

    # Per-kernel breakdown of a step (every rank runs the same steps; no collective).
    stages = None
    launches_of = {"patch": 1, "head": 1, "selector": ns}
    for k in ("ln1", "qkv", "attn", "proj", "ln2", "fc1", "fc2", "ffn"):
        launches_of[k] = 12

    def local_step():
        eng.infer(imgs, out=outs[0])

    int8_tops, int8_src = measure_int8_tops(torch)
    if world == 1 and not args.no_extras:
        stages = stage_breakdown(torch, eng, local_step, counts_local, int8_tops, hbm, launches_of)

    # End-to-end through the public host API: pinned host images in, host logits out,
    # every step's upload and download inside the timed region.  Pipelined: the
    # serving loop keeps two calls in flight (hv_infer_host_submit / _wait), so a
    # step's upload runs during the previous step's compute.  Blocking: one
    # hv_infer_host call per step.
    def e2e_rates_for(n_img, steps):
        pinned = torch.empty((n_img, 150528), dtype=torch.int8, pin_memory=True)
        pinned.numpy()[:] = host_imgs[:n_img]
        host_logits = [torch.empty((n_img, 1000), dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]

        def e2e_pipelined(k):
            for i in range(k):
                eng.infer_host_submit(pinned.numpy(), host_logits[i % 2])
                if i:
                    eng.infer_host_wait()
            eng.infer_host_wait()

        def e2e_blocking(k):
            for _ in range(k):
                eng.infer_host(pinned.numpy(), logits=host_logits[0])

        rates = {}
        for name, fn in (("pipelined", e2e_pipelined), ("blocking", e2e_blocking)):
            # warm-up: enough calls that every (image buffer, workspace, chunk size)
            # combination has its CUDA graph captured before the timed calls
            fn(6)
            if world > 1:
                dist.barrier()
            t0 = time.perf_counter()
            fn(steps)
            e2e_s = (time.perf_counter() - t0) / steps
            if world > 1:
                t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                e2e_s = float(t.item())
            rates[name] = world * n_img / e2e_s
        return rates, pinned

    e2e_rates, pinned = e2e_rates_for(b, args.e2e_steps)

    # Ceiling of the upload alone: the same bytes as plain pinned host-to-device
    # copies, on every rank at the same time, max over ranks.
    dimg = torch.empty_like(imgs)
    for _ in range(2):
        dimg.copy_(pinned, non_blocking=True)
    reps = max(3, min(10, args.e2e_steps))
    h2d_ms = time_steps(torch, lambda: dimg.copy_(pinned, non_blocking=True), reps, world) / reps
    h2d_ceiling = world * b / (h2d_ms * 1e-3)
    del dimg

    # Config 3 (the north-star configuration): pruned, 256 images on one GPU.
    config3 = None
    if world == 1 and not args.no_extras:
        b3 = min(256, b)
        img3 = imgs[:b3]
        out3 = eng.alloc_outputs(b3)

        def step3():
            eng.infer(img3, out=out3)

        _lib.check(L.hv_profile_start(eng.handle, 0, 0))
        for _ in range(args.warmup):
            step3()
        torch.cuda.synchronize()
        steps3 = max(args.steps, 20)
        ms3 = time_steps(torch, step3, steps3, 1) / steps3
        c3 = out3["token_counts"].cpu().numpy()
        stages3 = stage_breakdown(torch, eng, step3, c3, int8_tops, hbm, launches_of)
        macs3 = algorithmic_macs(c3)
        t3 = 2 * float(macs3.sum()) / (int8_tops * 1e12)
        e2e3, _ = e2e_rates_for(b3, max(args.e2e_steps, 20))
        config3 = {
            "workload": "config3: pruned, batch 256 on 1 GPU, the same seeded images and model",
            "value": b3 / (ms3 * 1e-3), "unit": "images/s", "ms_per_step": ms3, "steps": steps3,
            "images": b3, "mean_token_counts": [float(v) for v in c3.mean(0)],
            "model_roofline": {"frac": t3 / (ms3 * 1e-3), "bound": "tensor",
                               "frac_of_spec": 2 * float(macs3.sum()) / (INT8_SPEC_TOPS * 1e12) / (ms3 * 1e-3)},
            "e2e": {"value": e2e3["pipelined"], "unit": "images/s", "h2d_bytes_per_step": b3 * 150528,
                    "d2h_bytes_per_step": b3 * 4000, "mode": "pipelined host calls",
                    "blocking_value": e2e3["blocking"]},
            "stages": stages3,
            "_logits": out3["logits"].cpu().numpy(), "_counts": c3,
            "_warn": out3["warnings"].cpu().numpy(),
        }

    if rank == 0:
        macs = algorithmic_macs(counts_local)
        macs_per_step = float(macs.mean()) * world * b
        t_compute = 2 * macs_per_step / (int8_tops * 1e12)
        bytes_step = world * b * (150528 + 4004) + WEIGHT_BYTES * world
        t_mem = bytes_step / (hbm * 1e9) / world
        model_frac = max(t_compute / world, t_mem) / (ms_per_step * 1e-3)
        ps = args.profile_stage
        kavg = kms.value / max(1, launches.value)
        rows_avg = krows.value / max(1, launches.value)
        ops1, byt1 = stage_work(ps, counts_local, 1)
        traffic = STAGE_TRAFFIC_PER_ROW[ps] * rows_avg if ps in STAGE_TRAFFIC_PER_ROW else None
        roof = roofline_of(ps, kavg, ops1, byt1, int8_tops, hbm, traffic)
        roof.update({"traffic_unit": "bytes per launch (DRAM read + write, ncu capture scaled by rows)",
                     "kernel": f"{ps}: block 1's launch in the last timed step, {kavg:.4f} ms, {rows_avg:.0f} rows",
                     "peak_source": {"tensor": int8_src, "hbm": "MEASURED_PEAKS.json hbm_gbs (of measured)"},
                     "work": "algorithmic ops and bytes of that launch (see stage_work)"})
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/int32", "data": "synthetic",
            "config": {"workload": f"config4-{args.variant}: batch {b}/GPU of seeded 224x224x3 int8 images, "
                                   "benchmark DeiT-T (synth." + PARAMS_FN[args.variant] + "), selectors before blocks 4/7/10",
                       "images_per_gpu": b, "parallelism": f"image-sharded x{world}",
                       "gather": "dist.gather to rank 0 on a side stream, overlapped with the next step"
                                 if world > 1 else "none",
                       "l2": "inputs larger than L2 (images 154 MB/GPU per step)",
                       "mean_token_counts": [float(v) for v in counts_local.mean(0)]},
            "roofline": roof,
            "model_roofline": {"frac": model_frac, "bound": "tensor" if t_compute / world > t_mem else "hbm",
                               "algorithmic_gmac_per_image": float(macs.mean()) / 1e9,
                               "int8_peak_tops": int8_tops, "int8_spec_tops": INT8_SPEC_TOPS,
                               "frac_of_spec": (2 * macs_per_step / (INT8_SPEC_TOPS * 1e12) / world)
                               / (ms_per_step * 1e-3)},
            "e2e": {"value": e2e_rates["pipelined"], "unit": "images/s", "h2d_bytes_per_step": b * 150528,
                    "d2h_bytes_per_step": b * 4000, "steps": args.e2e_steps,
                    "mode": "pipelined host calls (hv_infer_host_submit/_wait, two in flight)",
                    "blocking_value": e2e_rates["blocking"],
                    "h2d_ceiling": {"value": h2d_ceiling, "unit": "images/s",
                                    "ms_per_copy": h2d_ms, "bytes_per_copy": b * 150528,
                                    "how": "plain pinned host-to-device copy of one step's images, all ranks at "
                                           "once, max over ranks"},
                    "frac_of_h2d_ceiling": e2e_rates["pipelined"] / h2d_ceiling},
            # init + patch + 12 x 7 block kernels + 2 per selector + CLS LN + head, plus one
            # row-count copy per profiled launch
            "gpu_launches": graph_kernels.value * args.steps,
            "clocks": clocks,
        }
        if stages:
            line["stages"] = stages
        ref = None
        if world == 1 and not args.no_cpu_baseline:
            rate, threads, n, dt, ref = cpu_oracle_rate(params, host_imgs)
            line["cpu_baseline"] = {"value": rate, "unit": "images/s", "cores": threads, "kind": "port",
                                    "sample": f"{n} images (the step's batch, cycled) in {dt:.1f}s on "
                                              f"{threads} threads; C restatement of verification/heatvit_ref",
                                    "golden_python": GOLDEN_PYTHON_NOTE}
        if not args.no_extras:
            line["parity"] = parity_check(params, synth.SEED, g_logits, g_counts, g_warn, ref=ref)
            if config3 is not None:
                lg3, c3, w3 = config3.pop("_logits"), config3.pop("_counts"), config3.pop("_warn")
                k3 = lg3.shape[0]
                if ref is not None and ref["logits"].shape[0] >= k3:
                    r3 = {key: ref[key][:k3] for key in ("logits", "counts", "warnings")}
                else:
                    r3 = None
                config3["parity"] = parity_check(params, synth.SEED, lg3, c3, w3, ref=r3, sample=k3)
                line["config3"] = config3
        print(json.dumps(line), flush=True)
    if world > 1:
        gat.flush()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
