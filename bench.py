#!/usr/bin/env python3
"""Throughput benchmark: batched pruned int8 DeiT-T (HeatViT) on B200.

One step = the full fused pipeline (patch embedding, 12 blocks, 3 token
selectors with ragged compaction, final LN, head) over one per-GPU batch of
seeded synthetic images already resident in HBM, followed (N > 1) by the
gather of logits and token counts.  Weak scaling: every rank processes
``--batch`` images per step (default 1024).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line on rank 0.  ``--impl reference`` times the reference
algorithm's CPU implementation (the C restatement in oracle/, since the
reference is a Python golden model that cannot travel) on the host cores.
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
          "head": 10}
# Algorithmic MACs per row of each GEMM stage (rows = live tokens of the launch).
STAGE_MACS_PER_ROW = {"qkv": 192 * 576, "proj": 192 * 192, "fc1": 192 * 768, "fc2": 768 * 192,
                      "patch": 768 * 192, "head": 192 * 1000}
# Algorithmic HBM bytes per row for the row-wise kernels (int8 in + int8 out).
STAGE_BYTES_PER_ROW = {"ln1": 384, "ln2": 384}
# DRAM bytes (read + write) per row of one launch, from the committed ncu captures of a
# full-size launch (block 1, 201,728 rows): profiles/tcp_gemm_qkv_proj_fc1_block1_b1024.md,
# profiles/tcp_gemm_fc2_block1_b1024.md, profiles/ln_kernel_ln1_block1_b1024.md.
# Traffic grows with the rows of a launch.
STAGE_TRAFFIC_PER_ROW = {"fc1": (38_966_016 + 100_830_720) / 201_728,
                         "fc2": (193_862_912 + 24_387_584) / 201_728,
                         "ln1": (38_799_616 + 1_387_776) / 201_728}


def algorithmic_macs(counts):
    """Reference MAC convention (tools/p8/_perf_common.py:88-123): patch +
    per block 442368*N + 384*N^2 + selectors 13938*C + head, per image."""
    counts = np.asarray(counts, np.int64)
    macs = np.full(counts.shape[0], 28_901_376 + 192_000, np.int64)
    ns = counts.shape[1] - 1
    sel_before = {4: 1, 7: 2, 10: 3} if ns == 3 else {}
    col = 0
    for b in range(1, 13):
        if b in sel_before:
            c = counts[:, col] - 1
            macs += 13_938 * c
            col = sel_before[b]
        n = counts[:, col]
        macs += 442_368 * n + 384 * n * n
    return macs


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


def cpu_oracle_rate(params, images, target_s=15.0, max_images=4096):
    """Images/s of the oracle (C restatement of the golden model) on all host
    threads over a bounded sample sized for about ``target_s`` seconds.  The
    sample is the step's own images, cycled when it needs more than one batch."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import hv_oracle
    hv_oracle.build()
    threads = hv_oracle.num_cpus()
    probe = min(images.shape[0], max(2 * threads, 8))
    t0 = time.perf_counter()
    hv_oracle.infer_batch(params, images[:probe], threads=threads)
    dt = time.perf_counter() - t0
    rate = probe / dt
    n = int(min(max_images, max(probe, rate * target_s)))
    sample = images[np.arange(n) % images.shape[0]]
    t0 = time.perf_counter()
    hv_oracle.infer_batch(params, sample, threads=threads)
    dt = time.perf_counter() - t0
    return n / dt, threads, n, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from heatvit_b200 import synth
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import hv_oracle
    hv_oracle.build()
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
                   "per_step_sample_images": per_step},
        "impl": "reference",
        "cpu_baseline": {"value": value, "unit": "images/s", "cores": threads, "kind": "port",
                         "sample": f"{per_step} seeded images per step, {args.steps} steps, C restatement of "
                                   "verification/heatvit_ref on all host threads"},
        "e2e": {"value": value, "unit": "images/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Config 4 runs the benchmark model unpruned, or pruned with config 3's selectors.
PARAMS_FN = {"pruned": "config3_params", "unpruned": "config_params(pruned=False)"}


def bench_params(synth, variant):
    if variant == "pruned":
        return synth.config3_params(synth.SEED)
    return synth.config_params(synth.SEED, pruned=False)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1024, help="images per GPU per step")
    ap.add_argument("--variant", default="pruned", choices=["pruned", "unpruned"])
    ap.add_argument("--profile-stage", default="fc1", choices=sorted(STAGES))
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    from heatvit_b200.shard import gather_outputs, shard_range

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    params = bench_params(synth, args.variant)
    eng = Engine(params)
    b = args.batch
    first, _ = shard_range(rank, world, b)
    host_imgs = synth.baseline_images(synth.SEED, b, first=first)
    imgs = torch.from_numpy(host_imgs).cuda()
    ns = eng.num_selectors
    peaks = measured_peaks()

    def step():
        out = eng.infer(imgs)
        return gather_outputs(out["logits"], out["token_counts"], world)

    # The first launch of the profiled stage in each step (block 1's, the largest) is
    # bracketed by CUDA events inside the replayed graph; the warm-up captures that
    # graph, so the timed steps only replay it.  One bracketed launch per step keeps
    # the events from breaking more than one programmatic-launch edge.
    _lib.check(_lib.lib().hv_profile_start(eng.handle, STAGES[args.profile_stage], 1))
    for _ in range(args.warmup):
        logits, counts = step()
    torch.cuda.synchronize()
    counts_np = counts.cpu().numpy()

    stream = torch.cuda.current_stream()
    sampler = ClockSampler(physical_gpu_index(torch, local)) if rank == 0 else None
    time.sleep(0.3 if sampler else 0)
    _lib.check(_lib.lib().hv_profile_start(eng.handle, STAGES[args.profile_stage], 1))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        logits, counts = step()
    ev1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed_ms = ev0.elapsed_time(ev1)
    # the profiled launches of the last timed step (events recorded by its replay)
    launches, kms, krows = C.c_int(), C.c_double(), C.c_longlong()
    _lib.check(_lib.lib().hv_profile_stop(eng.handle, C.byref(launches), C.byref(kms), C.byref(krows)))
    graph_kernels = C.c_int()
    _lib.check(_lib.lib().hv_graph_kernels(eng.handle, C.byref(graph_kernels)))
    clocks = sampler.stop() if sampler else None
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = world * b / (ms_per_step * 1e-3)

    # End-to-end through the public host API: pinned host images in, host logits out,
    # every step's upload and download inside the timed region.  Pipelined: the
    # serving loop keeps two calls in flight (hv_infer_host_submit / _wait), so a
    # step's upload runs during the previous step's compute.  Blocking: one
    # hv_infer_host call per step.
    pinned = torch.empty((b, 150528), dtype=torch.int8, pin_memory=True)
    pinned.numpy()[:] = host_imgs
    host_logits = [torch.empty((b, 1000), dtype=torch.int32, pin_memory=True).numpy() for _ in range(2)]

    def e2e_pipelined(steps):
        for i in range(steps):
            eng.infer_host_submit(pinned.numpy(), host_logits[i % 2])
            if i:
                eng.infer_host_wait()
        eng.infer_host_wait()

    def e2e_blocking(steps):
        for _ in range(steps):
            eng.infer_host(pinned.numpy(), logits=host_logits[0])

    e2e_rates = {}
    for name, fn in (("pipelined", e2e_pipelined), ("blocking", e2e_blocking)):
        # warm-up: enough calls that every (image buffer, workspace, chunk size)
        # combination has its CUDA graph captured before the timed calls
        fn(6)
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        fn(args.e2e_steps)
        e2e_s = (time.perf_counter() - t0) / args.e2e_steps
        if world > 1:
            t = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        e2e_rates[name] = world * b / e2e_s
    e2e_value = e2e_rates["pipelined"]

    if rank == 0:
        int8_tops, int8_src = measure_int8_tops(torch)
        macs = algorithmic_macs(counts_np[:b] if counts_np.shape[0] >= b else counts_np)
        macs_per_step = float(macs.mean()) * world * b
        t_compute = 2 * macs_per_step / (int8_tops * 1e12)
        bytes_step = world * b * (150528 + 4004) + WEIGHT_BYTES * world
        hbm = peaks.get("hbm_gbs", 6650.0)
        t_mem = bytes_step / (hbm * 1e9) / world
        model_frac = max(t_compute / world, t_mem) / (ms_per_step * 1e-3)
        st = args.profile_stage
        kavg = kms.value / max(1, launches.value)
        rows_avg = krows.value / max(1, launches.value)
        traffic = STAGE_TRAFFIC_PER_ROW[st] * rows_avg if st in STAGE_TRAFFIC_PER_ROW else None
        if st in STAGE_MACS_PER_ROW:
            work = 2.0 * STAGE_MACS_PER_ROW[st] * krows.value / max(1, launches.value)
            achieved = work / (kavg * 1e-3) / 1e12
            roof = {"bound": "tensor", "achieved": achieved, "peak": int8_tops, "unit": "TOPS",
                    "frac": achieved / int8_tops, "traffic": traffic, "traffic_unit": "bytes per launch",
                    "kernel": f"{st} (int8 GEMM; block 1's launch in the last timed step: {kavg:.4f} ms, {rows_avg:.0f} rows)",
                    "peak_source": int8_src, "work": "2*rows*K*N int8 ops per launch"}
        else:
            work = STAGE_BYTES_PER_ROW.get(st, 384) * krows.value / max(1, launches.value)
            achieved = work / (kavg * 1e-3) / 1e9
            roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "traffic": traffic, "traffic_unit": "bytes per launch", "kernel": f"{st} (block 1's launch in the last timed step: {kavg:.4f} ms, {rows_avg:.0f} rows)",
                    "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"}
        line = {
            "metric": METRIC, "value": value, "unit": "images/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8/int32", "data": "synthetic",
            "config": {"workload": f"config4-{args.variant}: batch {b}/GPU of seeded 224x224x3 int8 images, "
                                   "benchmark DeiT-T (synth." + PARAMS_FN[args.variant] + "), selectors before blocks 4/7/10",
                       "images_per_gpu": b, "parallelism": f"image-sharded x{world}",
                       "l2": "inputs larger than L2 (images 154 MB/GPU per step)",
                       "mean_token_counts": [float(v) for v in counts_np.mean(0)]},
            "roofline": roof,
            "model_roofline": {"frac": model_frac, "algorithmic_gmac_per_image": float(macs.mean()) / 1e9,
                               "int8_peak_tops": int8_tops, "int8_spec_tops": INT8_SPEC_TOPS,
                               "frac_of_spec": (2 * macs_per_step / (INT8_SPEC_TOPS * 1e12) / world)
                               / (ms_per_step * 1e-3)},
            "e2e": {"value": e2e_value, "unit": "images/s", "h2d_bytes_per_step": b * 150528,
                    "d2h_bytes_per_step": b * 4000, "steps": args.e2e_steps,
                    "mode": "pipelined host calls (hv_infer_host_submit/_wait, two in flight)",
                    "blocking_value": e2e_rates["blocking"]},
            # init + patch + 12 x 7 block kernels + 2 per selector + CLS LN + head, plus one
            # row-count copy per profiled launch
            "gpu_launches": graph_kernels.value * args.steps,
            "clocks": clocks,
        }
        if world == 1 and not args.no_cpu_baseline:
            rate, threads, n, dt = cpu_oracle_rate(params, host_imgs)
            line["cpu_baseline"] = {"value": rate, "unit": "images/s", "cores": threads, "kind": "port",
                                    "sample": f"{n} images (the step's batch, cycled) in {dt:.1f}s on "
                                              f"{threads} threads; C restatement of verification/heatvit_ref"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
