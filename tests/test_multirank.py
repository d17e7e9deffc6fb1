"""Multi-rank host logic on CPU: two gloo ranks shard a seeded batch exactly as
``bench.py --gpus 2`` does, each produces its images' logits, token counts and
warnings (the oracle stands in for the GPU here), and both the all-gather and
the gather to rank 0 of ``heatvit_b200.shard`` (the one ``bench.py`` uses) must
return every image's outputs in image order."""

import os
import socket

import numpy as np
import pytest

PER_RANK = 2
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, result_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "oracle"))
    import datetime
    import torch
    import torch.distributed as dist
    import hv_oracle
    from heatvit_b200 import synth
    from heatvit_b200.shard import gather_outputs, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=datetime.timedelta(seconds=60))
    params = synth.config_params(synth.SEED, pruned=True)
    first, count = shard_range(rank, WORLD, PER_RANK)
    imgs = synth.baseline_images(synth.SEED, count, first=first)
    ref = hv_oracle.infer_batch(params, imgs, threads=1)
    logits = torch.from_numpy(np.ascontiguousarray(ref["logits"], np.int32))
    counts = torch.from_numpy(np.ascontiguousarray(ref["counts"], np.int32))
    glog, gcnt = gather_outputs(logits, counts, WORLD)
    # the gather to rank 0 that bench.py uses: one flat int32 buffer per rank
    # (logits, token counts, warning bytes), received in rank order
    from heatvit_b200.shard import RootGather
    b, ns1 = logits.shape[0], counts.shape[1]
    warn = np.zeros(((b + 3) // 4) * 4, np.uint8)
    warn[:b] = ref["warnings"]
    flat = torch.from_numpy(np.concatenate([ref["logits"].reshape(-1), ref["counts"].reshape(-1),
                                            warn.view(np.int32)]).astype(np.int32))
    rg = RootGather(WORLD, rank, flat.numel(), torch.int32, "cpu")
    rows = rg.submit(flat)
    rg.flush()
    if rank == 0:
        np.savez(result_path, logits=glog.numpy(), counts=gcnt.numpy(), rows=rows.numpy(), b=b, ns1=ns1)
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_shard_and_gather(tmp_path, oracle):
    import torch.multiprocessing as mp
    from heatvit_b200 import synth
    out = tmp_path / "gathered.npz"
    mp.start_processes(_rank_main, args=(_free_port(), str(out)), nprocs=WORLD, start_method="spawn")
    got = np.load(out)
    params = synth.config_params(synth.SEED, pruned=True)
    whole = oracle.infer_batch(params, synth.baseline_images(synth.SEED, WORLD * PER_RANK), threads=2)
    np.testing.assert_array_equal(got["logits"], whole["logits"])
    np.testing.assert_array_equal(got["counts"], whole["counts"])
    from heatvit_b200.engine import Engine
    b, ns = int(got["b"]), int(got["ns1"]) - 1
    parts = [Engine.unpack_outputs(got["rows"][r], b, ns) for r in range(WORLD)]
    np.testing.assert_array_equal(np.concatenate([p[0] for p in parts]), whole["logits"])
    np.testing.assert_array_equal(np.concatenate([p[1] for p in parts]), whole["counts"])
    np.testing.assert_array_equal(np.concatenate([p[2] for p in parts]), whole["warnings"])


def test_shard_ranges_tile_the_batch():
    from heatvit_b200.shard import shard_range
    spans = [shard_range(r, 4, 1024) for r in range(4)]
    assert spans == [(0, 1024), (1024, 1024), (2048, 1024), (3072, 1024)]
    with pytest.raises(ValueError):
        shard_range(4, 4, 1024)
    with pytest.raises(ValueError):
        shard_range(0, 4, 0)
