"""Image sharding over the GPUs of one node (weak scaling).

Images are independent in the golden model (model.py:73-123 keeps no state
across images), so rank r of a W-rank job owns the contiguous image range
[r * per_rank, (r + 1) * per_rank), runs the whole model on it, and the only
inter-GPU traffic is the gather of the per-image outputs to rank 0.
"""


def shard_range(rank, world, per_rank):
    """(first image, image count) owned by ``rank``."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if per_rank <= 0:
        raise ValueError("per_rank must be positive")
    return rank * per_rank, per_rank


def gather_rows(t, world, group=None):
    """Concatenate every rank's ``t`` along dim 0 in rank order (one all-gather)."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return t
    out = torch.empty((world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    return out


def gather_outputs(logits, token_counts, world, group=None):
    """Logits [B, 1000] and token counts [B, S+1] of every rank, in image order."""
    return gather_rows(logits, world, group), gather_rows(token_counts, world, group)


class RootGather:
    """Gather of one flat per-rank buffer to rank 0, overlapped with later work.

    ``submit(buf)`` enqueues ``dist.gather`` of ``buf`` on a side stream that
    first waits for the work already queued on the caller's stream (the kernels
    that wrote ``buf``); the caller's stream continues at once, so the gather of
    step i runs under the compute of step i + 1.  ``fence(buf)`` makes the
    caller's stream wait until the gather that reads ``buf`` has finished (call
    it before ``buf`` is written again); ``flush()`` does so for every gather in
    flight.  Rank 0 receives into ``world`` slots of its result buffers, one per
    rank in rank order; the other ranks receive nothing.  With one rank the
    buffer itself is the result and nothing is queued.
    """

    def __init__(self, world, rank, numel, dtype, device, slots=2, group=None):
        import torch
        self.world, self.rank, self.group = world, rank, group
        device = torch.device(device)
        # CPU tensors (gloo) gather synchronously; CUDA tensors on a side stream
        self.side = torch.cuda.Stream(device=device) if world > 1 and device.type == "cuda" else None
        self.recv = []
        if world > 1 and rank == 0:
            self.recv = [torch.empty((world, numel), dtype=dtype, device=device) for _ in range(slots)]
        self.pending = {}
        self.n = 0

    def submit(self, buf):
        """Gather ``buf``; returns rank 0's [world, numel] result (or ``buf``)."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return buf
        slot = self.n % max(1, len(self.recv) or 2)
        self.n += 1
        out = self.recv[slot] if self.rank == 0 else None
        lst = list(out.unbind(0)) if out is not None else None
        if self.side is None:
            dist.gather(buf, lst, dst=0, group=self.group)
            return out
        cur = torch.cuda.current_stream(buf.device)
        self.side.wait_stream(cur)
        with torch.cuda.stream(self.side):
            work = dist.gather(buf, lst, dst=0, group=self.group, async_op=True)
        buf.record_stream(self.side)
        self.pending[buf.data_ptr()] = work
        return out

    def fence(self, buf):
        work = self.pending.pop(buf.data_ptr(), None)
        if work is not None:
            work.wait()  # the caller's current stream waits for the gather

    def flush(self):
        for key in list(self.pending):
            self.pending.pop(key).wait()
