"""Image sharding over the GPUs of one node (weak scaling).

Images are independent in the golden model (model.py:73-123 keeps no state
across images), so rank r of a W-rank job owns the contiguous image range
[r * per_rank, (r + 1) * per_rank), runs the whole model on it, and the only
inter-GPU traffic is one all-gather of the per-image outputs after the step.
"""


def shard_range(rank, world, per_rank):
    """(first image, image count) owned by ``rank``."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if per_rank <= 0:
        raise ValueError("per_rank must be positive")
    return rank * per_rank, per_rank


def gather_rows(t, world, group=None):
    """Concatenate every rank's ``t`` along dim 0 in rank order (one collective)."""
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
