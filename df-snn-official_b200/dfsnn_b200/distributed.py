"""Data parallelism for the LIF-FDE path: neuron sharding and the one gradient exchange.

Every neuron is independent (the recurrence runs along T inside a neuron), so ranks split the
neuron axis and exchange nothing in the forward.  The only shared parameters are the Softplus
masses of the glmulti schedule (and whatever the surrounding network owns); their gradients are
summed across ranks with ONE all-reduce of a flat buffer per step (NCCL over NVLink on B200,
gloo in CPU tests), as the reference's DDP does for the whole model
(examples/cnn128/train_transformer.py:853-855).
"""
import datetime

import torch
import torch.distributed as dist


def neuron_shard(n_total, rank, world):
    """Contiguous [start, stop) of the neuron axis owned by `rank` (sizes differ by <= 1)."""
    base, extra = divmod(int(n_total), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_flat(tensors, group=None, op=None):
    """Sum `tensors` across ranks with a single all-reduce of one flat buffer, in place."""
    tensors = [t for t in tensors if t is not None]
    if not tensors or not dist.is_available() or not dist.is_initialized():
        return tensors
    flat = torch.cat([t.reshape(-1) for t in tensors])
    dist.all_reduce(flat, op=op or dist.ReduceOp.SUM, group=group)
    off = 0
    for t in tensors:
        n = t.numel()
        t.copy_(flat[off:off + n].view_as(t))
        off += n
    return tensors


def init_process_group(backend, timeout_s=300, device=None):
    """init_process_group from the torchrun environment with a bounded collective timeout."""
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
