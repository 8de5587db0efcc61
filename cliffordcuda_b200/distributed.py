"""Batch data parallelism for the product layers and rotors.

The path shards by rows: every rank owns a contiguous block of the batch,
runs the kernels on it with no data-path collective, and the only exchange is
a sum all-reduce of the shared parameter's gradient (a layer's weight, 2^n
floats, or a rotor's bivector, C(n,2) floats) -- NCCL over NVLink on the GPU
box, gloo in the CPU tests. One process per GPU, launched by torchrun.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def world():
    """(world_size, rank), (1, 0) outside an initialised process group."""
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(), dist.get_rank()
    return 1, 0


def shard_rows(batch: int, world_size: int, rank: int):
    """Contiguous row range [start, stop) of `rank`; sizes differ by at most 1."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"invalid rank {rank} for world size {world_size}")
    base, extra = divmod(batch, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def allreduce_grads(module: torch.nn.Module, group=None):
    """Sum every parameter gradient of `module` over the ranks (in place).
    Parameters without a gradient contribute zeros, so all ranks issue the
    same collectives in the same order."""
    ws, _ = world()
    if ws == 1:
        return
    for p in module.parameters():
        if p.grad is None:
            p.grad = torch.zeros_like(p)
        dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, group=group)


def max_over_ranks(value: float, device=None) -> float:
    """Maximum of a host scalar over the ranks (step timings)."""
    ws, _ = world()
    if ws == 1:
        return value
    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()
