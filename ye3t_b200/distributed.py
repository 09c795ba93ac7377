"""Atom-block partition across ranks (one process per GPU).

Each atom's A- and B-basis depend only on its own neighbour row, so rank r of
P evaluates the centres ``[r N / P, (r + 1) N / P)`` from the replicated
positions; the collectives are sums of the per-rank energies and, with forces,
a reduce-scatter of the per-rank partial force arrays (each rank scatters its
rows' edge gradients into a full ``[N, 3]`` array and keeps the summed forces
of its own block).  With atoms stored in cell order a block is a slab of the
box, and each rank bins only its slab and a one-cell halo for its neighbour
lists.  The reference has no distributed code; this is new.
"""

from __future__ import annotations

import datetime
import os
from typing import Tuple

import torch
import torch.distributed as dist

__all__ = ["atom_block", "init_from_env", "sum_over_ranks", "max_over_ranks", "block_forces"]


def atom_block(rank: int, world: int, atom_count: int) -> Tuple[int, int]:
    """Contiguous centre range of ``rank``; blocks differ in size by at most one."""
    if not 0 <= rank < world:
        raise ValueError("rank out of range")
    return (atom_count * rank) // world, (atom_count * (rank + 1)) // world


def init_from_env(backend: str = "nccl", timeout_s: float = 300.0, device=None):
    """Initialise the default group from torchrun's environment; returns (rank, world)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and not dist.is_initialized():
        kwargs = {"timeout": datetime.timedelta(seconds=timeout_s)}
        if backend == "nccl" and device is not None:
            kwargs["device_id"] = device
        dist.init_process_group(backend, **kwargs)
    return rank, world


def sum_over_ranks(value: torch.Tensor) -> torch.Tensor:
    """In-place sum across ranks (no-op on one rank)."""
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(value, op=dist.ReduceOp.SUM)
    return value


def max_over_ranks(x: float, device) -> float:
    t = torch.tensor([x], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def block_forces(partial: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Sum the ranks' partial force arrays ``partial [P * chunk, 3]`` and keep this rank's
    ``chunk`` rows in ``out [chunk, 3]`` (a reduce-scatter; on a backend without one,
    such as gloo on CPU, an all-reduce and a slice give the same rows)."""
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        out.copy_(partial[:out.shape[0]])
        return out
    world, rank = dist.get_world_size(), dist.get_rank()
    if partial.shape[0] != world * out.shape[0]:
        raise ValueError("partial forces must hold world_size * chunk rows")
    if dist.get_backend() == "nccl":
        dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM)
    else:
        full = partial.clone()
        dist.all_reduce(full, op=dist.ReduceOp.SUM)
        out.copy_(full[rank * out.shape[0]:(rank + 1) * out.shape[0]])
    return out

