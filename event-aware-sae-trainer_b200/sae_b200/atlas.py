"""Layer atlas across GPUs: independent per-layer SAEs, one process per GPU.

The reference trains one SAE per transformer layer, layer after layer on one
device (``run_atlas_rolling``, sae_trainer_rolling.py:4040-4180). The layers
are independent units, so the B200 layout places them round-robin on the GPUs
of a node -- layer l on rank l mod world -- and runs them with no data-path
collective. The only cross-rank communication is bookkeeping (a barrier and
a max / sum of a timing or a count), done with ``torch.distributed``.
"""
from __future__ import annotations

from typing import List

import torch
import torch.distributed as dist


def layers_for_rank(n_layers: int, world: int, rank: int) -> List[int]:
    """Round-robin placement: rank r trains layers r, r + world, r + 2 world, ..."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    return list(range(rank, n_layers, world))


def ideal_speedup(n_layers: int, world: int) -> float:
    """Makespan bound of the round-robin atlas: n_layers / ceil(n_layers / world)."""
    per = -(-n_layers // world)
    return n_layers / per


def _reduce(value: float, op, device) -> float:
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=op)
    return float(t.item())


def max_over_ranks(value: float, device=None) -> float:
    """The slowest rank's time (every multi-GPU duration is reported this way)."""
    return _reduce(value, dist.ReduceOp.MAX, device)


def sum_over_ranks(value: float, device=None) -> float:
    return _reduce(value, dist.ReduceOp.SUM, device)
