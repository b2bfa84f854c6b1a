"""Revival writes on a dictionary split over ranks.

The reference revives dead features with masked in-place writes on the whole
dictionary (sae_trainer_rolling.py): the threshold reset gives the
chronically dead features the median log-threshold of the living ones and
zeroes their Adam moments (3107-3118, helper _revive_log_threshold 209-225);
the resample (resample_dead_neurons, 2784-2810) draws one high-error input
per dead feature (torch.randint over the error buffer), writes it -- unit
norm times RESAMPLE_SCALE times the mean norm of the living W_enc rows -- as
the feature's encoder row, zeroes its encoder bias, draws a fresh unit
Gaussian decoder column (torch.randn(d, n_dead)), zeroes the Adam moments of
those rows and columns, and then revives the thresholds as above (3151-3158).

On a shard (rank r of N holds features [r F/N, (r+1) F/N)) every quantity
that spans the dictionary is formed over all ranks, in global feature order,
so that the shards together hold exactly what the unsharded writes produce:
  * the dead masks are gathered (each rank's revival controller tracks its own
    features) and the dead features are numbered in global order;
  * the random draws are made once, on rank 0, with the same calls in the same
    order as the reference (randint, then randn), and broadcast; rank r takes
    the draws of its own dead features;
  * the live median of the log-thresholds and the mean living W_enc row norm
    are computed over the gathered values.
The candidates (the error buffer) are replicated: they are rows of the
replicated input batch.

Communication goes through a small interface (``Comm``): ``DistComm`` wraps
torch.distributed (NCCL on the GPUs, gloo on CPU); tests emulate ranks with
threads. The functions take any optimizer with torch Adam's state keys
(``B200Adam`` or ``torch.optim.Adam``).
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.distributed as dist

INIT_THRESHOLD = 0.1    # sae_trainer_rolling.py:212
RESAMPLE_SCALE = 1.0    # sae_trainer_rolling.py:236


class Comm:
    """What the revival writes need from the ranks sharing a dictionary."""

    rank: int = 0
    world: int = 1

    def all_gather(self, t: torch.Tensor) -> List[torch.Tensor]:
        """Every rank's tensor (equal shapes), in rank order."""
        return [t]

    def broadcast(self, t: torch.Tensor, src: int = 0) -> None:
        """In place: every rank receives rank src's values."""

    def all_reduce_sum(self, t: torch.Tensor) -> None:
        """In place sum over the ranks."""


class DistComm(Comm):
    """torch.distributed over ``group`` (default: the whole world)."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def all_gather(self, t):
        out = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(out, t.contiguous(), group=self.group)
        return out

    def broadcast(self, t, src=0):
        dist.broadcast(t, src=dist.get_global_rank(self.group, src) if self.group else src,
                       group=self.group)

    def all_reduce_sum(self, t):
        dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)


def _zero_adam_rows(optimizer, params_and_masks) -> None:
    """exp_avg[mask] = exp_avg_sq[mask] = 0 for each (param, mask, column)
    pair: rows of the tensor, or columns of the [d, F] decoder view."""
    for p, mask, columns in params_and_masks:
        state = optimizer.state.get(p, {})
        if "exp_avg" not in state:
            continue
        for k in ("exp_avg", "exp_avg_sq"):
            if columns:
                state[k][:, mask] = 0.0
            else:
                state[k][mask] = 0.0


def revive_log_threshold_value(log_threshold: torch.Tensor, mask: torch.Tensor,
                               comm: Optional[Comm] = None) -> torch.Tensor:
    """_revive_log_threshold (209-225) over the whole dictionary: the median
    of the living features' log-thresholds, log(INIT_THRESHOLD) when none is
    alive. A 0-d tensor on log_threshold's device, the same on every rank."""
    comm = comm or Comm()
    lt = torch.cat(comm.all_gather(log_threshold.detach()))
    alive = ~torch.cat(comm.all_gather(mask.to(torch.uint8))).bool()
    if bool(alive.any()):
        return lt[alive].median()
    return torch.tensor(math.log(INIT_THRESHOLD), device=log_threshold.device,
                        dtype=log_threshold.dtype)


@torch.no_grad()
def threshold_reset(sae, optimizer, dead_mask: torch.Tensor, comm: Optional[Comm] = None) -> int:
    """The RESET write (3107-3118) on this rank's features: log_threshold of
    the dead features <- the live median, their Adam moments zeroed. Returns
    the dead count over the whole dictionary."""
    comm = comm or Comm()
    n = torch.tensor([int(dead_mask.sum())], dtype=torch.int64, device=dead_mask.device)
    comm.all_reduce_sum(n)
    if int(n) == 0:
        return 0
    rev = revive_log_threshold_value(sae.log_threshold.data, dead_mask, comm)
    sae.log_threshold.data[dead_mask] = rev
    _zero_adam_rows(optimizer, [(sae.log_threshold, dead_mask, False)])
    return int(n)


@torch.no_grad()
def resample(sae, optimizer, dead_mask: torch.Tensor, candidates: Optional[torch.Tensor],
             comm: Optional[Comm] = None, scale: float = RESAMPLE_SCALE) -> int:
    """resample_dead_neurons (2784-2810) followed by the threshold revival of
    the resampled features (3151-3158), on this rank's features. ``candidates``
    [n, d]: the error buffer (replicated over the ranks). Returns the dead
    count over the whole dictionary (0: nothing written)."""
    comm = comm or Comm()
    dev = dead_mask.device
    counts = torch.cat(comm.all_gather(
        torch.tensor([int(dead_mask.sum())], dtype=torch.int64, device=dev)))
    n_dead = int(counts.sum())
    if n_dead == 0 or candidates is None or candidates.shape[0] == 0:
        return 0
    first = int(counts[:comm.rank].sum())
    mine = int(counts[comm.rank])
    W_enc = sae.W_enc.weight
    # the draws, once, in the reference's order (randint, then randn)
    idx = torch.empty(n_dead, dtype=torch.int64, device=dev)
    rand_dec = torch.empty(sae.d_in, n_dead, dtype=sae.W_dec.weight.dtype, device=dev)
    if comm.rank == 0:
        idx.copy_(torch.randint(0, candidates.shape[0], (n_dead,), device=dev))
        rand_dec.copy_(torch.randn(sae.d_in, n_dead, device=dev, dtype=rand_dec.dtype))
    comm.broadcast(idx, 0)
    comm.broadcast(rand_dec, 0)
    # mean norm of the living encoder rows over the whole dictionary: the
    # per-row norms gathered in feature order and averaged as one tensor, as
    # the unsharded .mean() does
    row_norms = torch.cat(comm.all_gather(W_enc.data.norm(dim=1)))
    alive = ~torch.cat(comm.all_gather(dead_mask.to(torch.uint8))).bool()
    alive_norm = row_norms[alive].mean() if bool(alive.any()) else \
        torch.tensor(1.0, device=dev)
    if mine > 0:
        sl = slice(first, first + mine)
        samples = candidates[idx[sl]]
        norms = samples.norm(dim=-1, keepdim=True).clamp(min=1e-8)
        W_enc.data[dead_mask] = ((samples / norms) * scale * alive_norm).to(W_enc.dtype)
        sae.W_enc.bias.data[dead_mask] = 0.0
        cols = rand_dec[:, sl]
        sae.W_dec.weight.data[:, dead_mask] = cols / cols.norm(dim=0, keepdim=True).clamp(min=1e-8)
        _zero_adam_rows(optimizer, [(W_enc, dead_mask, False), (sae.W_enc.bias, dead_mask, False),
                                    (sae.W_dec.weight, dead_mask, True)])
    rev = revive_log_threshold_value(sae.log_threshold.data, dead_mask, comm)
    if mine > 0:
        sae.log_threshold.data[dead_mask] = rev
        _zero_adam_rows(optimizer, [(sae.log_threshold, dead_mask, False)])
    if hasattr(sae, "mark_weights_dirty"):
        sae.mark_weights_dirty()
    return n_dead
