"""Activation feed: a layer's activation pool held in HBM.

The reference streams pool shards from disk with reader threads into pinned
host memory and copies each batch to the GPU on a side stream
(``RollingActivationProvider`` and ``_ActivationDoubleBuffer``,
sae_trainer_rolling.py:2104-2249). At the fused step's rate (≈3.7 M tokens/s at
d = 1536, ≈11 GB/s of bf16) a layer's whole pool fits comfortably in a B200's
180 GB -- the atlas configuration gives each layer 16 shards × 32768 tokens,
1.6 GB at d = 1536 -- so ``DeviceActivationPool`` loads the shards once and
hands out batches that already live in device memory: no per-step host work,
no PCIe traffic in the training loop.

It reads the reference's shard format (``shard_{i:05d}.pt``: a bf16 tensor
``[n_seqs, seq_len, d]`` written by ``torch.save``, 1606-1614) and mirrors the
provider's interface (``next_batch``, ``next_batch_to_device``, ``get_state``,
``restore_state``, ``close``), so the trainer can take it in place of the
provider + double buffer. Like the reference, each shard is one batch and the
shard order is reshuffled every epoch (seeded).
"""
from __future__ import annotations

import random
from pathlib import Path
from typing import List, Optional, Sequence

import torch


def shard_paths(pool_dir) -> List[Path]:
    """The pool's shard files in index order (the reference's naming)."""
    return sorted(Path(pool_dir).glob("shard_*.pt"))


class DeviceActivationPool:
    """All shards of one layer's pool resident on ``device``; each
    ``next_batch()`` returns the next shard ([tokens, d] bf16, a view, no copy)
    in a seeded per-epoch shuffled order."""

    def __init__(self, shards: Sequence[torch.Tensor], device, seed: int = 0):
        if not shards:
            raise ValueError("empty activation pool")
        dev = torch.device(device)
        d = shards[0].shape[-1]
        self.shards = []
        for t in shards:
            if t.shape[-1] != d:
                raise ValueError("pool shards disagree on d_in")
            t = t.reshape(-1, d)
            if t.dtype not in (torch.bfloat16, torch.float32):
                t = t.to(torch.bfloat16)
            self.shards.append(t.to(dev, non_blocking=True).contiguous())
        self.device = dev
        self.seed = int(seed)
        self.d_in = d
        self._epoch = 0
        self._pos = 0
        self._order = self._shuffled(0)

    @classmethod
    def from_dir(cls, pool_dir, device, seed: int = 0, limit: Optional[int] = None):
        paths = shard_paths(pool_dir)[:limit]
        if not paths:
            raise RuntimeError(f"No pool shards in {pool_dir}")
        shards = [torch.load(p, map_location="cpu", weights_only=True) for p in paths]
        return cls(shards, device, seed)

    def _shuffled(self, epoch: int) -> List[int]:
        order = list(range(len(self.shards)))
        random.Random(self.seed * 7919 + epoch).shuffle(order)
        return order

    def next_batch(self) -> torch.Tensor:
        if self._pos == len(self._order):
            self._epoch += 1
            self._pos = 0
            self._order = self._shuffled(self._epoch)
        t = self.shards[self._order[self._pos]]
        self._pos += 1
        return t

    def next_batch_to_device(self, non_blocking: bool = True) -> torch.Tensor:
        return self.next_batch()

    @property
    def tokens(self) -> int:
        return sum(t.shape[0] for t in self.shards)

    def get_state(self):
        return {"epoch": self._epoch, "pos": self._pos, "seed": self.seed}

    def restore_state(self, state) -> None:
        if not state:
            return
        self.seed = int(state.get("seed", self.seed))
        self._epoch = int(state["epoch"])
        self._pos = int(state["pos"])
        self._order = self._shuffled(self._epoch)

    def close(self) -> None:
        self.shards = []
