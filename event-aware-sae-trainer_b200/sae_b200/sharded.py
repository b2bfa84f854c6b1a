"""One wide JumpReLU SAE with its dictionary split over the GPUs of a node.

The reference trains a dictionary on one device (``train_sae_on_activations``,
sae_trainer_rolling.py:2382-3672). For dictionaries too large or too slow for
one GPU, rank r of N holds features [r F/N, (r+1) F/N): those rows of W_enc and
b_enc, those columns of W_dec (rows of the feature-major storage), those
entries of log_threshold, with their gradients and Adam state. The input batch
and b_dec are replicated. Every per-feature computation is then local and the
step needs exactly three sums over the ranks, all on the caller's stream
through ``torch.distributed`` (NCCL over NVLink on a B200 node):

1. forward: the shards' fp32 decoder outputs and per-token active counts,
   one buffer of ``n_tokens * (d + 1)`` floats (the partial x_hat and the L0
   counts); after it every rank forms the same residual, loss and go;
2. backward: the b_dec gradient, whose encoder term -(Σ_b dpre) W_enc (601)
   is a sum over features; rank 0 adds the go sum and the accumulated value;
3. the global gradient-norm sum of squares of ``clip_grad_norm_`` (3049),
   with the replicated b_dec gradient counted once.

Adam, both renormalisations (each W_dec column / W_enc row lives on one rank)
and the fired-feature mask are local; b_dec's Adam update sees identical
gradients and state on every rank and so stays replicated.
"""
from __future__ import annotations

import ctypes
import math
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib as L
from .sae import INIT_THRESHOLD, B200JumpReLUSAE, _stream, sae_from_tensors
from .step import B200Adam, FusedStep


def shard_range(n_features: int, rank: int, world: int) -> slice:
    """Features held by ``rank``: an even, contiguous split of the dictionary."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("need 0 <= rank < world")
    if n_features % world:
        raise ValueError(f"n_features={n_features} does not split evenly over {world} ranks")
    per = n_features // world
    return slice(rank * per, (rank + 1) * per)


@torch.no_grad()
def shard_sae(full: B200JumpReLUSAE, rank: int, world: int,
              device: Optional[torch.device] = None) -> B200JumpReLUSAE:
    """Rank ``rank``'s slice of a whole SAE (same values, b_dec replicated)."""
    s = shard_range(full.n_features, rank, world)
    fm = full._dec_fm()
    out = sae_from_tensors(full.W_enc.weight[s], full.W_enc.bias[s], fm[s], full.b_dec,
                           full.log_threshold[s])
    out.ste_bandwidth = full.ste_bandwidth
    return out.to(device) if device is not None else out


@torch.no_grad()
def make_shard_sae(d_in: int, n_features: int, rank: int, world: int, seed: int = 0, *,
                   device="cuda") -> B200JumpReLUSAE:
    """A shard initialised on the device without building the whole dictionary:
    unit-norm Gaussian decoder columns (the reference's orthogonal init is
    impossible once F > d anyway; its columns are unit-norm), W_enc = W_dec^T,
    b_enc = 0, threshold 0.1 -- the reference's init values apart from the
    orthogonalisation. Features are drawn in blocks of 4096 from a generator
    seeded by (seed, block), so the whole dictionary is the same for every
    world size whose shards are whole blocks."""
    s = shard_range(n_features, rank, world)
    per = s.stop - s.start
    dev = torch.device(device)
    fm = torch.empty(per, d_in, device=dev)
    g = torch.Generator(device=dev)
    blk = 4096
    for f0 in range(s.start, s.stop, blk):
        b = f0 // blk
        lo = f0 - b * blk                       # offset inside the block (0 when aligned)
        n = min(blk - lo, s.stop - f0)
        g.manual_seed(int(seed) * 1_000_003 + b)
        rows = torch.randn(blk, d_in, generator=g, device=dev)[lo:lo + n]
        fm[f0 - s.start:f0 - s.start + n] = rows
    fm /= fm.norm(dim=1, keepdim=True).clamp(min=1e-8)
    return sae_from_tensors(fm, torch.zeros(per, device=dev), fm, torch.zeros(d_in, device=dev),
                            torch.full((per,), math.log(INIT_THRESHOLD), device=dev))


class _DeviceBytes:
    """A raw device allocation seen as a torch uint8 tensor (no ownership)."""

    def __init__(self, ptr: int, nbytes: int, device: torch.device):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3, "strides": None}
        self.device = device


class PeerExchange:
    """The ranks' peer buffers (workspace + exchange + flags), mapped into every
    rank by CUDA IPC for sae_b200_shard_forward_p2p. Collective: every rank of
    ``group`` constructs it with the same sizes."""

    def __init__(self, max_tokens: int, d_in: int, n_features: int, csr_capacity: int, *,
                 group=None, device: torch.device):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > L.MAX_PEERS:
            raise ValueError(f"peer exchange supports at most {L.MAX_PEERS} ranks")
        nbytes = ctypes.c_size_t(0)
        ex = ctypes.c_uint64(0)
        fl = ctypes.c_uint64(0)
        L.call("sae_b200_peer_buffer_bytes", max_tokens, d_in, n_features, csr_capacity,
               ctypes.byref(nbytes), ctypes.byref(ex), ctypes.byref(fl))
        self.nbytes, self.exchange_offset, self.flags_offset = nbytes.value, ex.value, fl.value
        own = ctypes.c_void_p(0)
        handle = (ctypes.c_uint8 * L.PEER_HANDLE_BYTES)()
        with torch.cuda.device(device):
            L.call("sae_b200_peer_alloc", self.nbytes, ctypes.byref(own), handle)
        self.own = own.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases = [0] * self.world
        self._opened = []
        with torch.cuda.device(device):
            for p in range(self.world):
                if p == self.rank:
                    self.bases[p] = self.own
                    continue
                h = (ctypes.c_uint8 * L.PEER_HANDLE_BYTES).from_buffer_copy(handles[p])
                ptr = ctypes.c_void_p(0)
                L.call("sae_b200_peer_open", h, ctypes.byref(ptr))
                self.bases[p] = ptr.value
                self._opened.append(ptr.value)
        self.epoch = 0
        self.workspace = torch.as_tensor(_DeviceBytes(self.own, self.exchange_offset, device),
                                         device=device)

    def next_peers(self) -> L.Peers:
        self.epoch += 1
        p = L.Peers()
        p.rank, p.world, p.epoch = self.rank, self.world, self.epoch
        p.exchange_offset, p.flags_offset = self.exchange_offset, self.flags_offset
        for i, b in enumerate(self.bases):
            p.base[i] = b
        return p

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""
        if self.own is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)   # no rank touches another's buffer any more
        for ptr in self._opened:
            L.call("sae_b200_peer_close", ptr)
        dist.barrier(group=self.group)
        L.call("sae_b200_peer_free", self.own)
        self.own = None
        self.workspace = None


class ShardedFusedStep(FusedStep):
    """FusedStep over one dictionary shard, with the three cross-rank sums.

    ``group`` is the process group of the ranks sharing the dictionary
    (default: the whole world). With one rank (or no process group) the
    sequence reduces to the unsharded step. ``exchange``: "p2p" (default) sums
    the partial x_hat over NVLink peer memory fused with the residual
    (``PeerExchange``, one GPU per rank on one node); "nccl" all-reduces it
    with torch.distributed. ``allreduce`` (with ``rank`` and
    ``world``) replaces both by the caller's own in-place sum over the ranks,
    called with each of the three buffers in order. ``pre_store`` as in
    FusedStep: a shard whose CSR overflows after an entries-only forward
    stores the rest of its pre locally before the dense backward (the
    exchange is not repeated, so the ranks stay in step).
    ``step()``, ``microbatch()``, ``grad_norm()`` and the returned statistics
    have FusedStep's meaning; ``nnz`` and ``csr_overflow`` are this shard's."""

    def __init__(self, sae: B200JumpReLUSAE, optimizer: B200Adam, max_tokens: int, *,
                 group=None, csr_capacity: Optional[int] = None, force_simt: bool = False,
                 grad_feat: str = "sampled", exchange: str = "p2p", pre_store: str = "entries",
                 allreduce: Optional[Callable[[torch.Tensor], None]] = None,
                 rank: Optional[int] = None, world: Optional[int] = None):
        super().__init__(sae, optimizer, max_tokens, csr_capacity=csr_capacity,
                         force_simt=force_simt, grad_feat=grad_feat, pre_store=pre_store)
        if exchange not in ("nccl", "p2p"):
            raise ValueError("exchange must be 'nccl' or 'p2p'")
        self.group = group
        if allreduce is not None:
            if rank is None or world is None or not 0 <= rank < world:
                raise ValueError("a custom allreduce needs rank and world (0 <= rank < world)")
            self.rank, self.world = int(rank), int(world)
        elif dist.is_available() and dist.is_initialized():
            self.rank = dist.get_rank(group)
            self.world = dist.get_world_size(group)
        else:
            self.rank, self.world = 0, 1
        self._custom_allreduce = allreduce
        # per-phase timing: None (off) or a dict phase -> [(start, stop) events]
        self.timing = None
        self.sumsq = torch.zeros(1, device=self.device, dtype=torch.float32)
        self.peers = None
        if exchange == "p2p" and self.world > 1 and allreduce is None:
            # the step workspace lives in the IPC-mapped peer buffer
            self.peers = PeerExchange(self.max_tokens, sae.d_in, sae.n_features,
                                      self.csr_capacity, group=group, device=self.device)
            self.ws = self.peers.workspace
            self.ws_bytes = self.peers.exchange_offset
            self.exchange = None
        else:
            n_ex = int(L.load().sae_b200_shard_exchange_floats(self.max_tokens, sae.d_in))
            self.exchange = torch.empty(n_ex, device=self.device, dtype=torch.float32)

    def close(self) -> None:
        """Collective with the peer exchange: release the peer buffers."""
        if self.peers is not None:
            self.peers.close()
            self.peers = None

    def _allreduce(self, t: torch.Tensor) -> None:
        if self._custom_allreduce is not None:
            self._custom_allreduce(t)
        elif self.world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _mark(self) -> Optional[torch.cuda.Event]:
        """A timing event on the current stream when per-phase timing is on."""
        if self.timing is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    def _phase(self, name: str, start, stop) -> None:
        if self.timing is not None and start is not None:
            self.timing.setdefault(name, []).append((start, stop))

    def microbatch(self, x: torch.Tensor, *, accum_steps: int = 1, first: bool = True,
                   lambda_l0: float = 0.0, al_mu: float = 0.0, target_l0: float = 0.0,
                   x_hat_out: Optional[torch.Tensor] = None,
                   after_backward: Optional[Callable[[], None]] = None) -> dict:
        """FusedStep.microbatch on this shard. Every rank takes the same
        collective steps whatever its own CSR does: the sampled backward is
        queued before the host reads the forward's statistics (it leaves the
        gradients untouched if this shard's entries overflowed the CSR), the
        overflowed shard then redoes its backward on the dense path, and only
        after that do the ranks all-reduce the b_dec gradient."""
        sae = self.sae
        if self._aux is not None:
            raise NotImplementedError("the dead-feature aux loss needs a top-k over the whole "
                                      "dictionary; it is not available on a dictionary shard")
        x = self._check_input(x)
        n = x.shape[0]
        if first:
            self.fired.zero_()
        cfg = self._cfg(n, accum_steps, first, lambda_l0, al_mu, target_l0)
        model = sae._model_struct(need_shadows=True)
        stream = _stream()
        dt = L.DTYPE_BF16 if x.dtype == torch.bfloat16 else L.DTYPE_F32
        t0 = self._mark()
        if self.peers is not None:
            if x_hat_out is not None:
                raise ValueError("x_hat_out is not available with the peer exchange")
            peers = self.peers.next_peers()
            # encoder, decode partial, NVLink sum + residual, loss terms: one call
            L.call("sae_b200_shard_forward_p2p", ctypes.byref(model), L.ptr(x), dt,
                   ctypes.byref(cfg), ctypes.byref(peers), L.ptr(self.stats), L.ptr(self.fired),
                   stream)
        else:
            ex = self.exchange[:n * (sae.d_in + 1)]
            L.call("sae_b200_shard_forward", ctypes.byref(model), L.ptr(x), dt,
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                   L.ptr(self.fired), L.ptr(ex), stream)
            self._allreduce(ex)                                # partial x_hat + L0 counts
            L.call("sae_b200_shard_finish_forward", ctypes.byref(model), L.ptr(x), dt,
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                   L.ptr(ex), L.ptr(x_hat_out), stream)
        t1 = self._mark()
        pending = self._copy_stats(0)
        grads = self._grads_struct()
        sampled = self.grad_feat == "sampled"
        if sampled:
            # ahead of the read; a no-op if this shard's CSR overflowed
            L.call("sae_b200_shard_backward", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                   self.rank, None, 0, stream)
        t2 = self._mark()
        st = self._wait_stats(pending)
        if self.peers is not None and L.device_status() != 0:
            raise L.SaeB200Error(L.SAE_ERR_DEVICE_TIMEOUT,
                                 "a peer exchange barrier timed out (a rank stopped)")
        self.nnz_last = st["nnz"]
        rows_valid = sampled and not st["csr_overflow"]
        if st["csr_overflow"]:
            self.dense_fallbacks += 1
            scratch = self._dense_scratch_for(n)
            if cfg.pre_entries_only:
                # the dense path reads all of pre: this shard's encoder again,
                # locally (the exchange is not repeated)
                L.call("sae_b200_store_full_pre", ctypes.byref(model), ctypes.byref(cfg),
                       L.ptr(self.ws), self.ws_bytes, stream)
                cfg.pre_entries_only = 0
            L.call("sae_b200_shard_backward", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                   self.rank, L.ptr(scratch), scratch.numel(), stream)
        else:
            sae._sparse_decode_calls += 1
            if not sampled:
                L.call("sae_b200_shard_backward", ctypes.byref(model), ctypes.byref(grads),
                       ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                       self.rank, None, 0, stream)
        t3 = self._mark()
        self._allreduce(self.g_b_dec)                          # b_dec gradient
        t4 = self._mark()
        self._phase("forward", t0, t1)
        self._phase("backward", t1, t2 if not st["csr_overflow"] and sampled else t3)
        self._phase("bdec_allreduce", t3, t4)
        if after_backward is not None:
            self._rows_cfg = cfg if rows_valid else None
            try:
                after_backward()
            finally:
                self._rows_cfg = None
        self._bind_grads()
        self._auto_update(st, n)
        return st

    def grad_norm(self, max_norm: float = 1.0) -> None:
        """clip_grad_norm_ over the whole dictionary: this shard's sum of
        squares (from the sampled backward's per-feature partials when that
        backward ran to completion, else a pass over the gradients; the
        replicated b_dec counted on rank 0 only), summed over the ranks."""
        t0 = self._mark()
        model = self.sae._model_struct(need_shadows=False)
        grads = self._grads_struct()
        if self.rank != 0:
            grads.b_dec = 0          # the replicated b_dec gradient counts once
        stream = _stream()
        cfg = getattr(self, "_rows_cfg", None)
        if cfg is not None:
            L.call("sae_b200_grad_sumsq_sampled", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.norm_ws),
                   self.norm_ws.numel(), L.ptr(self.sumsq), stream)
        else:
            L.call("sae_b200_grad_sumsq", ctypes.byref(model), ctypes.byref(grads),
                   L.ptr(self.norm_ws), self.norm_ws.numel(), L.ptr(self.sumsq), stream)
        self._allreduce(self.sumsq)                            # clip_grad_norm_ sum
        L.call("sae_b200_clip_from_sumsq", L.ptr(self.sumsq), float(max_norm),
               L.ptr(self.stats), stream)
        self._phase("norm", t0, self._mark())

    def optimizer_step(self, wenc_factor: float = 1.0) -> None:
        t0 = self._mark()
        super().optimizer_step(wenc_factor)
        self._phase("adam", t0, self._mark())
