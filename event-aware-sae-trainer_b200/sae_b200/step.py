"""The training step of the reference loop on libsae_b200.

``B200Adam`` is a ``torch.optim.Optimizer`` with torch Adam's parameter groups,
hyper-parameter keys (``lr``, ``betas``, ``eps``, ``weight_decay``) and state
keys (``step``, ``exp_avg``, ``exp_avg_sq``), so the reference scheduler's
per-step writes to ``group["lr"/"betas"/"weight_decay"]``
(sae_scheduler.py:726-731, 1601-1620) and the revival code's writes to
``optimizer.state[p]["exp_avg"][mask]`` (sae_trainer_rolling.py:2803-2810,
3116-3118) keep working. Its update is classic L2 Adam (torch.optim.Adam with
weight_decay, not AdamW), one library call for all five tensors.

``FusedStep`` is the loop body of ``train_sae_on_activations``
(sae_trainer_rolling.py:2840-3090) as a handful of library calls per
microbatch: encoder GEMM + JumpReLU epilogue, gathered decode + loss, the
sampled backward (grad_feat on the active and in-band entries only, or the
dense grad_feat GEMM) with the STE and the sparse weight gradients, the global
gradient norm (summed from the sampled backward's per-feature partials), Adam
fused with the decoder-column / encoder-row renormalisation. No [B, F] tensor
other than the bf16 pre-activations is ever written.
"""
from __future__ import annotations

import ctypes
import os
from typing import Callable, Optional

import torch

from . import _lib as L
from .sae import B200JumpReLUSAE, _require_cuda, _stream

PARAM_ORDER = ("W_enc.weight", "W_enc.bias", "W_dec.weight", "b_dec", "log_threshold")


def _sae_params(sae: B200JumpReLUSAE):
    return (sae.W_enc.weight, sae.W_enc.bias, sae.W_dec.weight, sae.b_dec, sae.log_threshold)


def reference_param_groups(sae: B200JumpReLUSAE, lr: float, decoder_wd: float = 1e-4):
    """The trainer's four groups (sae_trainer_rolling.py:2536-2540)."""
    return [{"params": list(sae.W_enc.parameters()), "weight_decay": 0},
            {"params": list(sae.W_dec.parameters()), "weight_decay": decoder_wd},
            {"params": [sae.b_dec], "weight_decay": 0},
            {"params": [sae.log_threshold], "weight_decay": 0}]


class B200Adam(torch.optim.Optimizer):
    """L2-decay Adam over the five SAE tensors, computed by sae_b200_adam_step.

    ``renorm=True`` fuses the decoder-column and encoder-row renormalisation
    that the trainer runs right after ``optimizer.step()``
    (sae_trainer_rolling.py:3086-3090) into the same pass.
    """

    def __init__(self, params, lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, *,
                 sae: B200JumpReLUSAE, renorm: bool = False, fused=None, foreach=None):
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.sae = sae
        self.renorm = renorm
        self._index = {id(p): i for i, p in enumerate(_sae_params(sae))}
        for group in self.param_groups:
            for p in group["params"]:
                if id(p) not in self._index:
                    raise ValueError("B200Adam only optimises the parameters of its SAE")
        sae._state_probe = self._state_versions

    def _state_versions(self):
        out = []
        for i in (0, 2):
            p = _sae_params(self.sae)[i]
            st = self.state.get(p, {})
            if "exp_avg" in st:
                out.extend((st["exp_avg"]._version, st["exp_avg_sq"]._version))
        return out

    def _init_state(self, p):
        st = self.state[p]
        if "exp_avg" not in st:
            st["step"] = torch.tensor(0.0)
            st["exp_avg"] = torch.zeros_like(p, memory_format=torch.preserve_format)
            st["exp_avg_sq"] = torch.zeros_like(p, memory_format=torch.preserve_format)
        return st

    def load_state_dict(self, state_dict):
        super().load_state_dict(state_dict)
        # Loaded state may come from torch.optim.Adam with a [d, F]-contiguous
        # decoder state; move it to the feature-major layout of W_dec.weight.
        w_dec = self.sae.W_dec.weight
        st = self.state.get(w_dec, {})
        for k in ("exp_avg", "exp_avg_sq"):
            if k in st and not st[k].t().is_contiguous():
                st[k] = st[k].t().contiguous().t()
        for p, s in self.state.items():
            if "step" in s and torch.is_tensor(s["step"]) and s["step"].is_cuda:
                s["step"] = s["step"].detach().cpu()
        self.sae.mark_weights_dirty()

    @torch.no_grad()
    def step(self, closure=None, *, stats: Optional[torch.Tensor] = None,
             grad_scale_enc: float = 1.0):
        """One Adam update. ``stats`` (the device StepStats of a FusedStep)
        makes the update apply the clip coefficient computed on the device;
        ``grad_scale_enc`` is the W_enc dampening factor (3069-3074)."""
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        sae = self.sae
        params = _sae_params(sae)
        hyper = (L.AdamTensor * 5)()
        state = L.AdamState()
        grads = [None] * 5
        any_update = False
        for group in self.param_groups:
            b1, b2 = group["betas"]
            for p in group["params"]:
                i = self._index[id(p)]
                h = hyper[i]
                if p.grad is None:
                    h.skip = 1
                    continue
                _require_cuda(p, p.grad)
                st = self._init_state(p)
                st["step"] += 1
                g = p.grad
                if i == 2:
                    if not g.t().is_contiguous():
                        g = g.t().contiguous().t()
                        p.grad = g
                elif not g.is_contiguous():
                    g = g.contiguous()
                grads[i] = g
                h.lr = float(group["lr"])
                h.beta1 = float(b1)
                h.beta2 = float(b2)
                h.eps = float(group["eps"])
                h.weight_decay = float(group["weight_decay"])
                h.grad_scale = float(grad_scale_enc) if i in (0, 1) else 1.0
                h.step = int(round(float(st["step"])))
                h.use_clip = 1 if stats is not None else 0
                h.skip = 0
                h.renorm_rows = 1 if (self.renorm and i in (0, 2)) else 0
                state.exp_avg[i] = st["exp_avg"].data_ptr()
                state.exp_avg_sq[i] = st["exp_avg_sq"].data_ptr()
                any_update = True
        for i in range(5):
            if grads[i] is None:
                hyper[i].skip = 1
        if not any_update:
            return loss
        model = sae._model_struct(need_shadows=True)
        g = L.Grads(*(L.ptr(x) for x in grads))
        L.call("sae_b200_adam_step", ctypes.byref(model), ctypes.byref(g), ctypes.byref(state),
               hyper, L.ptr(stats), _stream())
        if hyper[0].skip == 0 and hyper[2].skip == 0:
            sae._shadows_written()
        else:
            sae.mark_weights_dirty()
        return loss


AUX_COEFF = 1.0 / 32   # sae_trainer_rolling.py:224 (Gao et al. 2024)


def _csr_capacity_default(tokens: int) -> int:
    per_token = int(os.environ.get("SAE_B200_CSR_PER_TOKEN", "512"))
    return max(1024, tokens * per_token)


class FusedStep:
    """Per-microbatch fused forward/backward plus the optimizer step."""

    def __init__(self, sae: B200JumpReLUSAE, optimizer: B200Adam, max_tokens: int,
                 csr_capacity: Optional[int] = None, force_simt: bool = False,
                 grad_feat: str = "sampled", pre_store: str = "entries",
                 auto_threshold: float = 400.0):
        _require_cuda(sae.W_enc.weight)
        if not isinstance(optimizer, B200Adam) or optimizer.sae is not sae:
            raise TypeError("FusedStep needs the B200Adam built over the same SAE")
        self.sae = sae
        self.opt = optimizer
        self.max_tokens = int(max_tokens)
        self.csr_capacity = int(csr_capacity or _csr_capacity_default(self.max_tokens))
        self.force_simt = bool(force_simt)
        if grad_feat not in ("sampled", "gemm", "auto"):
            raise ValueError("grad_feat must be 'sampled', 'gemm' or 'auto'")
        # "sampled": grad_feat = go . W_dec[f] only where the backward uses it
        # (active entries and the STE band); "gemm": the dense tcgen05 product;
        # "auto": sampled while the entries per token stay under auto_threshold
        # (the sampled cost grows with them, the GEMM's does not), the GEMM
        # above it, decided from the previous microbatch's statistics. Measured
        # at d=1536, F=49152: sampled still ahead at 299 entries per token
        # (14.7 against 16.5 ms per step), hence 400 (the CSR holds 512).
        self.grad_feat_mode = grad_feat
        self.grad_feat = "sampled" if grad_feat == "auto" else grad_feat
        self.auto_threshold = float(auto_threshold)
        self._band_ratio = 1.0    # entries / active entries of the last sampled microbatch
        if pre_store not in ("entries", "full"):
            raise ValueError("pre_store must be 'entries' or 'full'")
        # "entries": the encoder stores pre only in the 32-token words that hold
        # an active or in-band entry (all the sampled backward reads); "full":
        # all of it (for callers that read the workspace's pre). The aux loss and
        # the dense backward need it all and get it whatever this says.
        self.pre_store = pre_store
        dev = sae.W_enc.weight.device
        self.device = dev
        F, d = sae.n_features, sae.d_in
        self.ws_bytes = L.workspace_bytes(self.max_tokens, d, F, self.csr_capacity)
        self.ws = torch.empty(self.ws_bytes, device=dev, dtype=torch.uint8)
        self.stats = torch.zeros(L.STATS_FLOATS, device=dev, dtype=torch.int32)
        self.norm_ws = torch.empty(L.GRAD_NORM_WORKSPACE_BYTES, device=dev, dtype=torch.uint8)
        self.fired = torch.zeros(F, device=dev, dtype=torch.uint8)
        self._dense_scratch = None
        # Gradient buffers, bound as the parameters' .grad (W_dec's is the
        # [d, F] view of a feature-major buffer).
        self.g_W_enc = torch.zeros(F, d, device=dev)
        self.g_b_enc = torch.zeros(F, device=dev)
        self.g_W_dec_fm = torch.zeros(F, d, device=dev)
        self.g_b_dec = torch.zeros(d, device=dev)
        self.g_log_thr = torch.zeros(F, device=dev)
        # two pinned host copies of the StepStats: after the forward, after the norm
        self._host_stats_slots = [torch.zeros(L.STATS_FLOATS, dtype=torch.int32).pin_memory()
                                  for _ in range(2)] if torch.cuda.is_available() else None
        self.nnz_last = 0
        self.dense_fallbacks = 0
        # dead-feature aux loss state (set per step by set_aux)
        self._aux = None          # (dead int32 cuda tensor, k, coeff) or None
        # the StepConfig of a sampled backward whose per-feature sums of squares
        # grad_norm may use (set only while its after_backward runs)
        self._rows_cfg = None
        self._aux_ws = None
        self._x_hat = None

    # ------------------------------------------------------------ pieces
    def _bind_grads(self):
        sae = self.sae
        sae.W_enc.weight.grad = self.g_W_enc
        sae.W_enc.bias.grad = self.g_b_enc
        train_dec = sae.W_dec.weight.requires_grad
        sae.W_dec.weight.grad = self.g_W_dec_fm.t() if train_dec else None
        sae.b_dec.grad = self.g_b_dec
        sae.log_threshold.grad = self.g_log_thr

    def _grads_struct(self) -> L.Grads:
        train_dec = self.sae.W_dec.weight.requires_grad
        return L.Grads(L.ptr(self.g_W_enc), L.ptr(self.g_b_enc),
                       L.ptr(self.g_W_dec_fm) if train_dec else 0, L.ptr(self.g_b_dec),
                       L.ptr(self.g_log_thr))

    def _cfg(self, n_tokens, accum_steps, first, lambda_l0, al_mu, target_l0) -> L.StepConfig:
        entries = self.grad_feat == "sampled" and self.pre_store == "entries" and self._aux is None
        return L.StepConfig(int(n_tokens), self.csr_capacity, float(lambda_l0), float(al_mu),
                            float(target_l0), float(self.sae.ste_bandwidth), int(accum_steps),
                            0 if first else 1, 1 if self.sae.W_dec.weight.requires_grad else 0,
                            1 if self.force_simt else 0, 1 if self.grad_feat == "gemm" else 0,
                            1 if entries else 0)

    def set_aux(self, dead_indices: Optional[torch.Tensor], k: int = 0,
                coeff: float = AUX_COEFF) -> None:
        """Turn the dead-feature aux loss on for the following microbatches
        (sae_trainer_rolling.py:2986-2998): ``dead_indices`` are the features
        the revival controller reports dead (its ``aux_dead_mask()``, as
        ``torch.where(mask)[0]``), ``k`` the trainer's eff_k (clipped to the
        dead count). None or an empty set turns it off."""
        if dead_indices is None or dead_indices.numel() == 0 or k <= 0:
            self._aux = None
            return
        key = (id(dead_indices), dead_indices._version, int(k), float(coeff))
        if self._aux is not None and getattr(self, "_aux_key", None) == key:
            return          # the trainer refreshes its dead set every 250 steps
        self._aux_key = key
        dead = dead_indices.to(device=self.device, dtype=torch.int32).contiguous()
        lo, hi = int(dead.min()), int(dead.max())
        if lo < 0 or hi >= self.sae.n_features:
            raise ValueError("dead feature ids must lie in [0, n_features)")
        if dead.numel() > 1 and not bool((dead[1:] > dead[:-1]).all()):
            raise ValueError("dead feature ids must be strictly increasing")
        k = int(min(k, dead.numel()))
        need = L.aux_workspace_bytes(self.max_tokens, self.sae.d_in, self.sae.n_features,
                                     dead.numel(), k)
        if self._aux_ws is None or self._aux_ws.numel() < need:
            self._aux_ws = torch.empty(need, device=self.device, dtype=torch.uint8)
        if self._x_hat is None:
            self._x_hat = torch.empty(self.max_tokens, self.sae.d_in, device=self.device)
        self._aux = (dead, k, float(coeff))

    def _aux_struct(self) -> L.AuxConfig:
        dead, k, coeff = self._aux
        return L.AuxConfig(L.ptr(dead), dead.numel(), k, coeff)

    def _check_input(self, x: torch.Tensor) -> torch.Tensor:
        _require_cuda(x)
        if x.dim() != 2 or x.shape[1] != self.sae.d_in:
            raise ValueError(f"x must be [tokens, {self.sae.d_in}]")
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"microbatch of {x.shape[0]} tokens exceeds "
                             f"max_tokens={self.max_tokens}")
        if x.dtype not in (torch.bfloat16, torch.float32):
            x = x.float()
        return x.contiguous()

    def _dense_scratch_for(self, n_tokens: int) -> torch.Tensor:
        """Scratch of the dense weight-gradient path: the bf16 [F, ldp] dense
        operand plus the transposed xc and go (allocated on the first
        microbatch whose active set overflows the CSR)."""
        need = L.dense_scratch_bytes(n_tokens, self.sae.d_in, self.sae.n_features)
        if self._dense_scratch is None or self._dense_scratch.numel() < need:
            self._dense_scratch = torch.empty(need, device=self.device, dtype=torch.uint8)
        return self._dense_scratch

    def read_stats(self) -> dict:
        """One device->host copy of the StepStats (synchronises the stream)."""
        return self._wait_stats(self._copy_stats())

    def _copy_stats(self, slot: int = 0):
        """Queue a copy of the StepStats into pinned host slot ``slot``; returns
        the event to wait on (the stream keeps running behind it)."""
        buf = self._host_stats_slots[slot]
        buf.copy_(self.stats, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream())
        return slot, ev

    def _wait_stats(self, pending) -> dict:
        slot, ev = pending
        ev.synchronize()
        raw = L.StepStats.from_buffer_copy(self._host_stats_slots[slot].numpy().tobytes())
        return {k: getattr(raw, k) for k in L.STATS_FIELDS}

    def microbatch(self, x: torch.Tensor, *, accum_steps: int = 1, first: bool = True,
                   lambda_l0: float = 0.0, al_mu: float = 0.0, target_l0: float = 0.0,
                   x_hat_out: Optional[torch.Tensor] = None,
                   after_backward: Optional[Callable[[], None]] = None) -> dict:
        """Forward + backward of one microbatch; gradients overwrite (first) or
        add. Reads the forward statistics back once and returns them. The
        sampled backward is queued before that read: its kernels do nothing
        when the active set overflowed the CSR, and the read then selects the
        dense path (an active set larger than the workspace is never
        truncated). ``after_backward`` (e.g. the gradient norm) is queued right
        after the backward, before the host waits, and again if the backward
        had to be redone. A ``grad_norm`` that it calls straight after the
        sampled backward is summed from that backward's per-feature partials,
        so it must not edit the gradients before that call."""
        sae = self.sae
        x = self._check_input(x)
        n = x.shape[0]
        if first:
            self.fired.zero_()
        cfg = self._cfg(n, accum_steps, first, lambda_l0, al_mu, target_l0)
        model = sae._model_struct(need_shadows=True)
        stream = _stream()
        dt = L.DTYPE_BF16 if x.dtype == torch.bfloat16 else L.DTYPE_F32
        if self._aux is not None and x_hat_out is None:
            x_hat_out = self._x_hat[:n]

        def forward():
            L.call("sae_b200_train_forward", ctypes.byref(model), L.ptr(x), dt,
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                   L.ptr(x_hat_out), L.ptr(self.fired), stream)

        forward()
        if self._aux is not None:
            aux = self._aux_struct()
            L.call("sae_b200_aux_forward", ctypes.byref(model), L.ptr(x), dt, L.ptr(x_hat_out),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, ctypes.byref(aux),
                   L.ptr(self._aux_ws), self._aux_ws.numel(), L.ptr(self.stats), stream)
        pending = self._copy_stats(0)
        grads = self._grads_struct()

        def sparse_backward():
            L.call("sae_b200_train_backward", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats), stream)

        # without the aux loss, the sampled backward goes ahead of the read
        ahead = self._aux is None and self.grad_feat == "sampled"
        if ahead:
            sparse_backward()
            if after_backward is not None:
                # the norm from the backward's per-feature sums of squares; if the
                # CSR overflowed, the dense redo below queues the full norm again
                self._rows_cfg = cfg
                try:
                    after_backward()
                finally:
                    self._rows_cfg = None
        st = self._wait_stats(pending)
        self.nnz_last = st["nnz"]
        redone = not ahead
        if st["csr_overflow"]:
            self.dense_fallbacks += 1
            if cfg.pre_entries_only:
                # the dense backward reads all of pre: store it (the forward's
                # encoder again, on the same workspace)
                L.call("sae_b200_store_full_pre", ctypes.byref(model), ctypes.byref(cfg),
                       L.ptr(self.ws), self.ws_bytes, stream)
                cfg.pre_entries_only = 0
            scratch = self._dense_scratch_for(n)
            L.call("sae_b200_train_backward_dense", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, L.ptr(self.stats),
                   L.ptr(scratch), scratch.numel(), stream)
            redone = True
        else:
            sae._sparse_decode_calls += 1
            if not ahead:
                sparse_backward()
        if self._aux is not None:
            aux = self._aux_struct()
            L.call("sae_b200_aux_backward", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, ctypes.byref(aux),
                   L.ptr(self._aux_ws), self._aux_ws.numel(), stream)
        if redone and after_backward is not None:
            after_backward()
        self._bind_grads()
        self._auto_update(st, n)
        return st

    def _auto_update(self, st: dict, n_tokens: int) -> None:
        """grad_feat="auto": pick the next microbatch's backward from this one's
        entry count (sampled entries per token; in GEMM mode the active count
        scaled by the last sampled microbatch's entries-per-active ratio), with
        a 20% hysteresis so that it does not flip back and forth."""
        if self.grad_feat_mode != "auto" or st["csr_overflow"] or n_tokens <= 0:
            return
        if self.grad_feat == "sampled":
            self._band_ratio = st["csr_pairs"] / max(1, st["nnz"])
            if st["csr_pairs"] / n_tokens > self.auto_threshold:
                self.grad_feat = "gemm"
        elif st["nnz"] * self._band_ratio / n_tokens < 0.8 * self.auto_threshold:
            self.grad_feat = "sampled"

    def grad_norm(self, max_norm: float = 1.0) -> None:
        """Global L2 norm of all gradients + clip coefficient, on the device.
        Straight after a sampled backward (no aux loss) it is summed from that
        backward's per-feature partials instead of a pass over the gradients."""
        model = self.sae._model_struct(need_shadows=False)
        grads = self._grads_struct()
        cfg = getattr(self, "_rows_cfg", None)
        if cfg is not None:
            L.call("sae_b200_grad_norm_sampled", ctypes.byref(model), ctypes.byref(grads),
                   ctypes.byref(cfg), L.ptr(self.ws), self.ws_bytes, float(max_norm),
                   L.ptr(self.norm_ws), self.norm_ws.numel(), L.ptr(self.stats), _stream())
            return
        L.call("sae_b200_grad_norm", ctypes.byref(model), ctypes.byref(grads), float(max_norm),
               L.ptr(self.norm_ws), self.norm_ws.numel(), L.ptr(self.stats), _stream())

    def optimizer_step(self, wenc_factor: float = 1.0) -> None:
        self.opt.step(stats=self.stats, grad_scale_enc=wenc_factor if wenc_factor < 1.0 else 1.0)

    # ---------------------------------------------------------- full step
    def step(self, batch: torch.Tensor, *, microbatch_tokens: Optional[int] = None,
             lambda_l0: float = 0.0, al_mu: float = 0.0, target_l0: float = 0.0,
             max_norm: float = 1.0,
             wenc_dampen: Optional[Callable[[float], float]] = None,
             aux_dead: Optional[torch.Tensor] = None, aux_k: int = 0,
             aux_coeff: float = AUX_COEFF) -> dict:
        """One optimizer step over ``batch`` split into microbatches, in the
        reference loop's order; returns recon / l0 / grad_norm as floats after
        the same single stats read-back the loop does before Adam (3064-3066).
        ``aux_dead`` / ``aux_k``: the dead-feature aux loss (see set_aux)."""
        self.set_aux(aux_dead, aux_k, aux_coeff)
        mb = int(microbatch_tokens or batch.shape[0])
        n = batch.shape[0]
        if n % mb != 0:
            raise ValueError("batch tokens must be divisible by microbatch_tokens")
        accum = n // mb
        recon = 0.0
        l0 = 0.0
        loss = 0.0
        aux = 0.0
        norm_stats = []

        def norm():
            # clip_grad_norm_ (3049) and its statistics read, queued ahead of Adam
            self.grad_norm(max_norm)
            norm_stats[:] = [self._copy_stats(1)]

        for i in range(accum):
            s = self.microbatch(batch[i * mb:(i + 1) * mb], accum_steps=accum, first=(i == 0),
                                lambda_l0=lambda_l0, al_mu=al_mu, target_l0=target_l0,
                                after_backward=norm if i == accum - 1 else None)
            recon += s["recon_loss"] * accum     # accum_recon_t (3057)
            l0 += s["l0"]                        # accum_l0_t (3058)
            loss += s["loss"]
            aux += s["aux_loss"]
        l0_step = l0 / accum
        factor = 1.0 if wenc_dampen is None else float(wenc_dampen(l0_step))
        self.optimizer_step(factor)              # clip coefficient applied on the device
        s = self._wait_stats(norm_stats[0])      # Adam keeps running meanwhile
        return {"recon_loss": recon / accum, "l0": l0_step, "grad_norm": s["grad_norm"],
                "clip_coef": s["clip_coef"], "nnz": s["nnz"], "csr_pairs": s["csr_pairs"],
                "loss": loss,
                "aux_loss": aux, "wenc_factor": factor}

    @property
    def fired_mask(self) -> torch.Tensor:
        """Features that fired in this step's microbatches (fired_accum, 3016)."""
        return self.fired.view(torch.bool)
