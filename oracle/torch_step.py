"""The reference trainer's fp32 CPU training step, restated with torch CPU
operators -- TEST INFRASTRUCTURE AND CPU BASELINE ONLY.

The arithmetic is that of ``sae_oracle``'s "fp32" mode (one microbatch's
forward, closed-form backward, ``clip_grad_norm_``, the 4-group
``torch.optim.Adam`` and both renormalisations of
``sae_trainer_rolling.py:2914-3090``), written with the torch operators the
reference itself runs on a CPU (addmm / matmul on MKL, elementwise kernels,
``torch.optim.Adam``'s in-place update), so that timing it on the host cores
measures the reference's own CPU cost: ``bench.py``'s ``cpu_baseline`` and
``--impl reference`` legs time this module. ``tests/test_oracle_golden.py``
pins it to the reference-run fixture ``tests/golden/cfg1_f32.npz``. Only
``tests/`` and ``bench.py`` import it; the product path (``sae_b200``) never
does.
"""
from __future__ import annotations

import math

import torch

INIT_THRESHOLD = 0.1   # sae_trainer_rolling.py:212


class TorchReferenceStep:
    """One JumpReLU SAE with the reference layout (W_enc [F, d], W_dec [d, F])
    and the trainer's optimizer, on the CPU in fp32."""

    def __init__(self, d: int, F: int, *, seed: int = 0, lr: float = 2e-4,
                 decoder_wd: float = 1e-4, ste_bandwidth: float = 0.2, lambda_l0: float = 1e-3,
                 al_mu: float = 1e-2, target_l0: float = 50.0):
        # _make_sae (961-966) then _JumpReLUSAE.__init__ (772-800): two nn.Linear
        # initialisations (their RNG draws happen), orthogonal_ on the [d, F]
        # decoder, unit columns, W_enc = W_dec^T, b_enc = 0, log θ = log 0.1.
        torch.manual_seed(seed)
        enc = torch.nn.Linear(d, F, bias=True)
        dec = torch.nn.Linear(F, d, bias=False)
        with torch.no_grad():
            torch.nn.init.orthogonal_(dec.weight)
            dec.weight.div_(dec.weight.norm(dim=0, keepdim=True).clamp(min=1e-8))
            enc.weight.copy_(dec.weight.t())
            enc.bias.zero_()
        self.d, self.F = d, F
        self.W_enc = torch.nn.Parameter(enc.weight.detach().clone())
        self.b_enc = torch.nn.Parameter(enc.bias.detach().clone())
        self.W_dec = torch.nn.Parameter(dec.weight.detach().clone())
        self.b_dec = torch.nn.Parameter(torch.zeros(d))
        self.log_threshold = torch.nn.Parameter(torch.full((F,), math.log(INIT_THRESHOLD)))
        self.eps = float(ste_bandwidth)
        self.lambda_l0, self.al_mu, self.target_l0 = float(lambda_l0), float(al_mu), float(target_l0)
        self.lr, self.decoder_wd = float(lr), float(decoder_wd)
        # the trainer's four groups (2536-2540)
        self.opt = torch.optim.Adam(
            [{"params": [self.W_enc, self.b_enc], "weight_decay": 0},
             {"params": [self.W_dec], "weight_decay": decoder_wd},
             {"params": [self.b_dec], "weight_decay": 0},
             {"params": [self.log_threshold], "weight_decay": 0}], lr=lr, betas=(0.9, 0.999))

    def params(self):
        return (self.W_enc, self.b_enc, self.W_dec, self.b_dec, self.log_threshold)

    @torch.no_grad()
    def microbatch(self, x: torch.Tensor, accum_steps: int = 1, first: bool = True) -> dict:
        """Forward and backward of one microbatch; gradients overwrite (first)
        or add, as autograd's accumulation into .grad does."""
        B, d = x.shape
        W_enc, b_enc, W_dec, b_dec, log_thr = self.params()
        # _EncoderPreBias.forward 584-590, _jumprelu_forward 827-901
        xc = x - b_dec
        pre = torch.addmm(b_enc, xc, W_enc.t())
        theta = log_thr.exp()
        gate = (pre > theta).to(pre.dtype)
        feat = pre * gate
        # decode 922-925, loss 2963-2974
        x_hat = torch.addmm(b_dec, feat, W_dec.t())
        r = x - x_hat
        recon = float(r.square().mean()) / accum_steps
        l0 = float(gate.sum(dim=1).mean())
        diff = l0 - self.target_l0
        slack = max(diff, 0.0)
        gate_grad = (self.lambda_l0 + self.al_mu * slack) / accum_steps / B if diff >= 0 else 0.0
        # decoder backward (639-654 / the dense autograd of 924): go = dL/dx_hat
        go = r.mul_(-2.0 / (accum_steps * B * d))
        g_bdec = go.sum(dim=0)
        grad_feat = go @ W_dec
        dW_dec = go.t() @ feat
        # straight-through threshold gradient (_log_threshold_hook 792-825)
        comb = pre * grad_feat
        comb.add_(gate_grad)
        in_band = (pre - theta).abs_() < self.eps
        thr_sum = torch.where(in_band, comb, 0.0).sum(dim=0)
        g_logthr = -(thr_sum / (2 * self.eps)) * theta
        # encoder backward with the reassociated b_dec term (592-607)
        dpre = grad_feat.mul_(gate)
        db_enc = dpre.sum(dim=0)
        dW_enc = dpre.t() @ xc
        g_bdec.sub_(db_enc @ W_enc)
        for p, g in zip(self.params(), (dW_enc, db_enc, dW_dec, g_bdec, g_logthr)):
            if first or p.grad is None:
                p.grad = g
            else:
                p.grad.add_(g)
        return {"recon_loss": recon, "l0": l0}

    def optimizer_step(self, max_norm: float = 1.0) -> float:
        """clip_grad_norm_ (3049), Adam (3076), _normalize_decoder (778-782) and
        the W_enc row renorm (3089-3090). Returns the pre-clip norm."""
        norm = float(torch.nn.utils.clip_grad_norm_(self.params(), max_norm))
        self.opt.step()
        with torch.no_grad():
            self.W_dec.div_(self.W_dec.norm(dim=0, keepdim=True).clamp(min=1e-8))
            self.W_enc.div_(self.W_enc.norm(dim=1, keepdim=True).clamp(min=1e-8))
        return norm

    def step(self, xs) -> dict:
        """One optimizer step over the microbatches ``xs``."""
        outs = [self.microbatch(x, len(xs), i == 0) for i, x in enumerate(xs)]
        norm = self.optimizer_step()
        return {"recon_loss": sum(o["recon_loss"] for o in outs),
                "l0": sum(o["l0"] for o in outs) / len(outs), "grad_norm": norm}

    def slice_features(self, n: int) -> "TorchReferenceStep":
        """A copy restricted to the first n features (their W_enc rows, b_enc,
        W_dec columns, thresholds; b_dec whole), with fresh optimizer state and
        the same hyper-parameters: the clip norm, Adam and both renorms are
        passes over the parameters, so their time on a 1/k slice is 1/k of the
        full pass."""
        s = TorchReferenceStep.__new__(TorchReferenceStep)
        s.d, s.F = self.d, n
        s.W_enc = torch.nn.Parameter(self.W_enc.detach()[:n].clone())
        s.b_enc = torch.nn.Parameter(self.b_enc.detach()[:n].clone())
        s.W_dec = torch.nn.Parameter(self.W_dec.detach()[:, :n].contiguous())
        s.b_dec = torch.nn.Parameter(self.b_dec.detach().clone())
        s.log_threshold = torch.nn.Parameter(self.log_threshold.detach()[:n].clone())
        if self.W_enc.grad is not None:
            s.W_enc.grad = self.W_enc.grad[:n].clone()
            s.b_enc.grad = self.b_enc.grad[:n].clone()
            s.W_dec.grad = self.W_dec.grad[:, :n].contiguous()
            s.b_dec.grad = self.b_dec.grad.clone()
            s.log_threshold.grad = self.log_threshold.grad[:n].clone()
        s.eps, s.lambda_l0, s.al_mu, s.target_l0 = self.eps, self.lambda_l0, self.al_mu, \
            self.target_l0
        s.lr, s.decoder_wd = self.lr, self.decoder_wd
        s.opt = torch.optim.Adam(
            [{"params": [s.W_enc, s.b_enc], "weight_decay": 0},
             {"params": [s.W_dec], "weight_decay": self.decoder_wd},
             {"params": [s.b_dec], "weight_decay": 0},
             {"params": [s.log_threshold], "weight_decay": 0}], lr=self.lr, betas=(0.9, 0.999))
        return s
