"""CPU oracle for the JumpReLU SAE training step -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the per-step compute of the reference trainer
(JuiceB0xC0de/event-aware-SAE-trainer, ``sae_trainer_rolling.py``) so that the
CUDA library can be checked against it. It is imported only by ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py``; the product path (``sae_b200``) never imports it.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
module (``_make_sae``, ``encode_pre``, ``jumprelu_with_gate``, ``decode``, the
trainer's loss lines, ``loss.backward()``, ``clip_grad_norm_``, the 4-group
``torch.optim.Adam`` and both renormalisations) on CPU in float64 and float32
and stores the results under ``tests/golden/``; ``tests/test_oracle_golden.py``
checks this restatement against them.

Three precisions:
  * ``"fp64"`` / ``"fp32"``: the reference's CPU path (no autocast, all fp32),
    evaluated in that dtype.
  * ``"bf16"``: the reference's CUDA path under ``torch.amp.autocast(bf16)``
    (sae_trainer_rolling.py:2407-2410, 2919). Rounding to bf16 happens exactly
    where autocast puts it -- the ``x - b_dec`` input and the weights of the
    encoder addmm, its output ``pre``, the decoder GEMM's inputs and output, the
    loss gradient entering the decoder GEMMs, and ``grad_feat`` -- while every
    accumulation runs in float64. The reference additionally rounds the weight
    gradients of its bf16 GEMMs (dW_enc, dW_dec, db_enc and the b_dec GEMV) to
    bf16; ``round_weight_grads=True`` reproduces that, the default keeps them
    exact (what the CUDA library returns).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


# --------------------------------------------------------------------- bf16
def bf16(a) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even), returned as float32."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    u = a.view(np.uint32).astype(np.uint64)
    bias = ((u >> 16) & 1) + 0x7FFF
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.nan
    return out


# ------------------------------------------------------------------- config
@dataclass
class StepConfig:
    """Scalars of one training step (sae_trainer_rolling.py:2914-3090)."""
    lambda_l0: float = 1e-3          # scheduler.lambda_l0
    al_mu: float = 1e-2              # sae_cfg.al_mu
    target_l0: float = 50.0          # sae_cfg.target_l0 (= K)
    ste_bandwidth: float = 0.2       # sae.ste_bandwidth
    accum_steps: int = 1
    max_norm: float = 1.0            # clip_grad_norm_(..., 1.0), 3049
    wenc_factor: float = 1.0         # scheduler.wenc_dampen_factor(l0), 3069-3074
    lr: tuple = (1e-4, 1e-4, 1e-4, 1e-4)          # per param group
    betas: tuple = ((0.9, 0.999),) * 4
    weight_decay: tuple = (0.0, 1e-4, 0.0, 0.0)   # 2536-2540
    adam_eps: float = 1e-8
    train_decoder: bool = True
    # dead-feature aux loss (2986-2998): sorted dead feature ids, top-k per token
    aux_dead: np.ndarray | None = None
    aux_k: int = 0
    aux_coeff: float = 1.0 / 32      # AUX_COEFF, sae_trainer_rolling.py:224


@dataclass
class Params:
    """SAE parameters in the reference's layouts (W_dec is [d, F])."""
    W_enc: np.ndarray     # [F, d]
    b_enc: np.ndarray     # [F]
    W_dec: np.ndarray     # [d, F]
    b_dec: np.ndarray     # [d]
    log_threshold: np.ndarray  # [F]

    def copy(self) -> "Params":
        return Params(*(np.array(getattr(self, k), copy=True) for k in PARAM_NAMES))

    def astype(self, dt) -> "Params":
        return Params(*(np.asarray(getattr(self, k), dtype=dt) for k in PARAM_NAMES))


PARAM_NAMES = ("W_enc", "b_enc", "W_dec", "b_dec", "log_threshold")


@dataclass
class ForwardOut:
    theta: np.ndarray
    xc: np.ndarray
    pre: np.ndarray
    gate: np.ndarray
    feat: np.ndarray
    x_hat: np.ndarray
    residual: np.ndarray
    counts: np.ndarray
    recon_loss: float
    l0: float
    sparsity_loss: float
    gate_grad: float
    loss: float
    aux_loss: float = 0.0
    aux_acts: np.ndarray | None = None   # [B, n_dead] top-k relu(pre) of the dead features
    x_aux: np.ndarray | None = None


@dataclass
class Grads:
    W_enc: np.ndarray
    b_enc: np.ndarray
    W_dec: np.ndarray
    b_dec: np.ndarray
    log_threshold: np.ndarray
    extras: dict = field(default_factory=dict)


def _dt(precision: str):
    return np.float64 if precision == "fp64" else np.float32


# ------------------------------------------------------------------ forward
def forward(x: np.ndarray, p: Params, cfg: StepConfig, precision: str = "fp32",
            theta: np.ndarray | None = None, pre: np.ndarray | None = None) -> ForwardOut:
    """Encoder + JumpReLU + dense decode + loss terms of one microbatch.

    sae_trainer_rolling.py: _EncoderPreBias.forward 584-590 (pre = addmm(b_enc,
    x - b_dec, W_enc^T)); _jumprelu_forward 827-901 (theta = exp(logθ), gate =
    1[pre > theta], feat = pre * gate); decode 922-925 (x_hat = W_dec(feat) +
    b_dec); loss 2963-2974 (recon = mean((x - x_hat)^2)/accum, l0 = mean gate
    count, slack = max(0, l0 - target), sparsity = (λ s + ½ μ s²)/accum).

    ``theta`` overrides exp(log_threshold): bf16 pre-activations sit on a coarse
    grid, so a threshold one float32 ulp away moves whole grid points across
    the gate or the STE band edge. Parity checks of a GPU path therefore pass
    the thresholds that path computed (after checking them against exp).
    ``pre`` (bf16 mode) likewise replaces the pre-activations by the GPU's own
    bf16 values, so that a backward check sees exactly the same gates.
    """
    B = x.shape[0]
    acc_dt = np.float64 if precision in ("fp64", "bf16") else np.float32
    if precision == "bf16":
        if theta is None:
            theta = np.exp(p.log_threshold.astype(np.float32)).astype(np.float32)
        theta = np.asarray(theta, np.float32)
        xc = bf16(x.astype(np.float32) - p.b_dec.astype(np.float32))
        if pre is None:
            pre = bf16((xc.astype(acc_dt) @ bf16(p.W_enc).astype(acc_dt).T
                        + bf16(p.b_enc).astype(acc_dt)).astype(np.float32))
        pre = np.asarray(pre, np.float32)
        gate = (pre > theta).astype(np.float32)
        feat = pre * gate
        dec = bf16((bf16(feat).astype(acc_dt) @ bf16(p.W_dec).astype(acc_dt).T).astype(np.float32))
        x_hat = dec + p.b_dec.astype(np.float32)
        residual = x.astype(np.float32) - x_hat
    else:
        dt = _dt(precision)
        x = x.astype(dt)
        theta = np.exp(p.log_threshold.astype(dt)) if theta is None else np.asarray(theta, dt)
        xc = x - p.b_dec.astype(dt)
        pre = xc @ p.W_enc.astype(dt).T + p.b_enc.astype(dt)
        gate = (pre > theta).astype(dt)
        feat = pre * gate
        x_hat = feat @ p.W_dec.astype(dt).T + p.b_dec.astype(dt)
        residual = x - x_hat
    counts = gate.sum(axis=1)
    n = residual.size
    recon = float(np.square(residual.astype(acc_dt)).sum() / n / cfg.accum_steps)
    l0 = float(counts.astype(np.float64).mean())
    diff = l0 - cfg.target_l0
    slack = max(diff, 0.0)
    sparsity = (cfg.lambda_l0 * slack + 0.5 * cfg.al_mu * slack * slack) / cfg.accum_steps
    # d sparsity / d gate[b, f]: clamp(min=0) passes the gradient where diff >= 0,
    # the mean divides by B.
    gate_grad = ((cfg.lambda_l0 + cfg.al_mu * slack) / cfg.accum_steps / B) if diff >= 0 else 0.0
    fw = ForwardOut(theta, xc, pre, gate, feat, x_hat, residual, counts, recon, l0, sparsity,
                    gate_grad, recon + sparsity)
    if cfg.aux_dead is not None and len(cfg.aux_dead) and cfg.aux_k > 0:
        aux_forward(fw, p, cfg, precision)
    return fw


def aux_select(pre_dead: np.ndarray, k: int) -> np.ndarray:
    """relu then top-k per row (torch.topk, 2988-2991), dense [B, n_dead] with
    the unselected entries zero. Ties go to the lower dead index."""
    v = np.maximum(pre_dead, 0)
    idx = np.argsort(-v, axis=1, kind="stable")[:, :k]
    out = np.zeros_like(v)
    np.put_along_axis(out, idx, np.take_along_axis(v, idx, axis=1), axis=1)
    return out


def aux_forward(fw: ForwardOut, p: Params, cfg: StepConfig, precision: str) -> None:
    """Dead-feature aux loss (sae_trainer_rolling.py:2986-2998): the top-k
    relu'd pre-activations of the dead features reconstruct the (detached)
    residual through their decoder columns; aux = AUX_COEFF * mean((r - x_aux)^2)
    / accum. In bf16 mode x_aux is the bf16 output of the autocast matmul."""
    dead = np.asarray(cfg.aux_dead)
    k = min(int(cfg.aux_k), len(dead))
    acts = aux_select(fw.pre[:, dead], k)
    if precision == "bf16":
        x_aux = bf16((acts.astype(np.float64) @ bf16(p.W_dec[:, dead]).astype(np.float64).T)
                     .astype(np.float32))
        err = fw.residual.astype(np.float64) - x_aux
    else:
        dt = _dt(precision)
        x_aux = (acts.astype(dt) @ p.W_dec[:, dead].astype(dt).T).astype(dt)
        err = fw.residual.astype(dt) - x_aux
    fw.aux_acts = acts
    fw.x_aux = x_aux
    fw.aux_loss = float(np.square(err.astype(np.float64)).mean() * cfg.aux_coeff / cfg.accum_steps)
    fw.loss += fw.aux_loss


def aux_backward(x, p: Params, fw: ForwardOut, cfg: StepConfig, precision: str):
    """Gradients of the aux loss: g = dAux/dx_aux = -2 coeff (r - x_aux) /
    (B d accum); dpre[:, dead] = (g W_dec_dead) on the selected entries with
    pre > 0 (topk gather + relu backward); dW_dec[:, dead] = g^T aux_acts.
    The residual is detached (2996), so nothing flows into the main path."""
    B, d = x.shape
    dead = np.asarray(cfg.aux_dead)
    scale = 2.0 * cfg.aux_coeff / (B * d * cfg.accum_steps)
    sel = fw.aux_acts > 0
    if precision == "bf16":
        a = np.float64
        err = (fw.residual.astype(np.float64) - fw.x_aux).astype(np.float32)
        g = bf16((-np.float32(scale) * err).astype(np.float32))
        wd = bf16(p.W_dec[:, dead]).astype(a)                  # [d, n_dead]
        d_acts = bf16((g.astype(a) @ wd).astype(np.float32))   # [B, n_dead]
        dpre_dead = np.where(sel, d_acts, 0.0).astype(np.float32)
        dW_dead = g.astype(a).T @ bf16(fw.aux_acts).astype(a)  # [d, n_dead]
    else:
        dt = _dt(precision)
        err = fw.residual.astype(dt) - fw.x_aux
        g = (-scale * err).astype(dt)
        d_acts = g @ p.W_dec[:, dead].astype(dt)
        dpre_dead = np.where(sel, d_acts, 0.0).astype(dt)
        dW_dead = g.T @ fw.aux_acts.astype(dt)
    return dpre_dead, dW_dead


# ----------------------------------------------------------------- backward
def backward(x: np.ndarray, p: Params, fw: ForwardOut, cfg: StepConfig,
             precision: str = "fp32", round_weight_grads: bool = False) -> Grads:
    """Closed-form gradients of the microbatch loss.

    Decoder: go = dL/dx_hat = -2 r / (B d accum); grad_b_dec += Σ_b go (the
    fp32 add at 924); grad_feat = go W_dec (dense on purpose, 613-626);
    dW_dec = go^T feat (645-652).
    JumpReLU STE (_log_threshold_hook 792-825): combined = pre * grad_feat +
    gate_grad; dlogθ = -Σ_b where(|pre - θ| < ε, combined) / (2ε) * θ;
    grad_pre = grad_feat * gate.
    Encoder (_EncoderPreBias.backward 592-607): dW_enc = dpre^T xc,
    db_enc = Σ_b dpre, db_dec -= (Σ_b dpre) W_enc.
    """
    B, d = x.shape
    eps = cfg.ste_bandwidth
    if precision == "bf16":
        a = np.float64
        go = -(np.float32(1.0 / (cfg.accum_steps * B * d)) * (2.0 * fw.residual)).astype(np.float32)
        go_b = bf16(go)
        Wd = bf16(p.W_dec).astype(a)          # [d, F]
        We = bf16(p.W_enc).astype(a)          # [F, d]
        gb_dec = go.astype(a).sum(axis=0)
        grad_feat = bf16((go_b.astype(a) @ Wd).astype(np.float32))
        dW_dec = go_b.astype(a).T @ bf16(fw.feat).astype(a)
        pre = fw.pre.astype(np.float32)
        comb = (pre * grad_feat).astype(np.float32) + np.float32(fw.gate_grad)
        in_band = np.abs(pre - fw.theta) < np.float32(eps)
        thr_sum = np.where(in_band, comb, 0.0).astype(a).sum(axis=0)
        dpre = grad_feat * fw.gate
        db_enc = dpre.astype(a).sum(axis=0)
        dW_enc = dpre.astype(a).T @ fw.xc.astype(a)
        if round_weight_grads:
            dW_dec = bf16(dW_dec)
            dW_enc = bf16(dW_enc)
            db_enc = bf16(db_enc)
            gb_dec_enc = bf16(-(bf16(db_enc).astype(a) @ We))
        else:
            gb_dec_enc = -(db_enc @ We)
        g_logthr = -(thr_sum / (2 * eps)) * fw.theta.astype(a)
        if fw.aux_acts is not None:
            dead = np.asarray(cfg.aux_dead)
            dpre_dead, dW_dead = aux_backward(x, p, fw, cfg, precision)
            dpre_aux = np.zeros_like(dpre)
            dpre_aux[:, dead] = dpre_dead
            db_aux = dpre_aux.astype(a).sum(axis=0)
            db_enc = db_enc + db_aux
            dW_enc = dW_enc + dpre_aux.astype(a).T @ fw.xc.astype(a)
            dW_dec = dW_dec.copy()
            dW_dec[:, dead] += dW_dead
            gb_dec_enc = -(db_enc @ We)
            dpre = dpre + dpre_aux
        out = Grads(dW_enc.astype(np.float32), db_enc.astype(np.float32),
                    dW_dec.astype(np.float32), (gb_dec + gb_dec_enc).astype(np.float32),
                    g_logthr.astype(np.float32))
        out.extras = {"go": go_b, "grad_feat": grad_feat, "dpre": dpre}
    else:
        dt = _dt(precision)
        r = fw.residual.astype(dt)
        go = -(2.0 * r) / (cfg.accum_steps * B * d)
        go = go.astype(dt)
        gb_dec = go.sum(axis=0)
        grad_feat = go @ p.W_dec.astype(dt)                 # [B, F]
        dW_dec = go.T @ fw.feat                             # [d, F]
        comb = fw.pre * grad_feat + dt(fw.gate_grad)
        in_band = np.abs(fw.pre - fw.theta) < eps
        thr_sum = np.where(in_band, comb, 0.0).sum(axis=0)
        dpre = grad_feat * fw.gate
        if fw.aux_acts is not None:
            dead = np.asarray(cfg.aux_dead)
            dpre_dead, dW_dead = aux_backward(x, p, fw, cfg, precision)
            dpre = dpre.copy()
            dpre[:, dead] += dpre_dead
            dW_dec = dW_dec.copy()
            dW_dec[:, dead] += dW_dead
        db_enc = dpre.sum(axis=0)
        dW_enc = dpre.T @ fw.xc
        gb_dec = gb_dec - db_enc @ p.W_enc.astype(dt)
        g_logthr = -(thr_sum / (2 * eps)) * fw.theta
        out = Grads(dW_enc, db_enc, dW_dec, gb_dec, g_logthr.astype(dt))
        out.extras = {"go": go, "grad_feat": grad_feat, "dpre": dpre}
    if not cfg.train_decoder:
        out.W_dec = None
    return out


def add_grads(a: Grads | None, b: Grads) -> Grads:
    """Gradient accumulation across microbatches (autograd's += into .grad)."""
    if a is None:
        return b
    return Grads(*(None if getattr(a, k) is None else getattr(a, k) + getattr(b, k)
                   for k in PARAM_NAMES))


# ------------------------------------------------------------ clip + Adam
def clip_coef(g: Grads, max_norm: float) -> tuple[float, float]:
    """torch.nn.utils.clip_grad_norm_ (called at 3049): total L2 norm over all
    gradients and the clamped coefficient max_norm / (norm + 1e-6)."""
    tot = 0.0
    for k in PARAM_NAMES:
        v = getattr(g, k)
        if v is not None:
            tot += float(np.square(v.astype(np.float64)).sum())
    norm = math.sqrt(tot)
    return norm, min(1.0, max_norm / (norm + 1e-6))


@dataclass
class AdamState:
    exp_avg: dict
    exp_avg_sq: dict
    step: int = 0

    @staticmethod
    def zeros_like(p: Params) -> "AdamState":
        return AdamState({k: np.zeros_like(getattr(p, k)) for k in PARAM_NAMES},
                         {k: np.zeros_like(getattr(p, k)) for k in PARAM_NAMES}, 0)


_GROUP_OF = {"W_enc": 0, "b_enc": 0, "W_dec": 1, "b_dec": 2, "log_threshold": 3}


def adam_step(p: Params, g: Grads, st: AdamState, cfg: StepConfig, clip: float) -> Params:
    """Clip scale, W_enc dampening (3069-3074), then torch.optim.Adam with L2
    weight decay per param group (2536-2541; torch's _fused_adam order:
    g += wd*p; m = β1 m + (1-β1) g; v = β2 v + (1-β2) g²;
    p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps)), then the decoder-column and
    encoder-row renormalisations (_normalize_decoder 778-782, 3086-3090)."""
    st.step += 1
    out = p.copy()
    for k in PARAM_NAMES:
        gk = getattr(g, k)
        if gk is None:
            continue
        grp = _GROUP_OF[k]
        b1, b2 = cfg.betas[grp]
        lr, wd = cfg.lr[grp], cfg.weight_decay[grp]
        pk = getattr(out, k)
        gk = gk * clip
        if k in ("W_enc", "b_enc") and cfg.wenc_factor < 1.0:
            gk = gk * cfg.wenc_factor
        if wd != 0:
            gk = gk + wd * pk
        m = st.exp_avg[k] = b1 * st.exp_avg[k] + (1 - b1) * gk
        v = st.exp_avg_sq[k] = b2 * st.exp_avg_sq[k] + (1 - b2) * gk * gk
        bc1 = 1 - b1 ** st.step
        bc2 = 1 - b2 ** st.step
        denom = np.sqrt(v) / math.sqrt(bc2) + cfg.adam_eps
        setattr(out, k, (pk - (lr / bc1) * m / denom).astype(pk.dtype))
    if cfg.train_decoder:
        out.W_dec = out.W_dec / np.maximum(np.linalg.norm(out.W_dec, axis=0, keepdims=True), 1e-8)
    out.W_enc = out.W_enc / np.maximum(np.linalg.norm(out.W_enc, axis=1, keepdims=True), 1e-8)
    return out


# --------------------------------------------------------------- full step
@dataclass
class StepResult:
    params: Params
    grads: Grads
    fw: list
    grad_norm: float
    clip: float
    recon_loss: float
    l0: float


def train_step(xs, p: Params, st: AdamState, cfg: StepConfig, precision: str = "fp32",
               round_weight_grads: bool = False, theta: np.ndarray | None = None) -> StepResult:
    """One optimizer step over the microbatches in ``xs`` (the loop body
    2840-3090): forward/backward per microbatch with gradient accumulation,
    global clip, dampening, Adam, renormalisation."""
    g = None
    fws = []
    for x in xs:
        fw = forward(x, p, cfg, precision, theta)
        gb = backward(x, p, fw, cfg, precision, round_weight_grads)
        g = add_grads(g, gb)
        fws.append(fw)
    norm, clip = clip_coef(g, cfg.max_norm)
    newp = adam_step(p, g, st, cfg, clip)
    recon = sum(f.recon_loss for f in fws) * cfg.accum_steps / len(fws)
    l0 = sum(f.l0 for f in fws) / len(fws)
    return StepResult(newp, g, fws, norm, clip, recon, l0)


# --------------------------------------------------------- synthetic data
def superposition_batch(n_tokens: int, d: int, n_dirs: int, k_active: int, norm_mu: float,
                        norm_sigma: float, seed: int, noise: float = 0.05) -> np.ndarray:
    """The benchmark's synthetic activations on the CPU: each token is a sum of
    k_active distinct unit directions of a fixed Gaussian dictionary with
    Exponential(1) magnitudes, plus N(0, noise^2), rescaled to a LogNormal norm.
    (Stands in for the residual-stream activation pools; no public dataset is
    used.)"""
    rng_d = np.random.default_rng(seed)
    D = rng_d.standard_normal((n_dirs, d)).astype(np.float32)
    D /= np.linalg.norm(D, axis=1, keepdims=True)
    rng = np.random.default_rng(seed + 1)
    idx = np.argsort(rng.random((n_tokens, n_dirs)), axis=1)[:, :k_active] if n_dirs <= 4096 \
        else np.stack([rng.choice(n_dirs, k_active, replace=False) for _ in range(n_tokens)])
    coef = rng.exponential(1.0, (n_tokens, k_active)).astype(np.float32)
    x = np.einsum("tk,tkd->td", coef, D[idx])
    x += noise * rng.standard_normal(x.shape).astype(np.float32)
    norms = np.exp(norm_mu + norm_sigma * rng.standard_normal(n_tokens)).astype(np.float32)
    x *= (norms / np.maximum(np.linalg.norm(x, axis=1), 1e-8))[:, None]
    return x.astype(np.float32)


# ------------------------------------------------ dictionary-sharded step
# The reference trains one dictionary on one device. A wide SAE split over GPUs
# along the dictionary (rank r holds features [r F/N, (r+1) F/N): rows of W_enc,
# b_enc, log_threshold, columns of W_dec; x and b_dec replicated) computes the
# same step if exactly three cross-feature sums are added over the ranks: the
# decoder output and the per-token active counts (forward), the encoder term of
# the b_dec gradient (601), and the sum of squares of the global clip (3049).
# ``allreduce(a)`` is the caller's sum over ranks (identity for one rank).

def shard_params(p: Params, rank: int, world: int) -> Params:
    """Rank ``rank``'s slice of the dictionary (b_dec replicated)."""
    F = p.W_enc.shape[0]
    if F % world:
        raise ValueError("n_features must divide evenly over the ranks")
    s = slice(rank * F // world, (rank + 1) * F // world)
    return Params(p.W_enc[s].copy(), p.b_enc[s].copy(), p.W_dec[:, s].copy(), p.b_dec.copy(),
                  p.log_threshold[s].copy())


def sharded_forward(x, p: Params, cfg: StepConfig, allreduce, precision: str = "fp32",
                    theta=None) -> ForwardOut:
    """forward() over one shard: the decoder sum and counts are all-reduced
    before the bias, the residual and the loss terms."""
    B = x.shape[0]
    acc_dt = np.float64 if precision in ("fp64", "bf16") else np.float32
    if precision == "bf16":
        if theta is None:
            theta = np.exp(p.log_threshold.astype(np.float32)).astype(np.float32)
        theta = np.asarray(theta, np.float32)
        xc = bf16(x.astype(np.float32) - p.b_dec.astype(np.float32))
        pre = bf16((xc.astype(acc_dt) @ bf16(p.W_enc).astype(acc_dt).T
                    + bf16(p.b_enc).astype(acc_dt)).astype(np.float32))
        gate = (pre > theta).astype(np.float32)
        feat = pre * gate
        part = bf16(feat).astype(acc_dt) @ bf16(p.W_dec).astype(acc_dt).T
    else:
        dt = _dt(precision)
        x = x.astype(dt)
        theta = np.exp(p.log_threshold.astype(dt)) if theta is None else np.asarray(theta, dt)
        xc = x - p.b_dec.astype(dt)
        pre = xc @ p.W_enc.astype(dt).T + p.b_enc.astype(dt)
        gate = (pre > theta).astype(dt)
        feat = pre * gate
        part = feat @ p.W_dec.astype(dt).T
    exchange = np.concatenate([part.reshape(-1), gate.sum(axis=1).astype(part.dtype)])
    exchange = allreduce(exchange)
    dec = exchange[:B * x.shape[1]].reshape(B, -1)
    counts = exchange[B * x.shape[1]:]
    if precision == "bf16":
        x_hat = bf16(dec.astype(np.float32)) + p.b_dec.astype(np.float32)
        residual = x.astype(np.float32) - x_hat
    else:
        x_hat = (dec + p.b_dec.astype(dec.dtype)).astype(_dt(precision))
        residual = x - x_hat
    n = residual.size
    recon = float(np.square(residual.astype(acc_dt)).sum() / n / cfg.accum_steps)
    l0 = float(counts.astype(np.float64).mean())
    diff = l0 - cfg.target_l0
    slack = max(diff, 0.0)
    sparsity = (cfg.lambda_l0 * slack + 0.5 * cfg.al_mu * slack * slack) / cfg.accum_steps
    gate_grad = ((cfg.lambda_l0 + cfg.al_mu * slack) / cfg.accum_steps / B) if diff >= 0 else 0.0
    return ForwardOut(theta, xc, pre, gate, feat, x_hat, residual, counts, recon, l0, sparsity,
                      gate_grad, recon + sparsity)


def sharded_backward(x, p: Params, fw: ForwardOut, cfg: StepConfig, rank: int, allreduce,
                     precision: str = "fp32") -> Grads:
    """backward() over one shard. Everything but the b_dec gradient is local;
    rank 0 contributes Σ_b go, every rank its -(Σ_b dpre) W_enc term, and the
    sum over ranks is the full b_dec gradient."""
    g = backward(x, p, fw, cfg, precision)
    go = g.extras["go"]
    a = np.float64 if precision == "bf16" else _dt(precision)
    gb_go = go.astype(np.float32 if precision == "bf16" else a)
    if precision == "bf16":
        go_sum = (-(np.float32(1.0 / (cfg.accum_steps * x.shape[0] * x.shape[1]))
                    * (2.0 * fw.residual)).astype(np.float32)).astype(a).sum(axis=0)
        enc_term = -(g.b_enc.astype(a) @ bf16(p.W_enc).astype(a))
    else:
        go_sum = gb_go.sum(axis=0)
        enc_term = -(g.b_enc @ p.W_enc.astype(a))
    mine = (go_sum if rank == 0 else 0.0) + enc_term
    g.b_dec = allreduce(np.asarray(mine)).astype(g.b_dec.dtype)
    return g


def sharded_clip_coef(g: Grads, max_norm: float, rank: int, allreduce) -> tuple[float, float]:
    """clip_coef() over shards: the replicated b_dec gradient counts once."""
    tot = 0.0
    for k in PARAM_NAMES:
        v = getattr(g, k)
        if v is None or (k == "b_dec" and rank != 0):
            continue
        tot += float(np.square(v.astype(np.float64)).sum())
    tot = float(allreduce(np.array([tot]))[0])
    norm = math.sqrt(tot)
    return norm, min(1.0, max_norm / (norm + 1e-6))


def sharded_train_step(xs, p: Params, st: AdamState, cfg: StepConfig, rank: int, allreduce,
                       precision: str = "fp32", theta=None) -> StepResult:
    """train_step() of one shard; Adam and the renormalisations are local (each
    W_dec column and W_enc row lives on one rank)."""
    g = None
    fws = []
    for x in xs:
        fw = sharded_forward(x, p, cfg, allreduce, precision, theta)
        gb = sharded_backward(x, p, fw, cfg, rank, allreduce, precision)
        g = add_grads(g, gb)
        fws.append(fw)
    norm, clip = sharded_clip_coef(g, cfg.max_norm, rank, allreduce)
    newp = adam_step(p, g, st, cfg, clip)
    recon = sum(f.recon_loss for f in fws) * cfg.accum_steps / len(fws)
    l0 = sum(f.l0 for f in fws) / len(fws)
    return StepResult(newp, g, fws, norm, clip, recon, l0)
