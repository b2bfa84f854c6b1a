"""Generate the golden fixtures that pin the CPU oracle to the reference.

Runs the reference trainer's own SAE module and step sequence
(sae_trainer_rolling.py: _make_sae 961-966, encode_pre/jumprelu_with_gate/
decode 903-950, the loss lines 2954-2974, loss.backward(), clip_grad_norm_
3049, the 4-group torch.optim.Adam 2536-2541 and the renormalisations
3086-3090) on CPU and stores inputs and outputs as .npz files beside this
script. It needs the reference checkout, named by $SAE_REFERENCE_DIR, and is
run by hand:

    SAE_REFERENCE_DIR=<reference checkout> python tests/golden/make_golden.py

The fixtures are committed; nothing at test time imports the reference.
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get("SAE_REFERENCE_DIR"):
    sys.exit("set SAE_REFERENCE_DIR to a checkout of the reference trainer "
             "(the directory holding sae_trainer_rolling.py)")
REF = Path(os.environ["SAE_REFERENCE_DIR"])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(HERE.parents[1]))

import sae_trainer_rolling as T  # noqa: E402

from oracle.sae_oracle import superposition_batch  # noqa: E402

PNAMES = ("W_enc", "b_enc", "W_dec", "b_dec", "log_threshold")


def ref_params(sae):
    return {"W_enc": sae.W_enc.weight, "b_enc": sae.W_enc.bias, "W_dec": sae.W_dec.weight,
            "b_dec": sae.b_dec, "log_threshold": sae.log_threshold}


def run_reference_step(sae, xs, *, lam, mu, target, lr, wenc_factor=1.0, dead=None, eff_k=0):
    """The trainer's loop body on CPU (no autocast), microbatches ``xs``; with
    ``dead`` (sorted feature ids) and ``eff_k``, the dead-feature aux loss of
    sae_trainer_rolling.py:2986-2998 is added to each microbatch's loss."""
    optimizer = torch.optim.Adam(
        [{"params": sae.W_enc.parameters(), "weight_decay": 0},
         {"params": sae.W_dec.parameters(), "weight_decay": 1e-4},
         {"params": [sae.b_dec], "weight_decay": 0},
         {"params": [sae.log_threshold], "weight_decay": 0}],
        lr=lr, betas=(0.9, 0.999))
    accum = len(xs)
    optimizer.zero_grad()
    out = {"recon": [], "l0": [], "sparsity": [], "pre": [], "gate": [], "x_hat": [], "aux": []}
    for acts_mb in xs:
        pre = sae.encode_pre(acts_mb)
        feat_acts, gate = sae.jumprelu_with_gate(pre)
        gate_counts = gate.sum(dim=-1, dtype=pre.dtype)
        x_hat = sae.decode(feat_acts, active_max=None)
        residual = acts_mb - x_hat
        recon_loss = residual.pow(2).mean() / accum
        l0_mb = gate_counts.mean()
        slack = (l0_mb - target).clamp(min=0.0)
        sparsity_loss = (lam * slack + 0.5 * mu * slack * slack) / accum
        loss = recon_loss + sparsity_loss
        if dead is not None:
            dead_t = torch.as_tensor(dead, dtype=torch.long)
            pre_dead = pre[:, dead_t].relu()
            topk_vals, topk_idx = pre_dead.topk(eff_k, dim=-1)
            aux_acts = torch.zeros_like(pre_dead)
            aux_acts.scatter_(-1, topk_idx, topk_vals)
            w_dec_dead = sae.W_dec.weight.t()[dead_t]
            x_aux = aux_acts @ w_dec_dead
            aux_loss = ((residual.detach() - x_aux).pow(2).mean() * T.AUX_COEFF) / accum
            loss = loss + aux_loss
            out["aux"].append(float(aux_loss))
        loss.backward()
        out["recon"].append(float(recon_loss))
        out["l0"].append(float(l0_mb))
        out["sparsity"].append(float(sparsity_loss))
        out["pre"].append(pre.detach().numpy())
        out["gate"].append(gate.detach().numpy())
        out["x_hat"].append(x_hat.detach().numpy())
    grads = {k: v.grad.detach().clone().numpy() for k, v in ref_params(sae).items()}
    grad_norm = float(torch.nn.utils.clip_grad_norm_(sae.parameters(), 1.0))
    if wenc_factor < 1.0:
        sae.W_enc.weight.grad.mul_(wenc_factor)
        sae.W_enc.bias.grad.mul_(wenc_factor)
    optimizer.step()
    sae._normalize_decoder()
    with torch.no_grad():
        enc_norms = sae.W_enc.weight.norm(dim=1, keepdim=True).clamp(min=1e-8)
        sae.W_enc.weight.div_(enc_norms)
    after = {k: v.detach().clone().numpy() for k, v in ref_params(sae).items()}
    return out, grads, grad_norm, after


def make_case(name, *, d, F, xs, dtype, lam, mu, target, eps, lr, log_thr=None, b_dec=None,
              wenc_factor=1.0, seed=0, keep_dense=True, dead=None, eff_k=0):
    sae = T._make_sae(d, F, seed=seed).to(dtype)
    sae.ste_bandwidth = eps
    with torch.no_grad():
        if log_thr is not None:
            sae.log_threshold.copy_(torch.as_tensor(log_thr, dtype=dtype))
        if b_dec is not None:
            sae.b_dec.copy_(torch.as_tensor(b_dec, dtype=dtype))
    before = {k: v.detach().clone().numpy() for k, v in ref_params(sae).items()}
    xs_t = [torch.as_tensor(x, dtype=dtype) for x in xs]
    out, grads, gn, after = run_reference_step(sae, xs_t, lam=lam, mu=mu, target=target, lr=lr,
                                               wenc_factor=wenc_factor, dead=dead, eff_k=eff_k)
    rec = {"d": d, "F": F, "lam": lam, "mu": mu, "target": target, "eps": eps, "lr": lr,
           "wenc_factor": wenc_factor, "n_micro": len(xs), "grad_norm": gn,
           "recon": np.array(out["recon"]), "l0": np.array(out["l0"]),
           "sparsity": np.array(out["sparsity"])}
    if dead is not None:
        rec.update(dead=np.asarray(dead, np.int64), eff_k=eff_k, aux=np.array(out["aux"]),
                   aux_coeff=T.AUX_COEFF)
    if keep_dense:
        for i, x in enumerate(xs):
            rec[f"x{i}"] = np.asarray(x)
            rec[f"pre{i}"] = out["pre"][i]
            rec[f"x_hat{i}"] = out["x_hat"][i]
        for k in PNAMES:
            rec[f"p0_{k}"] = before[k]
            rec[f"grad_{k}"] = grads[k]
            rec[f"p1_{k}"] = after[k]
    else:
        # Large case: the inputs are regenerated from their seeds by the test
        # (checksums pin them); matrices are kept as checksums plus a fixed
        # sample of feature rows, vectors in full.
        rows = np.sort(np.random.default_rng(0).choice(F, 64, replace=False))
        rec["rows"] = rows
        rec["x_sum"] = np.float64(np.asarray(xs[0], np.float64).sum())
        rec["x_sumsq"] = np.float64(np.square(np.asarray(xs[0], np.float64)).sum())
        for tag, src in (("p0", before), ("grad", grads), ("p1", after)):
            for k in PNAMES:
                a = np.asarray(src[k])
                rec[f"{tag}_{k}_sum"] = np.float64(a.astype(np.float64).sum())
                rec[f"{tag}_{k}_sumsq"] = np.float64(np.square(a.astype(np.float64)).sum())
                if a.ndim == 1:
                    rec[f"{tag}_{k}"] = a
                elif k == "W_dec":
                    rec[f"{tag}_{k}_rows"] = a[:, rows].T.copy()
                else:
                    rec[f"{tag}_{k}_rows"] = a[rows].copy()
    np.savez_compressed(HERE / f"{name}.npz", **rec)
    print(f"{name}: l0={rec['l0']} recon={rec['recon']} grad_norm={gn:.6g}")


def main():
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    # 1. float64, the STE-equivalence shape (tests/test_ste_equivalence.py:33-45):
    #    thresholds spread over linspace(-1.5, 0) so many pre-activations are in band.
    g = torch.Generator().manual_seed(1235)
    x = torch.randn(64, 16, generator=g, dtype=torch.float64).numpy()
    make_case("ste_f64", d=16, F=32, xs=[x], dtype=torch.float64, lam=0.37, mu=0.05, target=4.0,
              eps=0.2, lr=1e-3, log_thr=np.linspace(-1.5, 0.0, 32), seed=1234)
    # 2. same inputs split into 2 and 4 microbatches (gradient accumulation).
    for n in (2, 4):
        make_case(f"ste_f64_accum{n}", d=16, F=32, xs=list(np.split(x, n)), dtype=torch.float64,
                  lam=0.37, mu=0.05, target=4.0, eps=0.2, lr=1e-3,
                  log_thr=np.linspace(-1.5, 0.0, 32), seed=1234)
    # 3. small superposition batch in float32, odd sizes, dampened W_enc.
    xs = superposition_batch(96, 24, 160, 6, math.log(4.0), 0.3, seed=7)
    make_case("super_f32_odd", d=24, F=160, xs=[xs], dtype=torch.float32, lam=1e-3, mu=1e-2,
              target=6.0, eps=0.2, lr=1e-4, log_thr=np.full(160, math.log(0.05)),
              b_dec=xs.mean(0), wenc_factor=0.8, seed=3)
    # 4. tile-aligned shape (d % 64 == 0, F % 128 == 0) in float32, sparse regime.
    xs = superposition_batch(256, 128, 512, 8, math.log(8.0), 0.3, seed=11)
    make_case("super_f32_tiles", d=128, F=512, xs=[xs], dtype=torch.float32, lam=1e-3, mu=1e-2,
              target=8.0, eps=0.2, lr=1e-4, log_thr=np.full(512, math.log(1.2)),
              b_dec=xs.mean(0), seed=0)
    # 5. the CPU-runnable benchmark configuration (d=256, F=8192, B=4096, K=50,
    #    log_threshold = log 0.05, b_dec = mean(x)); dense tensors not stored.
    xs = superposition_batch(4096, 256, 8192, 50, math.log(16.0), 0.3, seed=0)
    make_case("cfg1_f32", d=256, F=8192, xs=[xs], dtype=torch.float32, lam=1e-3, mu=1e-2,
              target=50.0, eps=0.2, lr=1e-4, log_thr=np.full(8192, math.log(0.05)),
              b_dec=xs.mean(0), seed=0, keep_dense=False)
    # 6. dead-feature aux loss (2986-2998): float64 and a tile-aligned float32 case,
    #    a sorted dead set with both positive and negative pre-activations.
    g = torch.Generator().manual_seed(77)
    x = torch.randn(64, 16, generator=g, dtype=torch.float64).numpy()
    dead = np.sort(np.random.default_rng(5).choice(32, 13, replace=False))
    make_case("aux_f64", d=16, F=32, xs=[x], dtype=torch.float64, lam=0.37, mu=0.05, target=4.0,
              eps=0.2, lr=1e-3, log_thr=np.linspace(-1.5, 0.0, 32), seed=1234, dead=dead,
              eff_k=4)
    make_case("aux_f64_accum2", d=16, F=32, xs=list(np.split(x, 2)), dtype=torch.float64,
              lam=0.37, mu=0.05, target=4.0, eps=0.2, lr=1e-3,
              log_thr=np.linspace(-1.5, 0.0, 32), seed=1234, dead=dead, eff_k=4)
    xs = superposition_batch(256, 128, 512, 8, math.log(8.0), 0.3, seed=13)
    dead = np.sort(np.random.default_rng(6).choice(512, 160, replace=False))
    make_case("aux_f32_tiles", d=128, F=512, xs=[xs], dtype=torch.float32, lam=1e-3, mu=1e-2,
              target=8.0, eps=0.2, lr=1e-4, log_thr=np.full(512, math.log(1.2)),
              b_dec=xs.mean(0), seed=0, dead=dead, eff_k=25)
    # 7. known-answer gate (tests/test_sae_model.py:41-55).
    sae = T._make_sae(4, 4, seed=0)
    with torch.no_grad():
        sae.log_threshold.fill_(math.log(0.1))
    pre = torch.tensor([[0.05, 0.2, -1.0, 0.5]])
    feat, gate = sae.jumprelu_with_gate(pre)
    np.savez_compressed(HERE / "gate_known_answer.npz", pre=pre.numpy(),
                        log_threshold=sae.log_threshold.detach().numpy(),
                        feat=feat.detach().numpy(), gate=gate.detach().numpy())
    # 8. reference init, bit for bit (_make_sae seeds, nn.Linear draws, orthogonal_).
    for (d, F, s) in ((4, 8, 0), (16, 32, 1234), (24, 160, 3)):
        sae = T._make_sae(d, F, seed=s)
        np.savez_compressed(HERE / f"init_d{d}_F{F}_s{s}.npz",
                            **{k: v.detach().numpy() for k, v in ref_params(sae).items()})
    print("done")


if __name__ == "__main__":
    main()
