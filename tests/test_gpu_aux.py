"""The dead-feature aux loss (sae_trainer_rolling.py:2986-2998) on the GPU
against the oracle, whose aux path is pinned to the reference's own outputs
(tests/golden/aux_*.npz).

Tolerances as in test_gpu_fused_step: bf16 operands, so the aux loss and the
gradients within 2e-2 relative (L2); the top-k selection runs on the kernel's
bf16 pre-activations, which may differ from the oracle's by one bf16 ulp, so a
value at the k-th boundary can be swapped with a neighbour."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import sae_oracle as O
from test_gpu_fused_step import BF16_TOL, _rel, build, kernel_theta, oracle_cfg, oracle_params

pytestmark = pytest.mark.gpu


def aux_cfg(g):
    cfg = oracle_cfg(g)
    cfg.aux_dead = g["dead"]
    cfg.aux_k = int(g["eff_k"])
    cfg.aux_coeff = float(g["aux_coeff"])
    return cfg


@pytest.mark.parametrize("name", ["aux_f32_tiles", "aux_f64", "aux_f64_accum2"])
@pytest.mark.parametrize("grad_feat", ["sampled", "gemm"])
def test_step_with_aux_matches_oracle(name, grad_feat):
    g = load_golden(name)
    n = int(g["n_micro"])
    xs = [g[f"x{i}"].astype(np.float32) for i in range(n)]
    x = torch.from_numpy(np.concatenate(xs)).cuda()
    sae, opt, fs = build(g, grad_feat=grad_feat)
    fs.max_tokens = x.shape[0]
    cfg = aux_cfg(g)
    dead = torch.from_numpy(g["dead"]).cuda()
    wf = float(g["wenc_factor"])
    out = fs.step(x, microbatch_tokens=xs[0].shape[0], lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu,
                  target_l0=cfg.target_l0, wenc_dampen=lambda l0: wf, aux_dead=dead,
                  aux_k=cfg.aux_k, aux_coeff=cfg.aux_coeff)
    torch.cuda.synchronize()
    from sae_b200 import _lib as L
    assert L.device_status() == 0
    p0 = oracle_params(g)
    ref = O.train_step(xs, p0, O.AdamState.zeros_like(p0), cfg, "bf16",
                       theta=kernel_theta(fs, xs[-1].shape[0]))
    aux_ref = sum(f.aux_loss for f in ref.fw)
    assert aux_ref > 0
    assert out["aux_loss"] == pytest.approx(aux_ref, rel=BF16_TOL)
    grads = {"W_enc": fs.g_W_enc, "b_enc": fs.g_b_enc, "W_dec": fs.g_W_dec_fm.t(),
             "b_dec": fs.g_b_dec, "log_threshold": fs.g_log_thr}
    for k, t in grads.items():
        err = _rel(t.cpu().numpy(), getattr(ref.grads, k))
        assert err < BF16_TOL, f"{k}: rel err {err:.3g}"
    # the aux term reaches only the dead features' encoder rows and decoder columns
    live = np.ones(sae.n_features, bool)
    live[g["dead"]] = False
    ref_plain_cfg = oracle_cfg(g)
    plain = O.train_step(xs, p0, O.AdamState.zeros_like(p0), ref_plain_cfg, "bf16",
                         theta=kernel_theta(fs, xs[-1].shape[0]))
    assert _rel(fs.g_W_enc.cpu().numpy()[live], plain.grads.W_enc[live]) < BF16_TOL
    assert _rel(fs.g_W_enc.cpu().numpy()[~live], plain.grads.W_enc[~live]) > 1e-3


def test_aux_off_again_gives_the_plain_step():
    g = load_golden("aux_f32_tiles")
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    cfg = aux_cfg(g)
    dead = torch.from_numpy(g["dead"]).cuda()
    res = []
    for use in (True, False):
        sae, opt, fs = build(g)
        if use:   # aux on for one microbatch, then off
            fs.set_aux(dead, cfg.aux_k)
            fs.microbatch(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
            fs.set_aux(None)
        st = fs.microbatch(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
        torch.cuda.synchronize()
        res.append((st["aux_loss"], fs.g_W_enc.clone(), fs.g_W_dec_fm.clone()))
    assert res[0][0] == 0.0 and res[1][0] == 0.0
    assert torch.equal(res[0][1], res[1][1]) and torch.equal(res[0][2], res[1][2])


def test_aux_rejects_bad_dead_sets():
    g = load_golden("aux_f32_tiles")
    sae, opt, fs = build(g)
    with pytest.raises(ValueError):
        fs.set_aux(torch.tensor([3, 2], device="cuda"), 1)
    with pytest.raises(ValueError):
        fs.set_aux(torch.tensor([0, sae.n_features], device="cuda"), 1)
