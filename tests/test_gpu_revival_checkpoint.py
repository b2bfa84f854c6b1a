"""The trainer's writes around the hot path, on the B200 module's feature-major
storage: revival (resample / threshold reset) mutations and checkpoint resume.

* Revival (sae_trainer_rolling.py:2796-2810, 3113-3118, 3152-3157) writes
  ``W_enc.weight.data[mask]``, ``W_dec.weight.data[:, mask]``,
  ``log_threshold.data[mask]`` and zeroes ``optimizer.state[p]["exp_avg"]``
  rows/columns; the next fused step must see the new weights (the bf16
  tensor-core copies are rebuilt) and match the oracle on them.
* Checkpoints (2255-2379): a torch.optim.Adam state_dict taken over the
  reference layout (W_dec [d, F] contiguous) loads into B200Adam, and the next
  update of both optimizers agrees (fp32 tolerance); B200 state_dicts have the
  reference keys and shapes.
"""
import io

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import sae_oracle as O
from test_gpu_fused_step import BF16_TOL, _rel, build, kernel_theta, oracle_cfg

pytestmark = pytest.mark.gpu


def test_revival_writes_reach_the_next_fused_step():
    g = load_golden("super_f32_tiles")
    sae, opt, fs = build(g)
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    fs.step(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
    torch.cuda.synchronize()
    F, d = sae.n_features, sae.d_in
    gen = torch.Generator(device="cpu").manual_seed(3)
    mask = torch.zeros(F, dtype=torch.bool)
    mask[torch.randperm(F, generator=gen)[:40]] = True
    mask = mask.cuda()
    new_rows = torch.randn(int(mask.sum()), d, generator=gen).cuda()
    new_rows /= new_rows.norm(dim=1, keepdim=True)
    with torch.no_grad():
        # resample (2796-2810): encoder rows, decoder columns, thresholds, Adam moments
        sae.W_enc.weight.data[mask] = new_rows * 0.5
        sae.W_dec.weight.data[:, mask] = new_rows.t()
        sae.log_threshold.data[mask] = float(np.log(0.9))
        for p in (sae.W_enc.weight, sae.W_enc.bias):
            opt.state[p]["exp_avg"][mask] = 0
            opt.state[p]["exp_avg_sq"][mask] = 0
        opt.state[sae.W_dec.weight]["exp_avg"][:, mask] = 0
        opt.state[sae.W_dec.weight]["exp_avg_sq"][:, mask] = 0
    assert sae.W_dec.weight.t().is_contiguous()          # still feature-major
    p1 = O.Params(sae.W_enc.weight.detach().cpu().numpy(), sae.W_enc.bias.detach().cpu().numpy(),
                  sae.W_dec.weight.detach().cpu().numpy(), sae.b_dec.detach().cpu().numpy(),
                  sae.log_threshold.detach().cpu().numpy())
    st = fs.microbatch(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
    torch.cuda.synchronize()
    # the tensor cores read the new weights
    np.testing.assert_array_equal(sae._shadow_enc.float().cpu().numpy(), O.bf16(p1.W_enc))
    np.testing.assert_array_equal(sae._shadow_dec.float().cpu().numpy(), O.bf16(p1.W_dec.T))
    fw = O.forward(g["x0"].astype(np.float32), p1, cfg, "bf16", theta=kernel_theta(fs, x.shape[0]))
    ref = O.backward(g["x0"].astype(np.float32), p1, fw, cfg, "bf16")
    assert st["l0"] == pytest.approx(fw.l0, rel=1e-2)
    for k, t in {"W_enc": fs.g_W_enc, "W_dec": fs.g_W_dec_fm.t(), "b_dec": fs.g_b_dec,
                 "log_threshold": fs.g_log_thr}.items():
        assert _rel(t.cpu().numpy(), getattr(ref, k)) < BF16_TOL, k


def test_torch_adam_checkpoint_resumes_in_b200adam():
    from sae_b200 import B200Adam, make_sae, reference_param_groups
    d, F, lr = 64, 256, 1e-3
    torch.manual_seed(0)
    ref = make_sae(d, F, seed=2)
    # the reference layout: plain parameters, W_dec [d, F] contiguous
    names = ("W_enc.weight", "W_enc.bias", "W_dec.weight", "b_dec", "log_threshold")
    plain = {k: torch.nn.Parameter(v.detach().clone().contiguous().cuda())
             for k, v in ref.state_dict().items()}
    groups = [{"params": [plain["W_enc.weight"], plain["W_enc.bias"]], "weight_decay": 0},
              {"params": [plain["W_dec.weight"]], "weight_decay": 1e-4},
              {"params": [plain["b_dec"]], "weight_decay": 0},
              {"params": [plain["log_threshold"]], "weight_decay": 0}]
    tadam = torch.optim.Adam(groups, lr=lr, betas=(0.9, 0.999))
    grads = [{k: 1e-2 * torch.randn_like(plain[k]) for k in names} for _ in range(2)]
    for k in names:
        plain[k].grad = grads[0][k].clone()
    tadam.step()
    buf = io.BytesIO()
    torch.save({"sae": {k: v.detach().cpu() for k, v in plain.items()},
                "opt": tadam.state_dict()}, buf)
    buf.seek(0)
    ck = torch.load(buf)
    # resume on the B200 module
    sae = make_sae(d, F, seed=9).cuda()
    sae.load_state_dict(ck["sae"])
    assert sae.W_dec.weight.t().is_contiguous()
    bopt = B200Adam(reference_param_groups(sae, lr), lr=lr, betas=(0.9, 0.999), sae=sae)
    bopt.load_state_dict(ck["opt"])
    assert bopt.state[sae.W_dec.weight]["exp_avg"].t().is_contiguous()
    for k, p in zip(names, (sae.W_enc.weight, sae.W_enc.bias, sae.W_dec.weight, sae.b_dec,
                            sae.log_threshold)):
        torch.testing.assert_close(bopt.state[p]["exp_avg"], tadam.state[plain[k]]["exp_avg"])
    # one more update on each, same gradients
    for k in names:
        plain[k].grad = grads[1][k].clone()
    tadam.step()
    sae.W_enc.weight.grad = grads[1]["W_enc.weight"].clone()
    sae.W_enc.bias.grad = grads[1]["W_enc.bias"].clone()
    sae.W_dec.weight.grad = grads[1]["W_dec.weight"].t().contiguous().t()
    sae.b_dec.grad = grads[1]["b_dec"].clone()
    sae.log_threshold.grad = grads[1]["log_threshold"].clone()
    bopt.step()
    torch.cuda.synchronize()
    for k, p in zip(names, (sae.W_enc.weight, sae.W_enc.bias, sae.W_dec.weight, sae.b_dec,
                            sae.log_threshold)):
        torch.testing.assert_close(p.detach(), plain[k].detach(), rtol=1e-5, atol=1e-6)
    # a B200 state_dict has the reference's keys and shapes
    sd = sae.state_dict()
    assert set(sd) == set(names)
    assert sd["W_dec.weight"].shape == (d, F) and sd["W_enc.weight"].shape == (F, d)
