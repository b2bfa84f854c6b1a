"""The reference loop body driven through the module API, against FusedStep.

A trainer that only swaps the SAE class (sae_b200.install) runs its own loop
body unchanged (sae_trainer_rolling.py:2914-3090): under bf16 autocast,
``encode_pre`` -> ``jumprelu_with_gate`` -> ``gate.sum(-1)`` -> ``decode`` ->
recon + sparsity loss -> ``loss.backward()`` over the microbatches, then
``clip_grad_norm_(sae.parameters(), 1.0)``, the W_enc gradient dampening,
``optimizer.step()``, ``_normalize_decoder()`` and the W_enc row renorm. Every
piece of that is a library call here (the dense products on the tcgen05 tile
GEMM). The same steps through the fused path (FusedStep, one call sequence
per microbatch) must train the same way: per-step L0 and reconstruction loss
within 1e-3, gradient norm within 2e-3, and after three steps the parameter
updates within the bf16 tolerance of Adam's sign-like first steps (the two
paths sum in different orders, and a tiny gradient of the opposite sign
flips an element's update).
"""
import copy
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

D, F, MB, ACCUM, K = 256, 2048, 1024, 2, 16
LAMBDA, MU, LR, WENC = 1e-3, 1e-2, 1e-3, 0.8


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp(min=1e-30))


@pytest.fixture(scope="module")
def runs():
    import sae_b200
    dev = torch.device("cuda")
    batches = [sae_b200.superposition_batch(MB * ACCUM, D, F, K, math.log(8.0), 0.3,
                                            seed=40 + s, device=dev) for s in range(3)]
    sae = sae_b200.make_sae(D, F, seed=1).to(dev)
    sae.ste_bandwidth = 0.2
    with torch.no_grad():
        sae.b_dec.copy_(batches[0].float().mean(0))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            pre = sae.encode_pre(batches[0][:MB])
        q = torch.quantile(pre.float().flatten()[:1_000_000], 1 - K / F).item()
        sae.log_threshold.fill_(math.log(q))
    p0 = {k: v.detach().clone() for k, v in sae.state_dict().items()}
    fused = copy.deepcopy(sae)

    # --- the reference loop body on the module API
    opt = sae_b200.B200Adam(sae_b200.reference_param_groups(sae, LR), lr=LR, sae=sae)
    loop = []
    for x in batches:
        opt.zero_grad(set_to_none=True)
        recon_t, l0_t = 0.0, 0.0
        for i in range(ACCUM):
            acts_mb = x[i * MB:(i + 1) * MB]
            with torch.autocast("cuda", dtype=torch.bfloat16):
                pre = sae.encode_pre(acts_mb)
                feat_acts, gate = sae.jumprelu_with_gate(pre)
                gate_counts = gate.sum(dim=-1, dtype=torch.float32)
                x_hat = sae.decode(feat_acts, active_max=None)
                residual_float = acts_mb.float() - x_hat.float()
                recon_loss = residual_float.pow(2).mean() / ACCUM
                l0_mb = gate_counts.mean()
                slack = (l0_mb - K).clamp(min=0.0)
                sparsity_loss = (LAMBDA * slack + 0.5 * MU * slack * slack) / ACCUM
                loss = recon_loss + sparsity_loss
            loss.backward()
            recon_t += float(recon_loss) * ACCUM
            l0_t += float(l0_mb)
        grad_norm = float(torch.nn.utils.clip_grad_norm_(sae.parameters(), 1.0))
        sae.W_enc.weight.grad.mul_(WENC)
        sae.W_enc.bias.grad.mul_(WENC)
        opt.step()
        sae._normalize_decoder()
        with torch.no_grad():
            sae.W_enc.weight.div_(sae.W_enc.weight.norm(dim=1, keepdim=True).clamp(min=1e-8))
        loop.append({"recon_loss": recon_t / ACCUM, "l0": l0_t / ACCUM, "grad_norm": grad_norm})
    torch.cuda.synchronize()

    # --- the fused path
    fopt = sae_b200.B200Adam(sae_b200.reference_param_groups(fused, LR), lr=LR, sae=fused,
                             renorm=True)
    fs = sae_b200.FusedStep(fused, fopt, max_tokens=MB)
    fsteps = [fs.step(x, microbatch_tokens=MB, lambda_l0=LAMBDA, al_mu=MU, target_l0=K,
                      wenc_dampen=lambda l0: WENC) for x in batches]
    torch.cuda.synchronize()
    return dict(p0=p0, module=sae.state_dict(), fused=fused.state_dict(), loop=loop,
                fsteps=fsteps)


def test_per_step_statistics_agree(runs):
    for a, b in zip(runs["loop"], runs["fsteps"]):
        assert a["l0"] > 1
        assert a["l0"] == pytest.approx(b["l0"], rel=1e-3)
        assert a["recon_loss"] == pytest.approx(b["recon_loss"], rel=1e-3)
        assert a["grad_norm"] == pytest.approx(b["grad_norm"], rel=2e-3)


def test_parameters_train_the_same_way(runs):
    p0, m, f = runs["p0"], runs["module"], runs["fused"]
    assert set(m) == set(f) == set(p0)
    for k in p0:
        assert _rel(m[k], f[k]) < 1e-2, k                  # the parameters themselves
        dm, df = m[k] - p0[k], f[k] - p0[k]
        if df.norm() > 0:
            assert _rel(dm, df) < 0.15, k                    # and their three-step updates
    with torch.no_grad():
        for sd in (m, f):
            torch.testing.assert_close(sd["W_dec.weight"].norm(dim=0),
                                       torch.ones(F, device="cuda"), rtol=0, atol=1e-5)
