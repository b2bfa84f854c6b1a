"""The fused optimizer pass against torch: clip, dampening, Adam and renorm.

B200Adam(renorm=True) runs, in one pass per row, what the reference loop does
after the backward (sae_trainer_rolling.py:3049-3090): clip_grad_norm_(1.0)
(here from sae_b200_grad_norm, applied through the StepStats), the W_enc
gradient dampening factor, torch.optim.Adam over the trainer's four groups
(L2 decay 1e-4 on W_dec, 2536-2541), then the decoder-column renormalisation
(_normalize_decoder, 778-782) and the W_enc row renormalisation (3089-3090).
The reference here is exactly that torch sequence on the reference layout
(W_dec.weight [d, F] contiguous), on the GPU in fp32. Both sides compute in
fp32 with the same operation order up to the order of the two gradient
scalings and the summation order of the clip norm (1e-5 relative), so the
parameters agree to 1e-5 relative after one and three steps and the second
moments, which square the clipped gradient, to 3e-5.
Both row widths are covered: d=64 (one warp per row) and d=1536 (the wide-row
kernel of the benchmark shape).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

NAMES = ("W_enc.weight", "W_enc.bias", "W_dec.weight", "b_dec", "log_threshold")


def _reference_renorm(plain):
    with torch.no_grad():
        w = plain["W_dec.weight"]
        w.div_(w.norm(dim=0, keepdim=True).clamp(min=1e-8))          # 778-782
        e = plain["W_enc.weight"]
        e.div_(e.norm(dim=1, keepdim=True).clamp(min=1e-8))          # 3089-3090


@pytest.mark.parametrize("d,F", [(64, 256), (1536, 512)])
@pytest.mark.parametrize("clip", [False, True])
def test_fused_adam_renorm_matches_torch(d, F, clip):
    import sae_b200
    lr = 1e-3
    sae = sae_b200.make_sae(d, F, seed=4).cuda()
    plain = {k: torch.nn.Parameter(v.detach().clone().contiguous())
             for k, v in sae.state_dict().items()}
    groups = [{"params": [plain["W_enc.weight"], plain["W_enc.bias"]], "weight_decay": 0},
              {"params": [plain["W_dec.weight"]], "weight_decay": 1e-4},
              {"params": [plain["b_dec"]], "weight_decay": 0},
              {"params": [plain["log_threshold"]], "weight_decay": 0}]
    tadam = torch.optim.Adam(groups, lr=lr, betas=(0.9, 0.999))
    bopt = sae_b200.B200Adam(sae_b200.reference_param_groups(sae, lr), lr=lr,
                             betas=(0.9, 0.999), sae=sae, renorm=True)
    fs = sae_b200.FusedStep(sae, bopt, max_tokens=256)
    gen = torch.Generator(device="cuda").manual_seed(d + F)
    scale = 0.1 if clip else 1e-3          # total norm ~10 (clipped) or ~0.1 (not)
    factors = (1.0, 0.7, 1.0)              # the W_enc dampening on the second step
    for step, factor in enumerate(factors, start=1):
        g = {k: scale * torch.randn(plain[k].shape, device="cuda", generator=gen) for k in NAMES}
        # reference loop: clip_grad_norm_, dampening, Adam, renorms
        for k in NAMES:
            plain[k].grad = g[k].clone()
        norm_ref = torch.nn.utils.clip_grad_norm_([plain[k] for k in NAMES], 1.0) if clip \
            else None
        if factor < 1.0:
            plain["W_enc.weight"].grad.mul_(factor)
            plain["W_enc.bias"].grad.mul_(factor)
        tadam.step()
        _reference_renorm(plain)
        # library: gradients in the FusedStep buffers (W_dec feature-major)
        fs.g_W_enc.copy_(g["W_enc.weight"])
        fs.g_b_enc.copy_(g["W_enc.bias"])
        fs.g_W_dec_fm.copy_(g["W_dec.weight"].t())
        fs.g_b_dec.copy_(g["b_dec"])
        fs.g_log_thr.copy_(g["log_threshold"])
        fs._bind_grads()
        if clip:
            fs.grad_norm(1.0)
            bopt.step(stats=fs.stats, grad_scale_enc=factor)
            st = fs.read_stats()
            assert st["grad_norm"] == pytest.approx(float(norm_ref), rel=1e-5)
            assert st["clip_coef"] < 1.0
        else:
            bopt.step(grad_scale_enc=factor)
        torch.cuda.synchronize()
        if step in (1, 3):
            for k, p in zip(NAMES, (sae.W_enc.weight, sae.W_enc.bias, sae.W_dec.weight,
                                    sae.b_dec, sae.log_threshold)):
                torch.testing.assert_close(p.detach(), plain[k].detach(), rtol=1e-5, atol=1e-6,
                                           msg=lambda m, k=k: f"{k} after step {step}: {m}")
            for k, p in zip(("W_enc.weight", "W_dec.weight"),
                            (sae.W_enc.weight, sae.W_dec.weight)):
                st_b = bopt.state[p]
                st_t = tadam.state[plain[k]]
                torch.testing.assert_close(st_b["exp_avg"], st_t["exp_avg"], rtol=2e-5, atol=1e-8)
                # the two clip coefficients come from fp32 sums of squares taken in
                # different orders (they agree to 1e-5 relative, asserted above):
                # exp_avg_sq holds the clipped gradient squared, so twice that
                torch.testing.assert_close(st_b["exp_avg_sq"], st_t["exp_avg_sq"], rtol=3e-5,
                                           atol=1e-12)
            # the bf16 tensor-core copies are the rounded fp32 masters
            assert torch.equal(sae._shadow_enc, sae.W_enc.weight.detach().to(torch.bfloat16))
            assert torch.equal(sae._shadow_dec,
                               sae.W_dec.weight.detach().t().to(torch.bfloat16))
