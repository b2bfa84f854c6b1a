"""The reference module's API on the B200 module.

Mirrors the reference's hot-path tests (tests/test_ste_equivalence.py,
test_sparse_decode.py, test_prebias_reassociation.py, test_sae_model.py) against
``B200JumpReLUSAE``: construction and state on CPU, every computation on the
GPU (the module refuses CPU tensors). The reference runs these in float64 on
CPU; the library computes in float32 (and bf16 under autocast), so the
tolerances are float32's (stated per test) and the closed forms are evaluated
in float64 from the module's own pre-activations.
"""
import math

import numpy as np
import pytest
import torch

from conftest import load_golden

TOL32 = 2e-5


def _sae(d, F, seed=0):
    from sae_b200 import make_sae
    return make_sae(d, F, seed=seed)


# ------------------------------------------------------------------ CPU tests
def test_init_is_bit_identical_to_the_reference():
    """_make_sae draws (tests/golden/init_*.npz were written by the reference)."""
    for d, F, s in ((4, 8, 0), (16, 32, 1234), (24, 160, 3)):
        g = load_golden(f"init_d{d}_F{F}_s{s}")
        sae = _sae(d, F, s)
        np.testing.assert_array_equal(sae.W_enc.weight.detach().numpy(), g["W_enc"])
        np.testing.assert_array_equal(sae.W_enc.bias.detach().numpy(), g["b_enc"])
        np.testing.assert_array_equal(sae.W_dec.weight.detach().numpy(), g["W_dec"])
        np.testing.assert_array_equal(sae.b_dec.detach().numpy(), g["b_dec"])
        np.testing.assert_array_equal(sae.log_threshold.detach().numpy(), g["log_threshold"])


def test_shapes_keys_and_tied_unit_norm_init():
    """reference tests/test_sae_model.py: shapes, unit decoder columns, W_enc = W_dec^T, theta."""
    sae = _sae(16, 48, seed=7)
    assert sae.W_enc.weight.shape == (48, 16) and sae.W_enc.bias.shape == (48,)
    assert sae.W_dec.weight.shape == (16, 48) and sae.b_dec.shape == (16,)
    assert sae.log_threshold.shape == (48,)
    assert list(sae.state_dict()) == ["b_dec", "log_threshold", "W_enc.weight", "W_enc.bias",
                                      "W_dec.weight"]
    torch.testing.assert_close(sae.W_dec.weight.norm(dim=0), torch.ones(48), rtol=0, atol=1e-6)
    torch.testing.assert_close(sae.W_enc.weight, sae.W_dec.weight.t(), rtol=0, atol=0)
    torch.testing.assert_close(sae.log_threshold.exp(), torch.full((48,), 0.1), rtol=1e-6, atol=0)
    # decoder storage is feature-major: W_dec.weight is the [d, F] view of [F, d]
    assert sae.W_dec.weight.t().is_contiguous()


def test_seed_determinism_and_state_dict_round_trip():
    a, b = _sae(8, 24, seed=5), _sae(8, 24, seed=5)
    for k, v in a.state_dict().items():
        assert torch.equal(v, b.state_dict()[k]), k
    c = _sae(8, 24, seed=6)
    c.load_state_dict(a.state_dict())
    for k, v in a.state_dict().items():
        assert torch.equal(v, c.state_dict()[k]), k
    assert c.W_dec.weight.t().is_contiguous()


def test_module_refuses_cpu_tensors():
    sae = _sae(8, 24)
    with pytest.raises(RuntimeError, match="CUDA"):
        sae.encode_pre(torch.randn(3, 8))


def test_reference_param_groups_match_the_trainer():
    from sae_b200 import reference_param_groups
    sae = _sae(8, 24)
    groups = reference_param_groups(sae, 2e-4)
    assert [len(g["params"]) for g in groups] == [2, 1, 1, 1]
    assert [g["weight_decay"] for g in groups] == [0, 1e-4, 0, 0]
    assert groups[0]["params"][0] is sae.W_enc.weight and groups[0]["params"][1] is sae.W_enc.bias
    assert groups[1]["params"][0] is sae.W_dec.weight


# ------------------------------------------------------------------ GPU tests
def _ste_setup():
    sae = _sae(16, 32, seed=1234).cuda()
    with torch.no_grad():
        sae.log_threshold.copy_(torch.linspace(-1.5, 0.0, 32))
    sae.ste_bandwidth = 0.2
    g = torch.Generator().manual_seed(1235)
    x = torch.randn(64, 16, generator=g).cuda()
    return sae, x


C_GATE = 0.37


@pytest.mark.gpu
def test_ste_threshold_gradient_matches_closed_form():
    """reference tests/test_ste_equivalence.py:59-87, float32 on the GPU."""
    sae, x = _ste_setup()
    pre = sae.encode_pre(x)
    feat, gate = sae.jumprelu_with_gate(pre)
    loss = feat.pow(2).sum() + C_GATE * gate.sum()
    sae.zero_grad(set_to_none=True)
    loss.backward()
    got = sae.log_threshold.grad.double().cpu()

    p = pre.detach().double().cpu()
    th = sae.log_threshold.detach().exp().double().cpu()
    eps = sae.ste_bandwidth
    gate_h = (p > th).double()
    comb = p * (2.0 * p * gate_h) + C_GATE
    in_band = (p - th).abs() < eps
    expected = -(torch.where(in_band, comb, torch.zeros_like(comb)).sum(0) / (2 * eps)) * th
    assert in_band.any()
    torch.testing.assert_close(got, expected, rtol=TOL32, atol=TOL32)


@pytest.mark.gpu
def test_grad_pre_is_gated():
    sae, x = _ste_setup()
    pre = sae.encode_pre(x).detach().requires_grad_(True)
    feat, gate = sae.jumprelu_with_gate(pre)
    (feat.pow(2).sum() + C_GATE * gate.sum()).backward()
    th = sae.log_threshold.detach().exp()
    gh = (pre.detach() > th).float()
    torch.testing.assert_close(pre.grad, 2.0 * pre.detach() * gh * gh, rtol=TOL32, atol=TOL32)


@pytest.mark.gpu
def test_gate_is_the_hard_indicator_and_feat_is_pre_times_gate():
    sae, x = _ste_setup()
    pre = sae.encode_pre(x)
    feat, gate = sae.jumprelu_with_gate(pre)
    expected = (pre > sae.log_threshold.exp()).float()
    torch.testing.assert_close(gate.detach(), expected, rtol=0, atol=0)
    torch.testing.assert_close(feat.detach(), (pre * gate).detach(), rtol=0, atol=0)
    assert sae.l0_indicator(pre).detach().equal(expected)
    torch.testing.assert_close(sae.apply_jumprelu(pre).detach(), feat.detach(), rtol=0, atol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("n_accum", [1, 2, 4])
def test_threshold_gradient_accumulates_across_microbatches(n_accum):
    sae, x = _ste_setup()
    sae.zero_grad(set_to_none=True)
    for chunk in x.chunk(n_accum, dim=0):
        pre = sae.encode_pre(chunk)
        feat, gate = sae.jumprelu_with_gate(pre)
        (feat.pow(2).sum() + C_GATE * gate.sum()).backward()
    acc = sae.log_threshold.grad.clone()
    sae.zero_grad(set_to_none=True)
    pre = sae.encode_pre(x)
    feat, gate = sae.jumprelu_with_gate(pre)
    (feat.pow(2).sum() + C_GATE * gate.sum()).backward()
    torch.testing.assert_close(acc, sae.log_threshold.grad, rtol=TOL32, atol=TOL32)


@pytest.mark.gpu
def test_known_answer_gate():
    """pre = [0.05, 0.2, -1, 0.5], theta = 0.1 -> [0, 0.2, 0, 0.5] (reference test_sae_model 41-55)."""
    g = load_golden("gate_known_answer")
    sae = _sae(4, 4).cuda()
    with torch.no_grad():
        sae.log_threshold.copy_(torch.from_numpy(g["log_threshold"]))
    feat, gate = sae.jumprelu_with_gate(torch.from_numpy(g["pre"]).cuda())
    np.testing.assert_array_equal(gate.detach().cpu().numpy(), g["gate"])
    np.testing.assert_array_equal(feat.detach().cpu().numpy(), g["feat"])


def _sparse_acts(B, F, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    acts = torch.zeros(B, F)
    for b in range(B):
        idx = torch.randperm(F, generator=g)[:k]
        acts[b, idx] = torch.rand(k, generator=g) + 0.5
    return acts


@pytest.mark.gpu
def test_decode_forward_and_all_gradients():
    """reference tests/test_sparse_decode.py:45-56: x_hat and the three gradients,
    against float64 on the CPU."""
    sae = _sae(7, 64, seed=0).cuda()
    acts = _sparse_acts(9, 64, k=5).cuda().requires_grad_(True)
    out = sae.decode(acts)
    w = torch.linspace(0.3, 1.7, out.numel(), device="cuda").reshape(out.shape)
    (out * w).sum().backward()
    Wd = sae.W_dec.weight.detach().double().cpu()
    a = acts.detach().double().cpu()
    wc = w.double().cpu()
    torch.testing.assert_close(out.detach().double().cpu(), a @ Wd.t() + sae.b_dec.double().cpu().detach(),
                               rtol=TOL32, atol=TOL32)
    torch.testing.assert_close(sae.W_dec.weight.grad.double().cpu(), wc.t() @ a, rtol=TOL32, atol=TOL32)
    torch.testing.assert_close(sae.b_dec.grad.double().cpu(), wc.sum(0), rtol=TOL32, atol=TOL32)
    torch.testing.assert_close(acts.grad.double().cpu(), wc @ Wd, rtol=TOL32, atol=TOL32)
    # grad_acts is dense: inactive features still receive a gradient (test_sparse_decode 58-70)
    inactive = (a == 0)
    assert (acts.grad.cpu()[inactive].abs() > 0).any()


@pytest.mark.gpu
def test_prebias_reassociation_matches_plain_path():
    """reference tests/test_prebias_reassociation.py:37-48: the reassociated b_dec gradient equals
    plain autograd (the x.requires_grad path)."""
    sae = _sae(5, 11, seed=0).cuda()
    torch.manual_seed(0)
    x = torch.randn(7, 5).cuda()

    def grads(x_in):
        for p in (sae.W_enc.weight, sae.W_enc.bias, sae.b_dec):
            p.grad = None
        pre = sae._pre(x_in)
        w = torch.linspace(0.5, 2.0, pre.numel(), device="cuda").reshape(pre.shape)
        (pre * w).sum().backward()
        return [p.grad.clone() for p in (sae.W_enc.weight, sae.W_enc.bias, sae.b_dec)], pre.detach()

    fast, pre_fast = grads(x)
    plain, pre_plain = grads(x.clone().requires_grad_(True))
    torch.testing.assert_close(pre_fast, pre_plain, rtol=TOL32, atol=TOL32)
    for a, b in zip(fast, plain):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-5)
    for p in (sae.W_enc.weight, sae.W_enc.bias, sae.b_dec):
        assert p.grad.dtype == p.dtype


@pytest.mark.gpu
def test_cuda_autocast_bf16_prebias():
    """reference tests/test_prebias_reassociation.py:110-134: under bf16 autocast the
    reassociated path (bf16 tile GEMM) and the plain path agree; grads come back in fp32.
    Tolerance: 2e-2 relative L2 per gradient (bf16 operands)."""
    sae = _sae(64, 128, seed=5).cuda()
    x = torch.randn(32, 64, device="cuda").to(torch.bfloat16)

    def run(fast):
        for p in (sae.W_enc.weight, sae.W_enc.bias, sae.b_dec):
            p.grad = None
        xi = x if fast else x.float().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            pre = sae._pre(xi)
        assert pre.dtype == torch.bfloat16
        pre.float().pow(2).sum().backward()
        for p in (sae.W_enc.weight, sae.W_enc.bias, sae.b_dec):
            assert p.grad.dtype == torch.float32
        return [p.grad.clone().float() for p in (sae.W_enc.weight, sae.W_enc.bias, sae.b_dec)]

    for a, b in zip(run(True), run(False)):
        assert float((a - b).norm() / b.norm()) < 2e-2


@pytest.mark.gpu
def test_forward_end_to_end_and_normalize_decoder():
    sae = _sae(64, 256, seed=2).cuda()
    x = torch.randn(40, 64, device="cuda")
    x_hat, acts = sae(x)
    assert x_hat.shape == (40, 64) and acts.shape == (40, 256)
    pre = (x - sae.b_dec) @ sae.W_enc.weight.t() + sae.W_enc.bias
    ref_acts = pre * (pre > sae.log_threshold.exp())
    torch.testing.assert_close(acts.detach(), ref_acts.detach(), rtol=1e-4, atol=1e-4)
    with torch.no_grad():
        sae.W_dec.weight.mul_(3.0)
    sae._normalize_decoder()
    torch.testing.assert_close(sae.W_dec.weight.detach().norm(dim=0),
                               torch.ones(256, device="cuda"), rtol=0, atol=1e-5)
