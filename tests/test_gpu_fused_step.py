"""Parity of the fused CUDA training step against the CPU oracle.

Inputs and initial parameters are the reference's own (tests/golden). The
oracle runs in its "bf16" precision, i.e. with the reference's CUDA autocast
rounding points and float64 accumulation. Tolerances:
  * thresholds: bit-identical to torch's CUDA exp (the reference's GPU path)
    and within one float32 ulp of numpy's exp; the oracle is then given the
    kernel's thresholds, since bf16 pre-activations lie on a grid and a
    one-ulp threshold change moves grid points across the gate / STE band;
  * active sets: bit-exact against the kernel's own pre-activations and
    thresholds (gate == pre > theta, mask bits == gate, counts == popcount);
    against the oracle, differences only where pre sits within one bf16 ulp
    of theta;
  * pre: <= 1 bf16 ulp; x_hat, loss, gradients: relative L2 error < 2e-2
    (bf16 operands, different fp32 accumulation order);
  * Adam + renorm: parameters within 2.5 * lr elementwise (one Adam step moves
    an element by at most ~lr; a gradient sign flip on a near-zero gradient
    moves it by 2 lr).
"""
import math

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import sae_oracle as O

pytestmark = pytest.mark.gpu

BF16_TOL = 2e-2


def _rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def build(g, *, force_simt=False, csr_capacity=None, renorm=True, grad_feat="sampled",
          pre_store="entries"):
    from sae_b200 import B200Adam, B200JumpReLUSAE, FusedStep, reference_param_groups
    d, F = int(g["d"]), int(g["F"])
    sae = B200JumpReLUSAE(d, F)
    with torch.no_grad():
        sae.W_enc.weight.copy_(torch.from_numpy(g["p0_W_enc"]).float())
        sae.W_enc.bias.copy_(torch.from_numpy(g["p0_b_enc"]).float())
        sae.W_dec.weight.copy_(torch.from_numpy(g["p0_W_dec"]).float())
        sae.b_dec.copy_(torch.from_numpy(g["p0_b_dec"]).float())
        sae.log_threshold.copy_(torch.from_numpy(g["p0_log_threshold"]).float())
    sae = sae.cuda()
    sae.ste_bandwidth = float(g["eps"])
    opt = B200Adam(reference_param_groups(sae, float(g["lr"])), lr=float(g["lr"]),
                   betas=(0.9, 0.999), sae=sae, renorm=renorm)
    n = int(g["n_micro"])
    B = g["x0"].shape[0]
    fs = FusedStep(sae, opt, max_tokens=B, csr_capacity=csr_capacity, force_simt=force_simt,
                   grad_feat=grad_feat, pre_store=pre_store)
    return sae, opt, fs


def oracle_params(g):
    return O.Params(*(g[f"p0_{k}"].astype(np.float32) for k in O.PARAM_NAMES))


def oracle_cfg(g):
    lr = float(g["lr"])
    return O.StepConfig(lambda_l0=float(g["lam"]), al_mu=float(g["mu"]),
                        target_l0=float(g["target"]), ste_bandwidth=float(g["eps"]),
                        accum_steps=int(g["n_micro"]), lr=(lr,) * 4,
                        wenc_factor=float(g["wenc_factor"]))


def workspace_views(fs, n_tokens):
    from sae_b200 import _lib as L
    sae = fs.sae
    d, F = sae.d_in, sae.n_features
    off = L.workspace_offsets(n_tokens, d, F, fs.csr_capacity)
    W = (F + 31) // 32
    ldp = L.pre_pitch(n_tokens)

    def view(name, dtype, count):
        o = off[name]
        nbytes = count * torch.tensor([], dtype=dtype).element_size()
        return fs.ws[o:o + nbytes].view(dtype)

    return {
        "theta": view("theta", torch.float32, F),
        "xc": view("xc", torch.bfloat16, n_tokens * d).view(n_tokens, d),
        # feature-major [F, ldp]; returned as the [B, F] view
        "pre": view("pre", torch.bfloat16, F * ldp).view(F, ldp)[:, :n_tokens].t(),
        "mask": view("mask", torch.int32, n_tokens * W).view(n_tokens, W),
        "go": view("go", torch.bfloat16, n_tokens * d).view(n_tokens, d),
        "tok_cnt": view("tok_cnt", torch.int32, n_tokens),
        "col_offs": view("col_offs", torch.int32, F + 1),
    }


def kernel_theta(fs, n_tokens):
    """The thresholds the kernels used in the last forward (theta of the
    parameters before the optimizer step)."""
    return workspace_views(fs, n_tokens)["theta"].cpu().numpy().copy()


def unpack_mask(mask, F):
    m = mask.cpu().numpy().view(np.uint32)
    bits = ((m[:, :, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(m.shape[0], -1)
    return bits[:, :F].astype(bool)


CASES = [
    ("super_f32_tiles", False),   # d % 64 == 0, F % 128 == 0: tcgen05 tile GEMMs
    ("super_f32_tiles", True),    # same shape through the CUDA-core tile GEMM
    ("super_f32_odd", False),     # F = 160: CUDA-core tile GEMM with ragged tiles
    ("ste_f64", False),           # in-band-heavy STE shape (d=16, F=32)
]


@pytest.mark.parametrize("name,force_simt", CASES)
def test_forward_matches_oracle_and_active_set_is_exact(name, force_simt):
    g = load_golden(name)
    sae, opt, fs = build(g, force_simt=force_simt, pre_store="full")
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    cfg = oracle_cfg(g)
    st = fs.microbatch(x, accum_steps=1, first=True, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu,
                       target_l0=cfg.target_l0)
    torch.cuda.synchronize()
    from sae_b200 import _lib as L
    assert L.device_status() == 0
    B, F = x.shape[0], sae.n_features
    v = workspace_views(fs, B)
    pre = v["pre"].float().cpu().numpy()
    theta = v["theta"].cpu().numpy()
    # thresholds: torch's CUDA exp bit for bit; numpy's exp within one ulp
    lt = torch.from_numpy(g["p0_log_threshold"].astype(np.float32)).cuda()
    np.testing.assert_array_equal(theta, lt.exp().cpu().numpy())
    np.testing.assert_allclose(theta, np.exp(g["p0_log_threshold"].astype(np.float32)),
                               rtol=2.5e-7)
    # active set, bit-exact given the kernel's pre and theta
    gate = pre > theta
    bits = unpack_mask(v["mask"], F)
    np.testing.assert_array_equal(bits, gate)
    np.testing.assert_array_equal(v["tok_cnt"].cpu().numpy(), gate.sum(1))
    assert st["nnz"] == int(gate.sum())
    # the sampled backward's CSR: active entries plus the inactive ones in the STE band
    eps = np.float32(g["eps"])
    band = (np.abs(pre - theta) < eps) & ~gate
    assert st["csr_pairs"] == int(gate.sum() + band.sum())
    assert int(v["col_offs"][-1]) == st["csr_pairs"]
    # against the oracle
    fw = O.forward(g["x0"], oracle_params(g), cfg, "bf16", theta=theta)
    ulp = np.abs(fw.pre) * 2.0 ** -7 + 1e-30
    assert np.all(np.abs(pre - fw.pre) <= ulp * 1.01)
    flip = gate != (fw.pre > fw.theta)
    near = np.abs(fw.pre - fw.theta) <= np.abs(fw.theta) * 2.0 ** -7 + 1e-6
    assert not np.any(flip & ~near), "gate differs away from the threshold"
    assert st["l0"] == pytest.approx(float(gate.sum(1).mean()), rel=1e-6)
    assert st["recon_loss"] == pytest.approx(fw.recon_loss, rel=BF16_TOL)
    assert fs.fired_mask.cpu().numpy().tolist() == gate.any(0).tolist()


@pytest.mark.parametrize("grad_feat", ["sampled", "gemm"])
@pytest.mark.parametrize("name,force_simt", CASES)
def test_full_step_matches_oracle(name, force_simt, grad_feat):
    g = load_golden(name)
    sae, opt, fs = build(g, force_simt=force_simt, grad_feat=grad_feat)
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    wf = float(g["wenc_factor"])
    out = fs.step(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0,
                  wenc_dampen=(lambda l0: wf))
    torch.cuda.synchronize()
    p0 = oracle_params(g)
    ref = O.train_step([g["x0"].astype(np.float32)], p0, O.AdamState.zeros_like(p0), cfg, "bf16",
                       theta=kernel_theta(fs, x.shape[0]))
    grads = {"W_enc": fs.g_W_enc, "b_enc": fs.g_b_enc, "W_dec": fs.g_W_dec_fm.t(),
             "b_dec": fs.g_b_dec, "log_threshold": fs.g_log_thr}
    for k, t in grads.items():
        err = _rel(t.cpu().numpy(), getattr(ref.grads, k))
        assert err < BF16_TOL, f"{k}: rel err {err:.3g}"
    assert out["grad_norm"] == pytest.approx(ref.grad_norm, rel=BF16_TOL)
    lr = float(g["lr"])
    now = {"W_enc": sae.W_enc.weight, "b_enc": sae.W_enc.bias, "W_dec": sae.W_dec.weight,
           "b_dec": sae.b_dec, "log_threshold": sae.log_threshold}
    for k, t in now.items():
        diff = np.abs(t.detach().cpu().numpy() - getattr(ref.params, k))
        assert diff.max() <= 2.5 * lr + 1e-6, f"{k}: max |diff| {diff.max():.3g}"
    # the bf16 copies the next step reads are the updated weights
    np.testing.assert_array_equal(sae._shadow_enc.float().cpu().numpy(),
                                  O.bf16(sae.W_enc.weight.detach().cpu().numpy()))
    np.testing.assert_array_equal(sae._shadow_dec.float().cpu().numpy(),
                                  O.bf16(sae.W_dec.weight.detach().t().cpu().numpy()))
    # unit decoder columns / encoder rows after the fused renormalisation
    np.testing.assert_allclose(sae.W_dec.weight.detach().norm(dim=0).cpu().numpy(), 1.0, atol=1e-5)
    np.testing.assert_allclose(sae.W_enc.weight.detach().norm(dim=1).cpu().numpy(), 1.0, atol=1e-5)


@pytest.mark.parametrize("grad_feat", ["sampled", "gemm"])
@pytest.mark.parametrize("n", [2, 4])
def test_microbatch_accumulation_matches_oracle(n, grad_feat):
    g = load_golden(f"ste_f64_accum{n}")
    sae, opt, fs = build(g, grad_feat=grad_feat)
    cfg = oracle_cfg(g)
    xs = [g[f"x{i}"].astype(np.float32) for i in range(n)]
    x = torch.from_numpy(np.concatenate(xs)).cuda()
    fs.max_tokens = x.shape[0]
    out = fs.step(x, microbatch_tokens=xs[0].shape[0], lambda_l0=cfg.lambda_l0,
                  al_mu=cfg.al_mu, target_l0=cfg.target_l0)
    p0 = oracle_params(g)
    ref = O.train_step(xs, p0, O.AdamState.zeros_like(p0), cfg, "bf16",
                       theta=kernel_theta(fs, xs[-1].shape[0]))
    for k, t in {"W_enc": fs.g_W_enc, "log_threshold": fs.g_log_thr, "b_dec": fs.g_b_dec,
                 "W_dec": fs.g_W_dec_fm.t(), "b_enc": fs.g_b_enc}.items():
        assert _rel(t.cpu().numpy(), getattr(ref.grads, k)) < BF16_TOL, k
    assert out["l0"] == pytest.approx(ref.l0, rel=1e-2)


def test_dense_fallback_matches_sparse_path():
    """An active set larger than the workspace's CSR capacity takes the dense
    weight-gradient path (tcgen05 weight-gradient GEMMs, or CUDA cores with
    force_simt); the result must match the sampled and the GEMM sparse paths."""
    g = load_golden("super_f32_tiles")
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    res = []
    for cap, mode, simt in ((None, "sampled", False), (16, "sampled", False),
                            (None, "gemm", False), (16, "sampled", True)):
        sae, opt, fs = build(g, csr_capacity=cap, grad_feat=mode, force_simt=simt)
        fs.microbatch(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
        torch.cuda.synchronize()
        res.append((fs.dense_fallbacks, fs.g_W_enc.clone(), fs.g_W_dec_fm.clone(),
                    fs.g_b_dec.clone(), fs.g_log_thr.clone()))
    assert res[0][0] == 0 and res[1][0] == 1 and res[2][0] == 0 and res[3][0] == 1
    for other in (res[1], res[2], res[3]):
        for a, b in zip(res[0][1:], other[1:]):
            # the sampled dot products and the tensor-core GEMM sum in different
            # orders: grad_feat may differ by one bf16 ulp on a few entries
            assert _rel(b.cpu().numpy(), a.cpu().numpy()) < 2e-3


@pytest.mark.parametrize("swap", [False, True])
def test_overflow_inside_accumulation_matches_sparse_step(swap):
    """The sampled backward is queued before the host reads the forward's
    statistics; a microbatch whose entries overflow the CSR leaves the
    gradients untouched and is redone on the dense path. With one of two
    accumulated microbatches overflowing (first or second), the step equals
    the step without overflow."""
    g = load_golden("ste_f64_accum2")
    cfg = oracle_cfg(g)
    xs = [g[f"x{i}"].astype(np.float32) for i in range(2)]
    if swap:
        xs = xs[::-1]
    mb = xs[0].shape[0]
    x = torch.from_numpy(np.concatenate(xs)).cuda()
    _, _, probe = build(g)
    pairs = [probe.microbatch(torch.from_numpy(xi).cuda(), lambda_l0=cfg.lambda_l0,
                              al_mu=cfg.al_mu, target_l0=cfg.target_l0)["csr_pairs"] for xi in xs]
    if pairs[0] == pairs[1]:
        pytest.skip("both microbatches have the same number of entries")
    runs = []
    for cap in (None, min(pairs)):
        sae, opt, fs = build(g, csr_capacity=cap)
        fs.max_tokens = x.shape[0]
        out = fs.step(x, microbatch_tokens=mb, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu,
                      target_l0=cfg.target_l0)
        torch.cuda.synchronize()
        runs.append((fs.dense_fallbacks, out,
                     [t.clone() for t in (fs.g_W_enc, fs.g_b_enc, fs.g_W_dec_fm, fs.g_b_dec,
                                          fs.g_log_thr)],
                     [t.detach().clone() for t in (sae.W_enc.weight, sae.W_dec.weight,
                                                   sae.log_threshold)]))
    (f0, o0, g0, p0), (f1, o1, g1, p1) = runs
    assert f0 == 0 and f1 == 1
    for a, b in zip(g0, g1):
        assert _rel(b.cpu().numpy(), a.cpu().numpy()) < 2e-3
    assert o1["grad_norm"] == pytest.approx(o0["grad_norm"], rel=2e-3)
    assert o1["l0"] == o0["l0"] and o1["recon_loss"] == o0["recon_loss"]
    lr = float(g["lr"])
    for a, b in zip(p0, p1):
        assert float((a - b).abs().max()) <= 2.5 * lr


def test_step_is_deterministic():
    g = load_golden("super_f32_tiles")
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    outs = []
    for _ in range(2):
        sae, opt, fs = build(g)
        fs.step(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
        torch.cuda.synchronize()
        outs.append([t.clone() for t in (fs.g_W_enc, fs.g_W_dec_fm, fs.g_b_dec, fs.g_log_thr,
                                         sae.W_enc.weight.detach(), sae.W_dec.weight.detach())])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_bf16_input_matches_oracle():
    """The trainer feeds bf16 activations (provider shards, 1606-1609)."""
    g = load_golden("super_f32_tiles")
    sae, opt, fs = build(g)
    cfg = oracle_cfg(g)
    xb = torch.from_numpy(g["x0"].astype(np.float32)).to(torch.bfloat16)
    st = fs.microbatch(xb.cuda(), lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu,
                       target_l0=cfg.target_l0)
    fw = O.forward(xb.float().numpy(), oracle_params(g), cfg, "bf16",
                   theta=kernel_theta(fs, xb.shape[0]))
    assert st["recon_loss"] == pytest.approx(fw.recon_loss, rel=BF16_TOL)
    ref = O.backward(xb.float().numpy(), oracle_params(g), fw, cfg, "bf16")
    assert _rel(fs.g_W_enc.cpu().numpy(), ref.W_enc) < BF16_TOL
    assert _rel(fs.g_log_thr.cpu().numpy(), ref.log_threshold) < BF16_TOL


@pytest.mark.parametrize("grad_feat", ["sampled", "gemm"])
def test_wide_rows_match_oracle(grad_feat):
    """d = 2048: the wide-row variant of the sampled backward (two 16-byte
    vectors per thread) against the oracle's backward on the same gates."""
    import math
    from sae_b200 import B200Adam, FusedStep, make_sae, reference_param_groups
    d, F, B = 2048, 256, 192
    x = O.superposition_batch(B, d, 512, 12, math.log(12.0), 0.3, seed=23)
    sae = make_sae(d, F, seed=4)
    with torch.no_grad():
        sae.b_dec.copy_(torch.from_numpy(x.mean(0)))
        sae.log_threshold.fill_(math.log(0.25))
    p0 = O.Params(sae.W_enc.weight.detach().numpy().copy(), sae.W_enc.bias.detach().numpy().copy(),
                  sae.W_dec.weight.detach().numpy().copy(), sae.b_dec.detach().numpy().copy(),
                  sae.log_threshold.detach().numpy().copy())
    sae = sae.cuda()
    sae.ste_bandwidth = 0.05
    lr = 1e-4
    opt = B200Adam(reference_param_groups(sae, lr), lr=lr, sae=sae, renorm=True)
    fs = FusedStep(sae, opt, max_tokens=B, grad_feat=grad_feat, pre_store="full")
    cfg = O.StepConfig(lambda_l0=1e-3, al_mu=1e-2, target_l0=8.0, ste_bandwidth=0.05,
                       lr=(lr,) * 4)
    xt = torch.from_numpy(x).cuda()
    st = fs.microbatch(xt, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
    torch.cuda.synchronize()
    v = workspace_views(fs, B)
    # the oracle's backward given the kernel's own thresholds and bf16 pre-activations
    # (a dense case: ~17% active, many entries within one bf16 ulp of the threshold)
    fw = O.forward(x, p0, cfg, "bf16", theta=v["theta"].cpu().numpy(),
                   pre=v["pre"].float().cpu().numpy())
    assert fw.l0 > 2 and st["l0"] == pytest.approx(fw.l0, rel=1e-6)
    ref = O.backward(x, p0, fw, cfg, "bf16")
    for k, t in {"W_enc": fs.g_W_enc, "b_enc": fs.g_b_enc, "W_dec": fs.g_W_dec_fm.t(),
                 "b_dec": fs.g_b_dec, "log_threshold": fs.g_log_thr}.items():
        assert _rel(t.cpu().numpy(), getattr(ref, k)) < 5e-3, k


@pytest.mark.parametrize("B", [1, 33, 333])
def test_ragged_token_counts_match_oracle(B):
    """Token counts that fill no whole tile, 32-token word or 8-token group on
    the tcgen05 path (d % 64 == 0, F % 256 == 0): gradients against the
    oracle's backward on the kernel's own gates, and the default entries-only
    pre store bit-identical to the full store."""
    import math
    from sae_b200 import B200Adam, FusedStep, make_sae, reference_param_groups
    d, F = 128, 512
    x = O.superposition_batch(B, d, 1024, 12, math.log(8.0), 0.3, seed=41 + B)
    p0 = None
    grads = {}
    for store in ("full", "entries"):
        sae = make_sae(d, F, seed=6)
        with torch.no_grad():
            sae.b_dec.copy_(torch.from_numpy(x.mean(0)))
            sae.log_threshold.fill_(math.log(0.2))
        if p0 is None:
            p0 = O.Params(*(t.detach().numpy().copy() for t in (
                sae.W_enc.weight, sae.W_enc.bias, sae.W_dec.weight, sae.b_dec,
                sae.log_threshold)))
        sae = sae.cuda()
        sae.ste_bandwidth = 0.05
        opt = B200Adam(reference_param_groups(sae, 1e-4), lr=1e-4, sae=sae, renorm=True)
        fs = FusedStep(sae, opt, max_tokens=B, pre_store=store)
        cfg = O.StepConfig(lambda_l0=1e-3, al_mu=1e-2, target_l0=4.0, ste_bandwidth=0.05,
                           lr=(1e-4,) * 4)
        st = fs.microbatch(torch.from_numpy(x).cuda(), lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu,
                           target_l0=cfg.target_l0)
        torch.cuda.synchronize()
        from sae_b200 import _lib as L
        assert L.device_status() == 0
        grads[store] = (st, [t.clone() for t in (fs.g_W_enc, fs.g_b_enc, fs.g_W_dec_fm,
                                                 fs.g_b_dec, fs.g_log_thr)])
        if store == "full":
            v = workspace_views(fs, B)
            fw = O.forward(x, p0, cfg, "bf16", theta=v["theta"].cpu().numpy(),
                           pre=v["pre"].float().cpu().numpy())
            assert st["l0"] == pytest.approx(fw.l0, rel=1e-6)
            assert st["nnz"] == int(round(fw.l0 * B))
            ref = O.backward(x, p0, fw, cfg, "bf16")
            for k, t in {"W_enc": fs.g_W_enc, "b_enc": fs.g_b_enc, "W_dec": fs.g_W_dec_fm.t(),
                         "b_dec": fs.g_b_dec, "log_threshold": fs.g_log_thr}.items():
                r = getattr(ref, k)
                if np.linalg.norm(r) > 0:
                    assert _rel(t.cpu().numpy(), r) < 5e-3, k
                else:
                    assert float(t.abs().max()) == 0.0, k
    assert grads["full"][0] == grads["entries"][0]
    for a, b in zip(grads["full"][1], grads["entries"][1]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("name,force_simt", CASES)
def test_entries_only_pre_store_matches_full_store(name, force_simt):
    """The default forward stores pre only in the 32-token words that hold an
    active or in-band entry. Stats and gradients are bit-identical to the full
    store, the stored words hold the same values, and no other word is touched
    (the workspace's pre region starts as NaN)."""
    g = load_golden(name)
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    B = x.shape[0]
    runs = {}
    for mode in ("full", "entries"):
        sae, opt, fs = build(g, force_simt=force_simt, pre_store=mode)
        F = sae.n_features
        from sae_b200 import _lib as L
        ldp = L.pre_pitch(B)
        o = L.workspace_offsets(B, sae.d_in, F, fs.csr_capacity)["pre"]
        fs.ws[o:o + 2 * F * ldp].fill_(255)          # bf16 0xFFFF: NaN
        st = fs.microbatch(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0)
        torch.cuda.synchronize()
        assert L.device_status() == 0
        grads = [t.clone() for t in (fs.g_W_enc, fs.g_b_enc, fs.g_W_dec_fm, fs.g_b_dec,
                                     fs.g_log_thr)]
        pre = fs.ws[o:o + 2 * F * ldp].view(torch.bfloat16).view(F, ldp)[:, :B]
        runs[mode] = (st, grads, pre.float().cpu().numpy(), kernel_theta(fs, B), fs.fired.clone())
    st_f, g_f, pre_f, theta, fired_f = runs["full"]
    st_e, g_e, pre_e, _, fired_e = runs["entries"]
    assert st_f == st_e
    assert torch.equal(fired_f, fired_e)
    for a, b in zip(g_f, g_e):
        assert torch.equal(a, b)
    assert not np.isnan(pre_f).any()
    eps = np.float32(g["eps"])
    entry = (pre_f - theta[:, None]) > -eps              # active or in band, fp32 as the kernel
    F = entry.shape[0]
    nw = (B + 31) // 32
    pad = np.zeros((F, nw * 32), dtype=bool)
    pad[:, :B] = entry
    word = np.repeat(pad.reshape(F, nw, 32).any(-1), 32, axis=1)[:, :B]
    np.testing.assert_array_equal(pre_e[word], pre_f[word])
    assert np.isnan(pre_e[~word]).all()


@pytest.mark.parametrize("case", ["single", "accum2", "frozen_decoder", "overflow"])
def test_norm_from_backward_partials_matches_full_pass(case):
    """The clip norm queued straight after the sampled backward is summed from
    that backward's per-feature partials (sae_b200_grad_norm_sampled); it must
    equal the norm of a full pass over the final gradients (sae_b200_grad_norm)
    up to the fp32 summation order, after accumulation, with a frozen decoder,
    and when an overflowing microbatch sends the backward down the dense path
    (which queues the full pass again)."""
    name = "ste_f64_accum2" if case == "accum2" else "super_f32_tiles"
    g = load_golden(name)
    sae, opt, fs = build(g, csr_capacity=16 if case == "overflow" else None)
    if case == "frozen_decoder":
        sae.W_dec.weight.requires_grad_(False)
    cfg = oracle_cfg(g)
    n = 2 if case == "accum2" else 1
    xs = [torch.from_numpy(g[f"x{i}"].astype(np.float32)).cuda() for i in range(n)]
    fs.max_tokens = max(x.shape[0] for x in xs)
    for i, x in enumerate(xs):
        fs.microbatch(x, accum_steps=n, first=(i == 0), lambda_l0=cfg.lambda_l0,
                      al_mu=cfg.al_mu, target_l0=cfg.target_l0,
                      after_backward=(lambda: fs.grad_norm(1.0)) if i == n - 1 else None)
    fused = fs.read_stats()
    fs.grad_norm(1.0)
    full = fs.read_stats()
    assert fs.dense_fallbacks == (1 if case == "overflow" else 0)
    assert full["grad_norm"] > 0
    assert fused["grad_norm"] == pytest.approx(full["grad_norm"], rel=1e-5)
    assert fused["clip_coef"] == pytest.approx(full["clip_coef"], rel=1e-5)
