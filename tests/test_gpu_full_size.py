"""Parity at the benchmark size (d=1536, F=49152, 32768 tokens), by properties
that do not need a full CPU recomputation:

  * active sets: mask bits == (pre > theta) for sampled tokens (bit-exact);
    per-token counts == popcount; nnz == sum of counts; the backward's CSR
    holds them plus the inactive in-band entries;
  * decode: sampled tokens (including the one with the most active features)
    recomputed in float64 from the kernel's own pre-activations and bf16
    decoder rows: x_hat within one bf16 ulp of the float64 sum (+ b_dec);
  * loss: recon == mean((x - x_hat)^2) over all tokens (1e-5 relative);
  * backward: for sampled features, grad_feat recomputed in float64 from the
    kernel's bf16 go and decoder row, then the STE sum, db_enc and the dW_enc /
    dW_dec rows: relative error < 1e-3 (grad_feat is rounded to bf16, and an
    fp32 accumulation can round to the neighbouring bf16 value);
  * the sampled backward (default) and the dense tcgen05 grad_feat GEMM give
    the same gradients (2e-3 relative);
  * determinism: the same step twice gives bit-identical gradients;
  * after Adam: unit-norm W_enc rows / W_dec columns, bf16 copies == rounding
    of the fp32 masters.
"""
import math

import numpy as np
import pytest
import torch

from oracle.sae_oracle import bf16

pytestmark = pytest.mark.gpu

D, F, B = 1536, 49152, 32768


@pytest.fixture(scope="module")
def setup():
    import sae_b200
    from sae_b200 import _lib as L
    dev = torch.device("cuda")
    x = sae_b200.superposition_batch(B, D, F, 50, math.log(60.0), 0.4, seed=17, device=dev)
    sae = sae_b200.make_sae(D, F, seed=0).to(dev)
    sae.ste_bandwidth = 0.2
    with torch.no_grad():
        sae.b_dec.copy_(x.float().mean(0))
        with torch.autocast("cuda", dtype=torch.bfloat16):
            pre = sae.encode_pre(x[:1024])
        flat = pre.float().flatten()
        q = torch.quantile(flat[torch.randperm(flat.numel(), device=dev)[:2_000_000]],
                           1.0 - 50.0 / F).item()
        sae.log_threshold.fill_(math.log(q))
    opt = sae_b200.B200Adam(sae_b200.reference_param_groups(sae, 2e-4), lr=2e-4, sae=sae,
                            renorm=True)
    fs = sae_b200.FusedStep(sae, opt, max_tokens=B, pre_store="full")
    x_hat = torch.empty(B, D, device=dev)
    st = fs.microbatch(x, lambda_l0=1e-3, al_mu=1e-2, target_l0=50, x_hat_out=x_hat)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    off = L.workspace_offsets(B, D, F, fs.csr_capacity)
    ldp = L.pre_pitch(B)

    def region(name, dtype, count):
        nb = count * torch.tensor([], dtype=dtype).element_size()
        return fs.ws[off[name]:off[name] + nb].view(dtype)

    ws = {
        "theta": region("theta", torch.float32, F),
        "pre_fm": region("pre", torch.bfloat16, F * ldp).view(F, ldp),
        "mask": region("mask", torch.int32, B * (F // 32)).view(B, F // 32),
        "go": region("go", torch.bfloat16, B * D).view(B, D),
        "tok_cnt": region("tok_cnt", torch.int32, B),
        "col_offs": region("col_offs", torch.int32, F + 1),
    }
    grads = {k: t.clone() for k, t in (("W_enc", fs.g_W_enc), ("b_enc", fs.g_b_enc),
                                        ("W_dec_fm", fs.g_W_dec_fm), ("b_dec", fs.g_b_dec),
                                        ("log_threshold", fs.g_log_thr))}
    return dict(sae=sae, fs=fs, x=x, x_hat=x_hat, st=st, ws=ws, grads=grads, ldp=ldp)


def _bits(words):
    w = words.cpu().numpy().view(np.uint32)
    return ((w[:, :, None] >> np.arange(32, dtype=np.uint32)) & 1).reshape(w.shape[0], -1) > 0


def test_active_sets_are_exact(setup):
    ws, st = setup["ws"], setup["st"]
    cnt = ws["tok_cnt"].cpu().numpy()
    assert 20 < st["l0"] < 120
    assert st["nnz"] == int(cnt.sum())
    assert st["csr_pairs"] == int(ws["col_offs"][-1]) >= st["nnz"]
    rng = np.random.default_rng(0)
    toks = np.unique(np.concatenate([rng.choice(B, 48, replace=False), [int(cnt.argmax())]]))
    theta = ws["theta"].cpu().numpy()
    pre = ws["pre_fm"][:, torch.from_numpy(toks).cuda()].float().cpu().numpy().T   # [n, F]
    gate = pre > theta
    bits = _bits(ws["mask"][torch.from_numpy(toks).cuda()])
    np.testing.assert_array_equal(bits, gate)
    np.testing.assert_array_equal(cnt[toks], gate.sum(1))


def test_decode_and_loss(setup):
    ws, sae, x, x_hat, st = setup["ws"], setup["sae"], setup["x"], setup["x_hat"], setup["st"]
    cnt = ws["tok_cnt"].cpu().numpy()
    toks = [int(cnt.argmax())] + list(np.random.default_rng(1).choice(B, 24, replace=False))
    theta = ws["theta"].cpu().numpy()
    wdec = sae._shadow_dec.float().cpu().numpy().astype(np.float64)   # bf16 rows [F, D]
    bdec = sae.b_dec.detach().cpu().numpy()
    for t in toks:
        p = ws["pre_fm"][:, t].float().cpu().numpy()
        act = np.nonzero(p > theta)[0]
        s = (p[act].astype(np.float64)[:, None] * wdec[act]).sum(0)
        ref = bf16(s.astype(np.float32)).astype(np.float64) + bdec
        got = x_hat[t].cpu().numpy().astype(np.float64)
        ulp = np.abs(s) * 2.0 ** -7 + 1e-6
        assert np.all(np.abs(got - ref) <= ulp + 1e-6), f"token {t}"
    r = (x.double() - x_hat.double())
    recon = float(r.pow(2).mean())
    assert st["recon_loss"] == pytest.approx(recon, rel=1e-5)
    # go = bf16(-(2 r) / (B d))
    go_ref = bf16((-(2.0 * r[:64]) / (B * D)).float().cpu().numpy())
    np.testing.assert_allclose(ws["go"][:64].float().cpu().numpy(), go_ref, rtol=2 ** -7, atol=0)


def test_backward_sampled_features(setup):
    ws, sae, g, st = setup["ws"], setup["sae"], setup["grads"], setup["st"]
    eps = 0.2
    feats = np.random.default_rng(2).choice(F, 48, replace=False)
    fi = torch.from_numpy(feats).cuda()
    theta = ws["theta"][fi].double().cpu().numpy()
    go = ws["go"].double().cpu().numpy()                               # [B, D] bf16 values
    wdec = sae._shadow_dec[fi].double().cpu().numpy()                  # bf16 rows
    pre = ws["pre_fm"][fi, :B].double().cpu().numpy()                  # [n, B]
    gf = bf16((go @ wdec.T).T.astype(np.float32)).astype(np.float64)   # [n, B]
    # gate_grad from the loss terms: (lambda + mu * slack) / B where l0 >= target
    slack = max(st["l0"] - 50.0, 0.0)
    c = ((1e-3 + 1e-2 * slack) / B) if st["l0"] >= 50.0 else 0.0
    comb = pre * gf + c
    in_band = np.abs(pre - theta[:, None]) < eps
    thr = np.where(in_band, comb, 0.0).sum(1)
    g_lt = -(thr / (2 * eps)) * theta
    got_lt = g["log_threshold"][fi].double().cpu().numpy()
    assert np.linalg.norm(got_lt - g_lt) <= 1e-3 * np.linalg.norm(g_lt)
    act = pre > theta[:, None]
    db = np.where(act, gf, 0.0).sum(1)
    got_db = g["b_enc"][fi].double().cpu().numpy()
    assert np.linalg.norm(got_db - db) <= 1e-3 * max(np.linalg.norm(db), 1e-30)
    xc = bf16((setup["x"].float() - sae.b_dec.detach().float()).cpu().numpy()).astype(np.float64)
    dW_enc = np.where(act, gf, 0.0) @ xc                                # [n, D]
    dW_dec = np.where(act, pre, 0.0) @ go                               # [n, D]
    got_we = g["W_enc"][fi].double().cpu().numpy()
    got_wd = g["W_dec_fm"][fi].double().cpu().numpy()
    assert np.linalg.norm(got_we - dW_enc) <= 1e-3 * np.linalg.norm(dW_enc)
    assert np.linalg.norm(got_wd - dW_dec) <= 1e-4 * np.linalg.norm(dW_dec)


def test_sampled_and_gemm_backward_agree_at_full_size(setup):
    """The default backward computes grad_feat only on the active and in-band
    entries; the dense tcgen05 grad_feat GEMM must give the same gradients (up
    to one-bf16-ulp differences of grad_feat from the summation order)."""
    import sae_b200
    sae, x, g = setup["sae"], setup["x"], setup["grads"]
    fs2 = sae_b200.FusedStep(sae, setup["fs"].opt, max_tokens=B, grad_feat="gemm")
    st2 = fs2.microbatch(x, lambda_l0=1e-3, al_mu=1e-2, target_l0=50)
    torch.cuda.synchronize()
    assert st2["nnz"] == setup["st"]["nnz"]
    for k, t in (("W_enc", fs2.g_W_enc), ("b_enc", fs2.g_b_enc), ("W_dec_fm", fs2.g_W_dec_fm),
                 ("b_dec", fs2.g_b_dec), ("log_threshold", fs2.g_log_thr)):
        a, b = t.double(), g[k].double()
        assert float((a - b).norm() / b.norm()) < 2e-3, k
    del fs2


def test_dense_fallback_at_full_size(setup):
    """A microbatch whose entries overflow the CSR takes the dense weight-
    gradient path: dW_enc = dpre^T xc and dW_dec = acts^T go as two tcgen05
    GEMMs contracting over the 32768 tokens. Same gradients as the sampled
    backward (2e-3 relative: the weight gradients are summed in another order
    and grad_feat may differ by one bf16 ulp)."""
    import sae_b200
    sae, x, g = setup["sae"], setup["x"], setup["grads"]
    fs4 = sae_b200.FusedStep(sae, setup["fs"].opt, max_tokens=B, csr_capacity=4096)
    st4 = fs4.microbatch(x, lambda_l0=1e-3, al_mu=1e-2, target_l0=50)
    torch.cuda.synchronize()
    assert fs4.dense_fallbacks == 1
    assert st4["nnz"] == setup["st"]["nnz"]
    for k, t in (("W_enc", fs4.g_W_enc), ("b_enc", fs4.g_b_enc), ("W_dec_fm", fs4.g_W_dec_fm),
                 ("b_dec", fs4.g_b_dec), ("log_threshold", fs4.g_log_thr)):
        a, b = t.double(), g[k].double()
        assert float((a - b).norm() / b.norm()) < 2e-3, k
    del fs4


def test_entries_only_pre_store_is_bit_identical_at_full_size(setup):
    """The default forward stores pre only where an entry is; at the full
    workload its statistics and gradients equal the full store's bit for bit."""
    import sae_b200
    sae, x, g = setup["sae"], setup["x"], setup["grads"]
    fs3 = sae_b200.FusedStep(sae, setup["fs"].opt, max_tokens=B)
    assert fs3.pre_store == "entries"
    st3 = fs3.microbatch(x, lambda_l0=1e-3, al_mu=1e-2, target_l0=50)
    torch.cuda.synchronize()
    assert st3 == setup["st"]
    for k, t in (("W_enc", fs3.g_W_enc), ("b_enc", fs3.g_b_enc), ("W_dec_fm", fs3.g_W_dec_fm),
                 ("b_dec", fs3.g_b_dec), ("log_threshold", fs3.g_log_thr)):
        assert torch.equal(t, g[k]), k
    del fs3


def test_aux_loss_at_full_size(setup):
    """The dead-feature aux loss at the full workload (every 10th feature dead,
    k = 25): the kernel's aux loss against the oracle's restatement of
    2986-2998 evaluated on the kernel's own bf16 pre-activations and x_hat
    (top-k with ties to the lower dead index, relu, bf16 decoder operands and
    output, fp64 sums). Differences come from summation order only."""
    import sae_b200
    from sae_b200 import _lib as L
    sae, x = setup["sae"], setup["x"]
    dead = torch.arange(0, F, 10, device="cuda", dtype=torch.int32)
    k, coeff = 25, 1.0 / 32
    fs = sae_b200.FusedStep(sae, setup["fs"].opt, max_tokens=B)
    fs.set_aux(dead, k, coeff)
    st = fs.microbatch(x, lambda_l0=1e-3, al_mu=1e-2, target_l0=50)
    torch.cuda.synchronize()
    assert L.device_status() == 0
    ldp = L.pre_pitch(B)
    off = L.workspace_offsets(B, D, F, fs.csr_capacity)["pre"]
    pre = fs.ws[off:off + 2 * F * ldp].view(torch.bfloat16).view(F, ldp)
    dl = dead.long()
    pre_dead = pre[dl, :B].t().float().cpu().numpy()                 # [B, n_dead]
    resid = (x.float() - fs._x_hat[:B]).cpu().numpy().astype(np.float64)
    wd = torch.from_numpy(bf16(sae.W_dec.weight.detach()[:, dl].t().contiguous().cpu().numpy()))
    v = np.maximum(pre_dead, 0)
    kth = -np.partition(-v, k - 1, axis=1)[:, k - 1:k]                # k-th largest per token
    gt = v > kth
    eq = (v == kth) & (kth > 0)
    need = k - gt.sum(1, keepdims=True)
    sel = gt | (eq & (np.cumsum(eq, axis=1) <= need))
    sel &= v > 0
    sq = 0.0
    for b0 in range(0, B, 2048):
        rows = slice(b0, b0 + 2048)
        acts = torch.from_numpy(np.where(sel[rows], v[rows], 0).astype(np.float64))
        x_aux = bf16((acts @ wd.double()).numpy().astype(np.float32)).astype(np.float64)
        sq += float(np.square(resid[rows] - x_aux).sum())
    aux_ref = coeff * sq / (B * D)
    assert aux_ref > 0
    assert st["aux_loss"] == pytest.approx(aux_ref, rel=1e-3)
    del fs


def test_step_is_deterministic_at_full_size(setup):
    fs, x, g = setup["fs"], setup["x"], setup["grads"]
    fs.microbatch(x, lambda_l0=1e-3, al_mu=1e-2, target_l0=50)
    torch.cuda.synchronize()
    for k, t in (("W_enc", fs.g_W_enc), ("b_enc", fs.g_b_enc), ("W_dec_fm", fs.g_W_dec_fm),
                 ("b_dec", fs.g_b_dec), ("log_threshold", fs.g_log_thr)):
        assert torch.equal(t, g[k]), k


def test_adam_renorm_and_bf16_copies(setup):
    sae, fs = setup["sae"], setup["fs"]
    fs.grad_norm(1.0)
    fs.optimizer_step()
    torch.cuda.synchronize()
    with torch.no_grad():
        ne = sae.W_enc.weight.norm(dim=1)
        nd = sae.W_dec.weight.norm(dim=0)
    torch.testing.assert_close(ne, torch.ones_like(ne), rtol=0, atol=1e-5)
    torch.testing.assert_close(nd, torch.ones_like(nd), rtol=0, atol=1e-5)
    rows = torch.arange(0, F, 997, device="cuda")
    np.testing.assert_array_equal(sae._shadow_enc[rows].float().cpu().numpy(),
                                  bf16(sae.W_enc.weight.detach()[rows].cpu().numpy()))
    np.testing.assert_array_equal(sae._shadow_dec[rows].float().cpu().numpy(),
                                  bf16(sae.W_dec.weight.detach().t()[rows].cpu().numpy()))

