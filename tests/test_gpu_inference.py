"""Fused inference (encoder GEMM + JumpReLU gate + gathered decode, no backward
state) against the oracle's bf16 forward and against the training forward.

Tolerances: active counts bit-exact against the kernel's own pre-activations
and thresholds; x_hat within 2e-2 relative L2 of the oracle (bf16 operands),
and bit-identical to the x_hat of the training forward (same kernels)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import sae_oracle as O
from test_gpu_fused_step import BF16_TOL, _rel, build, oracle_cfg, oracle_params

pytestmark = pytest.mark.gpu


def _views(sae, B):
    from sae_b200 import _lib as L
    F = sae.n_features
    off = L.workspace_offsets(B, sae.d_in, F, 0)
    ws = sae._infer_ws
    ldp = L.pre_pitch(B)
    theta = ws[off["theta"]:off["theta"] + 4 * F].view(torch.float32)
    pre = ws[off["pre"]:off["pre"] + 2 * F * ldp].view(torch.bfloat16).view(F, ldp)[:, :B].t()
    return theta.cpu().numpy(), pre.float().cpu().numpy()


@pytest.mark.parametrize("name,dtype", [("super_f32_tiles", torch.float32),
                                        ("super_f32_tiles", torch.bfloat16),
                                        ("super_f32_odd", torch.float32),
                                        ("ste_f64", torch.float32)])
def test_reconstruct_matches_oracle_forward(name, dtype):
    g = load_golden(name)
    sae, opt, fs = build(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).to(dtype).cuda()
    fired = torch.zeros(sae.n_features, dtype=torch.uint8, device="cuda")
    from sae_b200 import _lib as L
    # pre is stored only in the 32-token words holding an active entry; the
    # rest of the workspace stays NaN (bf16 0xFFFF), which no gate passes
    need = L.workspace_bytes(x.shape[0], sae.d_in, sae.n_features, 0)
    sae._infer_ws = torch.full((need,), 255, dtype=torch.uint8, device="cuda")
    x_hat, counts = sae.reconstruct(x, fired=fired)
    torch.cuda.synchronize()
    from sae_b200 import _lib as L
    assert L.device_status() == 0
    theta, pre = _views(sae, x.shape[0])
    gate = pre > theta
    np.testing.assert_array_equal(counts.cpu().numpy(), gate.sum(1))
    B = x.shape[0]
    nw = (B + 31) // 32
    pad_g = np.zeros((nw * 32, sae.n_features), dtype=bool)
    pad_g[:B] = gate
    pad_w = np.zeros((nw * 32, sae.n_features), dtype=bool)
    pad_w[:B] = ~np.isnan(pre)
    # a word is stored exactly when it holds an active entry
    np.testing.assert_array_equal(pad_w.reshape(nw, 32, -1).any(1), pad_g.reshape(nw, 32, -1).any(1))
    assert fired.bool().cpu().numpy().tolist() == gate.any(0).tolist()
    fw = O.forward(x.float().cpu().numpy(), oracle_params(g), oracle_cfg(g), "bf16", theta=theta)
    assert _rel(x_hat.cpu().numpy(), fw.x_hat) < BF16_TOL
    # the training forward computes the same x_hat with the same kernels
    ref = torch.empty_like(x_hat)
    cfg = oracle_cfg(g)
    fs.microbatch(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0,
                  x_hat_out=ref)
    torch.cuda.synchronize()
    assert torch.equal(ref, x_hat)


def test_reconstruct_twice_is_identical_and_rejects_bad_shapes():
    g = load_golden("super_f32_tiles")
    sae, _, _ = build(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    a, ca = sae.reconstruct(x)
    b, cb = sae.reconstruct(x)
    assert torch.equal(a, b) and torch.equal(ca, cb)
    with pytest.raises(ValueError):
        sae.reconstruct(x[:, :-1])
