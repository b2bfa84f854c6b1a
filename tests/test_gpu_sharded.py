"""Parity of the dictionary-sharded step (one wide SAE split over ranks by
features) on the GPU.

On one GPU the ranks are emulated: each shard has its own ShardedFusedStep
running in its own host thread, and the three cross-rank sums are done by a
thread barrier plus an in-order torch sum on the shared stream (no kernel
waits on another). With two or more GPUs the same step runs as torchrun
processes over NCCL. Both are checked against the oracle's whole-dictionary
step (bf16 mode, the kernel's own thresholds) and against the unsharded
FusedStep; tolerances as in test_gpu_fused_step: active sets bit-exact given
the kernel's pre-activations, pre within one bf16 ulp of the unsharded pass,
gradients within 2e-2 relative L2 of the oracle, Adam within 2.5 lr.
"""
import json
import os
import subprocess
import sys
import threading
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import sae_oracle as O
from test_gpu_fused_step import (BF16_TOL, _rel, build, kernel_theta, oracle_cfg, oracle_params,
                                 unpack_mask, workspace_views)

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


class ThreadSum:
    """In-place sum over emulated ranks (host threads sharing one stream)."""

    def __init__(self, world):
        self.world = world
        self.bar = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def for_rank(self, r):
        def allreduce(t):
            self.slots[r] = t
            self.bar.wait()
            if r == 0:
                tot = self.slots[0].clone()
                for s in self.slots[1:]:
                    tot += s
                for s in self.slots:
                    s.copy_(tot)
            self.bar.wait()
        return allreduce


def run_emulated(g, world, x, cfg, steps=1, microbatch_tokens=None, pre_store="entries",
                 csr_capacity=None):
    import sae_b200
    from sae_b200 import B200Adam, ShardedFusedStep, reference_param_groups
    full, _, _ = build(g)
    lr = float(g["lr"])
    shards, steppers = [], []
    ts = ThreadSum(world)
    for r in range(world):
        s = sae_b200.shard_sae(full, r, world)
        s.ste_bandwidth = float(g["eps"])
        opt = B200Adam(reference_param_groups(s, lr), lr=lr, betas=(0.9, 0.999), sae=s,
                       renorm=True)
        steppers.append(ShardedFusedStep(s, opt, max_tokens=x.shape[0],
                                         allreduce=ts.for_rank(r), rank=r, world=world,
                                         pre_store=pre_store, csr_capacity=csr_capacity))
        shards.append(s)
    outs = [None] * world
    errs = []
    wf = float(g["wenc_factor"])

    def work(r):
        try:
            for _ in range(steps):
                outs[r] = steppers[r].step(x, microbatch_tokens=microbatch_tokens,
                                           lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu,
                                           target_l0=cfg.target_l0, wenc_dampen=lambda l0: wf)
        except BaseException as e:   # surfaced below
            errs.append(e)
            ts.bar.abort()

    th = [threading.Thread(target=work, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    if errs:
        raise errs[0]
    torch.cuda.synchronize()
    return shards, steppers, outs


def gather(shards, steppers):
    cat = lambda ts, dim=0: torch.cat([t.detach().cpu() for t in ts], dim=dim).numpy()
    return {
        "g_W_enc": cat([s.g_W_enc for s in steppers]),
        "g_b_enc": cat([s.g_b_enc for s in steppers]),
        "g_W_dec": cat([s.g_W_dec_fm for s in steppers]).T,
        "g_log_threshold": cat([s.g_log_thr for s in steppers]),
        "g_b_dec": steppers[0].g_b_dec.cpu().numpy(),
        "W_enc": cat([s.W_enc.weight for s in shards]),
        "b_enc": cat([s.W_enc.bias for s in shards]),
        "W_dec": cat([s.W_dec.weight for s in shards], dim=1),
        "b_dec": shards[0].b_dec.detach().cpu().numpy(),
        "log_threshold": cat([s.log_threshold for s in shards]),
    }


@pytest.mark.parametrize("world", [2, 4])
def test_emulated_shards_match_oracle_and_unsharded(world):
    g = load_golden("super_f32_tiles")
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    # (pre stored in full: the test reads every shard's pre-activations)
    shards, steppers, outs = run_emulated(g, world, x, cfg, pre_store="full")
    from sae_b200 import _lib as L
    assert L.device_status() == 0
    # every rank sees the same loss, L0 and grad norm, and the same b_dec
    for o in outs[1:]:
        assert o["l0"] == outs[0]["l0"]
        assert o["recon_loss"] == outs[0]["recon_loss"]
        assert o["grad_norm"] == outs[0]["grad_norm"]
    for s in shards[1:]:
        assert torch.equal(s.b_dec, shards[0].b_dec)
    # unsharded reference pass on the same GPU
    sae, opt, fs = build(g, pre_store="full")
    wf = float(g["wenc_factor"])
    one = fs.step(x, lambda_l0=cfg.lambda_l0, al_mu=cfg.al_mu, target_l0=cfg.target_l0,
                  wenc_dampen=lambda l0: wf)
    theta = kernel_theta(fs, x.shape[0])
    B, F = x.shape[0], sae.n_features
    per = F // world
    pre_full = workspace_views(fs, B)["pre"].float().cpu().numpy()
    for r, st in enumerate(steppers):
        v = workspace_views(st, B)
        pre = v["pre"].float().cpu().numpy()
        th = v["theta"].cpu().numpy()
        np.testing.assert_array_equal(th, theta[r * per:(r + 1) * per])
        gate = pre > th
        np.testing.assert_array_equal(unpack_mask(v["mask"], per), gate)
        ulp = np.abs(pre_full[:, r * per:(r + 1) * per]) * 2.0 ** -7 + 1e-30
        assert np.all(np.abs(pre - pre_full[:, r * per:(r + 1) * per]) <= ulp * 1.01)
    assert outs[0]["l0"] == pytest.approx(one["l0"], rel=1e-3)
    assert outs[0]["recon_loss"] == pytest.approx(one["recon_loss"], rel=1e-3)
    got = gather(shards, steppers)
    unsh = {"g_W_enc": fs.g_W_enc, "g_b_enc": fs.g_b_enc, "g_W_dec": fs.g_W_dec_fm.t(),
            "g_log_threshold": fs.g_log_thr, "g_b_dec": fs.g_b_dec}
    for k, t in unsh.items():
        assert _rel(got[k], t.cpu().numpy()) < 2e-3, k
    p0 = oracle_params(g)
    ref = O.train_step([g["x0"].astype(np.float32)], p0, O.AdamState.zeros_like(p0), cfg,
                       "bf16", theta=theta)
    for k in O.PARAM_NAMES:
        assert _rel(got["g_" + k], getattr(ref.grads, k)) < BF16_TOL, k
        diff = np.abs(got[k] - getattr(ref.params, k))
        assert diff.max() <= 2.5 * float(g["lr"]) + 1e-6, k
    assert outs[0]["grad_norm"] == pytest.approx(ref.grad_norm, rel=BF16_TOL)


def test_emulated_shards_entries_only_and_overflow_match_full_store():
    """The shards' default forward stores pre at the entries only; a shard
    whose CSR overflows stores the rest locally (no second exchange) before
    its dense backward. Against the full-store run without overflow: same
    statistics, gradients within the sampled/dense tolerance."""
    g = load_golden("super_f32_tiles")
    cfg = oracle_cfg(g)
    x = torch.from_numpy(g["x0"].astype(np.float32)).cuda()
    ref_sh, ref_st, ref_out = run_emulated(g, 2, x, cfg, pre_store="full")
    ref = gather(ref_sh, ref_st)
    ent_sh, ent_st, ent_out = run_emulated(g, 2, x, cfg)
    assert all(s.dense_fallbacks == 0 for s in ent_st)
    ent = gather(ent_sh, ent_st)
    for k in ("g_W_enc", "g_b_enc", "g_W_dec", "g_log_threshold", "g_b_dec"):
        np.testing.assert_array_equal(ent[k], ref[k])
    # a capacity below every shard's entry count: all shards take the dense path
    ovf_sh, ovf_st, ovf_out = run_emulated(g, 2, x, cfg, csr_capacity=16)
    assert all(s.dense_fallbacks == 1 for s in ovf_st)
    from sae_b200 import _lib as L
    assert L.device_status() == 0
    ovf = gather(ovf_sh, ovf_st)
    assert ovf_out[0]["l0"] == ref_out[0]["l0"]
    assert ovf_out[0]["recon_loss"] == ref_out[0]["recon_loss"]
    for k in ("g_W_enc", "g_b_enc", "g_W_dec", "g_log_threshold", "g_b_dec"):
        assert _rel(ovf[k], ref[k]) < 2e-3, k


def test_emulated_shards_accumulate_microbatches():
    g = load_golden("ste_f64_accum2")
    cfg = oracle_cfg(g)
    xs = [g[f"x{i}"].astype(np.float32) for i in range(2)]
    x = torch.from_numpy(np.concatenate(xs)).cuda()
    shards, steppers, outs = run_emulated(g, 2, x, cfg, microbatch_tokens=xs[0].shape[0])
    got = gather(shards, steppers)
    p0 = oracle_params(g)
    theta = np.concatenate([kernel_theta(s, xs[-1].shape[0]) for s in steppers])
    ref = O.train_step(xs, p0, O.AdamState.zeros_like(p0), cfg, "bf16", theta=theta)
    for k in O.PARAM_NAMES:
        assert _rel(got["g_" + k], getattr(ref.grads, k)) < BF16_TOL, k


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("exchange", ["nccl", "p2p"])
def test_two_gpu_shards_match_oracle(tmp_path, exchange):
    """Two ranks over NCCL (all-reduce of the partial x_hat) or over the NVLink
    peer exchange (peer loads of the partials, peer stores of go)."""
    env = dict(os.environ)
    env["NCCL_NVLS_ENABLE"] = "0"
    port = "29517" if exchange == "nccl" else "29518"
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", port,
           str(ROOT / "tests" / "sharded_worker.py"), str(tmp_path), exchange]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    g = load_golden("super_f32_tiles")
    cfg = oracle_cfg(g)
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(2)]
    got = {k: np.concatenate([res[0][k], res[1][k]], axis=1 if k in ("W_dec", "g_W_dec") else 0)
           for k in ("g_W_enc", "g_b_enc", "g_W_dec", "g_log_threshold", "W_enc", "b_enc",
                     "W_dec", "log_threshold", "theta")}
    for k in ("g_b_dec", "b_dec"):
        np.testing.assert_array_equal(res[0][k], res[1][k])
        got[k] = res[0][k]
    p0 = oracle_params(g)
    ref = O.train_step([g["x0"].astype(np.float32)], p0, O.AdamState.zeros_like(p0), cfg,
                       "bf16", theta=got["theta"])
    for k in O.PARAM_NAMES:
        assert _rel(got["g_" + k], getattr(ref.grads, k)) < BF16_TOL, k
        assert np.abs(got[k] - getattr(ref.params, k)).max() <= 2.5 * float(g["lr"]) + 1e-6, k
    stats = [json.loads((tmp_path / f"rank{r}.json").read_text()) for r in range(2)]
    assert stats[0]["l0"] == stats[1]["l0"] and stats[0]["grad_norm"] == stats[1]["grad_norm"]


def test_peer_barrier_gives_up_and_reports_a_timeout():
    """A rank whose peer never arrives: the exchange's flag barrier waits for a
    flag nothing sets, gives up after its bounded wait (2 s), records
    SAE_ERR_DEVICE_TIMEOUT in the device status word and returns; the host
    sees the status, the context stays usable. One GPU: the "peer" is this
    rank's own buffer mapped twice, so no other kernel is waited on."""
    import ctypes
    import math
    import sae_b200
    from sae_b200 import _lib as L
    torch.cuda.synchronize()
    assert L.device_status() == 0
    d, F, B = 128, 256, 256
    sae = sae_b200.make_shard_sae(d, F, 0, 1, seed=1, device="cuda")
    x = sae_b200.superposition_batch(B, d, 512, 8, math.log(8.0), 0.3, seed=3, device="cuda")
    nbytes, ex, fl = ctypes.c_size_t(), ctypes.c_uint64(), ctypes.c_uint64()
    L.call("sae_b200_peer_buffer_bytes", B, d, F, B * 64, ctypes.byref(nbytes), ctypes.byref(ex),
           ctypes.byref(fl))
    own = ctypes.c_void_p()
    handle = (ctypes.c_uint8 * L.PEER_HANDLE_BYTES)()
    L.call("sae_b200_peer_alloc", nbytes.value, ctypes.byref(own), handle)
    try:
        peers = L.Peers()
        peers.rank, peers.world, peers.epoch = 0, 2, 1
        peers.exchange_offset, peers.flags_offset = ex.value, fl.value
        peers.base[0] = own.value
        peers.base[1] = own.value
        cfg = L.StepConfig(B, B * 64, 1e-3, 1e-2, 8.0, 0.2, 1, 0, 1, 0, 0)
        stats = torch.zeros(L.STATS_FLOATS, device="cuda", dtype=torch.int32)
        fired = torch.zeros(F, device="cuda", dtype=torch.uint8)
        model = sae._model_struct(need_shadows=True)
        L.call("sae_b200_shard_forward_p2p", ctypes.byref(model), L.ptr(x), L.DTYPE_BF16,
               ctypes.byref(cfg), ctypes.byref(peers), L.ptr(stats), L.ptr(fired),
               torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert L.device_status() == L.SAE_ERR_DEVICE_TIMEOUT   # read and cleared
        assert L.device_status() == 0
        # the context still works
        y = torch.ones(4, device="cuda") * 2
        assert float(y.sum()) == 8.0
    finally:
        torch.cuda.synchronize()
        L.call("sae_b200_peer_free", own.value)
