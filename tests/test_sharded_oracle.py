"""The dictionary-sharded step's decomposition, on CPU.

The oracle's sharded restatement (three sums over ranks: decoder output and
active counts, the b_dec gradient, the clip sum of squares) must reproduce the
whole-dictionary step. Two and four gloo ranks run it as separate processes;
the sum over ranks is torch.distributed.all_reduce, as on the GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sae_oracle as O


def _case(precision, seed=3, B=48, d=24, F=64, n_micro=2):
    rng = np.random.default_rng(seed)
    x = [O.superposition_batch(B, d, 32, 4, np.log(4.0), 0.3, seed=seed + i) for i in range(n_micro)]
    W = rng.standard_normal((F, d)).astype(np.float32)
    W /= np.linalg.norm(W, axis=1, keepdims=True)
    p = O.Params(W.copy(), 0.01 * rng.standard_normal(F).astype(np.float32), W.T.copy(),
                 np.mean(x[0], 0).astype(np.float32),
                 np.log(np.full(F, 0.35, np.float32)) + 0.1 * rng.standard_normal(F).astype(np.float32))
    if precision == "fp64":
        p = p.astype(np.float64)
        x = [a.astype(np.float64) for a in x]
    cfg = O.StepConfig(lambda_l0=1e-2, al_mu=1e-1, target_l0=3.0, ste_bandwidth=0.3,
                       accum_steps=n_micro, lr=(1e-3,) * 4, wenc_factor=0.7)
    return x, p, cfg


def _compare(full, shards, world, precision):
    tol = 1e-10 if precision == "fp64" else 2e-5
    F = full.params.W_enc.shape[0]
    per = F // world

    def rel(a, b):
        return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))

    for r, res in enumerate(shards):
        s = slice(r * per, (r + 1) * per)
        assert res["l0"] == pytest.approx(full.l0, rel=1e-12)
        assert res["recon"] == pytest.approx(full.recon_loss, rel=tol * 10)
        assert res["grad_norm"] == pytest.approx(full.grad_norm, rel=tol * 10)
        assert rel(res["g_W_enc"], full.grads.W_enc[s]) < tol
        assert rel(res["g_W_dec"], full.grads.W_dec[:, s]) < tol
        assert rel(res["g_b_enc"], full.grads.b_enc[s]) < tol
        assert rel(res["g_log_threshold"], full.grads.log_threshold[s]) < tol
        assert rel(res["g_b_dec"], full.grads.b_dec) < tol
        assert rel(res["W_enc"], full.params.W_enc[s]) < tol
        assert rel(res["W_dec"], full.params.W_dec[:, s]) < tol
        assert rel(res["b_dec"], full.params.b_dec) < tol
        assert rel(res["log_threshold"], full.params.log_threshold[s]) < tol


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, precision, q):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path.insert(0, str(root))
    from oracle import sae_oracle as Ow
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))

    def allreduce(a):
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.float64))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.numpy().astype(np.asarray(a).dtype)

    x, p, cfg = _case(precision)
    mine = Ow.shard_params(p, rank, world)
    st = Ow.AdamState.zeros_like(mine)
    res = Ow.sharded_train_step(x, mine, st, cfg, rank, allreduce, precision)
    q.put((rank, {"l0": res.l0, "recon": res.recon_loss, "grad_norm": res.grad_norm,
                  "g_W_enc": res.grads.W_enc, "g_W_dec": res.grads.W_dec,
                  "g_b_enc": res.grads.b_enc, "g_log_threshold": res.grads.log_threshold,
                  "g_b_dec": res.grads.b_dec, "W_enc": res.params.W_enc,
                  "W_dec": res.params.W_dec, "b_dec": res.params.b_dec,
                  "log_threshold": res.params.log_threshold}))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,precision", [(2, "fp64"), (4, "fp32"), (2, "bf16")])
def test_gloo_ranks_reproduce_the_whole_dictionary_step(world, precision):
    x, p, cfg = _case(precision)
    full = O.train_step(x, p, O.AdamState.zeros_like(p), cfg, precision)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, precision, q))
             for r in range(world)]
    for pr in procs:
        pr.start()
    got = dict(q.get(timeout=180) for _ in procs)
    for pr in procs:
        pr.join(timeout=60)
        assert pr.exitcode == 0
    if precision == "bf16":
        # x_hat = bf16(sum of shard partials): the fp64 partial sums differ from the
        # whole sum in the last bits, which can move a bf16 rounding; everything
        # downstream then differs at the bf16 level at most.
        for r in range(world):
            assert got[r]["l0"] == pytest.approx(full.l0, rel=1e-12)
            assert got[r]["recon"] == pytest.approx(full.recon_loss, rel=1e-3)
        return
    _compare(full, [got[r] for r in range(world)], world, precision)


def test_one_rank_is_the_unsharded_step():
    x, p, cfg = _case("fp64")
    full = O.train_step(x, p, O.AdamState.zeros_like(p), cfg, "fp64")
    one = O.sharded_train_step(x, O.shard_params(p, 0, 1), O.AdamState.zeros_like(p), cfg, 0,
                               lambda a: a, "fp64")
    for k in O.PARAM_NAMES:
        np.testing.assert_allclose(getattr(one.params, k), getattr(full.params, k), rtol=1e-12,
                                   atol=1e-15)
    assert one.grad_norm == pytest.approx(full.grad_norm, rel=1e-12)


def test_shard_ranges_split_evenly_and_reject_ragged():
    import sae_b200
    assert [sae_b200.shard_range(64, r, 4) for r in range(4)] == \
        [slice(0, 16), slice(16, 32), slice(32, 48), slice(48, 64)]
    with pytest.raises(ValueError):
        sae_b200.shard_range(66, 0, 4)
    with pytest.raises(ValueError):
        sae_b200.shard_range(64, 4, 4)
    with pytest.raises(ValueError):
        O.shard_params(_case("fp32")[1], 0, 3)


def test_shard_init_is_the_same_dictionary_for_every_world_size():
    """make_shard_sae draws features in seeded blocks: the shards of any split
    concatenate to the same whole dictionary (so strong-scaling runs at
    1/2/4/8 GPUs train the same SAE)."""
    import torch
    import sae_b200
    d, F = 8, 3 * 4096 + 4096
    whole = sae_b200.make_shard_sae(d, F, 0, 1, seed=7, device="cpu")
    for world in (2, 4, 8):
        parts = [sae_b200.make_shard_sae(d, F, r, world, seed=7, device="cpu") for r in range(world)]
        assert torch.equal(torch.cat([p.W_enc.weight for p in parts]), whole.W_enc.weight)
        assert torch.equal(torch.cat([p.W_dec.weight for p in parts], dim=1), whole.W_dec.weight)
    torch.testing.assert_close(whole.W_dec.weight.norm(dim=0), torch.ones(F))
