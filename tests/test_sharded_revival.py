"""Revival writes on a dictionary split over ranks, on CPU.

``sae_b200.revival`` restates the reference's threshold reset (3107-3118,
_revive_log_threshold 209-225) and resample (resample_dead_neurons 2784-2810,
then 3151-3158) so that a sharded dictionary ends up holding exactly what the
unsharded writes produce. Checked here:
  * one rank against a restatement of the reference's own lines, bit for bit
    (same torch RNG draws in the same order);
  * two gloo ranks, each holding half of the dictionary, against the unsharded
    result, bit for bit: the random draws are made once on rank 0 and
    broadcast, the live median and the mean living row norm are taken over
    the gathered values.
The module's parameters live on the CPU here: the revival writes are plain
tensor writes (no library call), so the decomposition is tested where gloo
runs.
"""
import copy
import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

D, F, WORLD = 16, 64, 2
SEED = 7


def _build():
    """A module with non-trivial weights and a populated Adam state."""
    from sae_b200 import make_sae, reference_param_groups
    sae = make_sae(D, F, seed=3)
    g = torch.Generator().manual_seed(11)
    with torch.no_grad():
        sae.W_enc.weight.mul_(1.0 + torch.rand(F, 1, generator=g))
        sae.W_enc.bias.copy_(0.1 * torch.randn(F, generator=g))
        sae.log_threshold.copy_(math.log(0.1) + 0.3 * torch.randn(F, generator=g))
    opt = torch.optim.Adam(reference_param_groups(sae, 1e-3), lr=1e-3)
    for p in sae.parameters():
        p.grad = torch.randn(p.shape, generator=g)
    opt.step()
    dead = torch.zeros(F, dtype=torch.bool)
    dead[[1, 5, 6, 20, 33, 34, 40, 63]] = True          # on both halves
    cand = torch.randn(48, D, generator=g)
    return sae, opt, dead, cand


def _reference_resample(sae, optimizer, dead_mask, candidates):
    """The reference's lines (2784-2810 then 3151-3158), on the whole dictionary."""
    n_dead = int(dead_mask.sum().item())
    with torch.no_grad():
        idx = torch.randint(0, candidates.shape[0], (n_dead,), device=candidates.device)
        samples = candidates[idx]
        norms = samples.norm(dim=-1, keepdim=True).clamp(min=1e-8)
        alive_mask = ~dead_mask
        alive_norm = sae.W_enc.weight[alive_mask].norm(dim=1).mean()
        rows = ((samples / norms) * 1.0 * alive_norm).to(sae.W_enc.weight.dtype)
        sae.W_enc.weight.data[dead_mask] = rows
        sae.W_enc.bias.data[dead_mask] = 0.0
        rand_dec = torch.randn(sae.d_in, n_dead, dtype=sae.W_dec.weight.dtype)
        rand_dec = rand_dec / rand_dec.norm(dim=0, keepdim=True).clamp(min=1e-8)
        sae.W_dec.weight.data[:, dead_mask] = rand_dec
        for group in optimizer.param_groups:
            for p in group["params"]:
                state = optimizer.state.get(p, {})
                if p is sae.W_enc.weight or p is sae.W_enc.bias:
                    state["exp_avg"][dead_mask] = 0.0
                    state["exp_avg_sq"][dead_mask] = 0.0
                elif p is sae.W_dec.weight:
                    state["exp_avg"][:, dead_mask] = 0.0
                    state["exp_avg_sq"][:, dead_mask] = 0.0
        rev = sae.log_threshold.data[~dead_mask].median()
        sae.log_threshold.data[dead_mask] = rev
        st = optimizer.state[sae.log_threshold]
        st["exp_avg"][dead_mask] = 0.0
        st["exp_avg_sq"][dead_mask] = 0.0


def _snapshot(sae, opt):
    params = (sae.W_enc.weight, sae.W_enc.bias, sae.W_dec.weight, sae.b_dec, sae.log_threshold)
    out = {}
    for name, p in zip(("W_enc", "b_enc", "W_dec", "b_dec", "log_threshold"), params):
        out[name] = p.detach().clone()
        st = opt.state[p]
        out[name + ".m"] = st["exp_avg"].clone()
        out[name + ".v"] = st["exp_avg_sq"].clone()
    return out


def test_one_rank_matches_the_reference_lines_bit_for_bit():
    from sae_b200 import revival
    sae, opt, dead, cand = _build()
    ref_sae, ref_opt = copy.deepcopy((sae, opt))
    torch.manual_seed(SEED)
    _reference_resample(ref_sae, ref_opt, dead, cand)
    torch.manual_seed(SEED)
    assert revival.resample(sae, opt, dead, cand) == int(dead.sum())
    got, want = _snapshot(sae, opt), _snapshot(ref_sae, ref_opt)
    for k in want:
        assert torch.equal(got[k], want[k]), k


def test_threshold_reset_one_rank():
    from sae_b200 import revival
    sae, opt, dead, _ = _build()
    before = sae.log_threshold.detach().clone()
    assert revival.threshold_reset(sae, opt, dead) == int(dead.sum())
    assert torch.equal(sae.log_threshold[dead], before[~dead].median().expand(int(dead.sum())))
    assert torch.equal(sae.log_threshold[~dead], before[~dead])
    assert not opt.state[sae.log_threshold]["exp_avg"][dead].any()
    assert revival.threshold_reset(sae, opt, torch.zeros(F, dtype=torch.bool)) == 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shard_optimizer(full_opt, full, shard, rank, world):
    from sae_b200 import reference_param_groups, shard_range
    s = shard_range(F, rank, world)
    opt = torch.optim.Adam(reference_param_groups(shard, 1e-3), lr=1e-3)
    pairs = ((full.W_enc.weight, shard.W_enc.weight, s, False),
             (full.W_enc.bias, shard.W_enc.bias, s, False),
             (full.W_dec.weight, shard.W_dec.weight, s, True),
             (full.b_dec, shard.b_dec, None, False),
             (full.log_threshold, shard.log_threshold, s, False))
    for fp, sp, sl, cols in pairs:
        st = full_opt.state[fp]
        pick = (lambda t: t.clone()) if sl is None else \
            ((lambda t: t[:, sl].clone()) if cols else (lambda t: t[sl].clone()))
        opt.state[sp] = {"step": st["step"].clone(), "exp_avg": pick(st["exp_avg"]),
                         "exp_avg_sq": pick(st["exp_avg_sq"])}
    return opt


def _worker(rank, world, port, q):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "event-aware-sae-trainer_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    from sae_b200 import revival, shard_range, shard_sae
    full, full_opt, dead, cand = _build()
    s = shard_range(F, rank, world)
    comm = revival.DistComm()
    # threshold reset on a fresh copy, then the resample
    sh = shard_sae(full, rank, world)
    opt = _shard_optimizer(full_opt, full, sh, rank, world)
    n_reset = revival.threshold_reset(sh, opt, dead[s], comm)
    reset = sh.log_threshold.detach().clone()
    sh = shard_sae(full, rank, world)
    opt = _shard_optimizer(full_opt, full, sh, rank, world)
    torch.manual_seed(SEED + 100 * rank)      # only rank 0's draws may matter
    if rank == 0:
        torch.manual_seed(SEED)
    n = revival.resample(sh, opt, dead[s], cand, comm)
    # numpy copies: tensors sent through a spawn queue refer to the sender's
    # shared memory, which is gone once the worker exits
    q.put((rank, n_reset, n, reset.numpy(), {k: v.numpy() for k, v in _snapshot(sh, opt).items()}))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_shards_match_the_unsharded_writes_bit_for_bit():
    sae, opt, dead, cand = _build()
    rsae, ropt = copy.deepcopy((sae, opt))
    before = sae.log_threshold.detach().clone()
    torch.manual_seed(SEED)
    _reference_resample(rsae, ropt, dead, cand)
    want = _snapshot(rsae, ropt)

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=180) for _ in procs), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] == int(dead.sum()) and r[2] == int(dead.sum()) for r in res)
    # threshold reset: the global live median on every shard's dead features
    reset = torch.cat([torch.from_numpy(r[3]) for r in res])
    assert torch.equal(reset[dead], before[~dead].median().expand(int(dead.sum())))
    assert torch.equal(reset[~dead], before[~dead])
    # resample: concatenated shards == the unsharded writes
    shards = [{k: torch.from_numpy(v) for k, v in r[4].items()} for r in res]
    for k, v in want.items():
        if k.startswith("b_dec"):
            for sh in shards:
                assert torch.equal(sh[k], v), k
            continue
        dim = 1 if k.startswith("W_dec") else 0
        assert torch.equal(torch.cat([sh[k] for sh in shards], dim=dim), v), k
