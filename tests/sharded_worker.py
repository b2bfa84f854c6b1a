"""One rank of the two-GPU dictionary-sharded parity test (run by torchrun
from test_gpu_sharded.py): trains its shard of the super_f32_tiles golden
case for one step over NCCL and saves its gradients and parameters."""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path[:0] = [str(ROOT), str(ROOT / "event-aware-sae-trainer_b200"), str(ROOT / "tests")]


def main(out_dir, exchange="nccl"):
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    import sae_b200
    from conftest import load_golden
    from sae_b200 import B200Adam, B200JumpReLUSAE, ShardedFusedStep, reference_param_groups
    g = load_golden("super_f32_tiles")
    d, F = int(g["d"]), int(g["F"])
    full = B200JumpReLUSAE(d, F)
    with torch.no_grad():
        full.W_enc.weight.copy_(torch.from_numpy(g["p0_W_enc"]).float())
        full.W_enc.bias.copy_(torch.from_numpy(g["p0_b_enc"]).float())
        full.W_dec.weight.copy_(torch.from_numpy(g["p0_W_dec"]).float())
        full.b_dec.copy_(torch.from_numpy(g["p0_b_dec"]).float())
        full.log_threshold.copy_(torch.from_numpy(g["p0_log_threshold"]).float())
    sae = sae_b200.shard_sae(full, rank, world, device=dev)
    sae.ste_bandwidth = float(g["eps"])
    lr = float(g["lr"])
    opt = B200Adam(reference_param_groups(sae, lr), lr=lr, betas=(0.9, 0.999), sae=sae,
                   renorm=True)
    x = torch.from_numpy(g["x0"].astype(np.float32)).to(dev)
    fs = ShardedFusedStep(sae, opt, max_tokens=x.shape[0], exchange=exchange)
    wf = float(g["wenc_factor"])
    out = fs.step(x, lambda_l0=float(g["lam"]), al_mu=float(g["mu"]), target_l0=float(g["target"]),
                  wenc_dampen=lambda l0: wf)
    torch.cuda.synchronize()
    from sae_b200 import _lib as L
    off = L.workspace_offsets(x.shape[0], d, sae.n_features, fs.csr_capacity)["theta"]
    theta = fs.ws[off:off + 4 * sae.n_features].view(torch.float32).cpu().numpy()
    np.savez(Path(out_dir) / f"rank{rank}.npz",
             g_W_enc=fs.g_W_enc.cpu().numpy(), g_b_enc=fs.g_b_enc.cpu().numpy(),
             g_W_dec=fs.g_W_dec_fm.t().cpu().numpy(), g_log_threshold=fs.g_log_thr.cpu().numpy(),
             g_b_dec=fs.g_b_dec.cpu().numpy(), W_enc=sae.W_enc.weight.detach().cpu().numpy(),
             b_enc=sae.W_enc.bias.detach().cpu().numpy(),
             W_dec=sae.W_dec.weight.detach().cpu().numpy(), b_dec=sae.b_dec.detach().cpu().numpy(),
             log_threshold=sae.log_threshold.detach().cpu().numpy(), theta=theta)
    (Path(out_dir) / f"rank{rank}.json").write_text(json.dumps(out))
    # a second step exercises the flag barriers' epochs and the buffers' reuse
    out2 = fs.step(x, lambda_l0=float(g["lam"]), al_mu=float(g["mu"]),
                   target_l0=float(g["target"]), wenc_dampen=lambda l0: wf)
    assert np.isfinite(out2["loss"])
    fs.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "nccl")
