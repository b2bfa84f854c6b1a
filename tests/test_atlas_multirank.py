"""Multi-rank host logic of the layer atlas, on CPU with two gloo ranks."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def test_round_robin_placement_covers_every_layer_once():
    from sae_b200.atlas import ideal_speedup, layers_for_rank
    for world in (1, 2, 4, 8):
        seen = sorted(sum((layers_for_rank(35, world, r) for r in range(world)), []))
        assert seen == list(range(35))
    assert layers_for_rank(35, 8, 3) == [3, 11, 19, 27]
    assert ideal_speedup(35, 8) == pytest.approx(7.0)   # 35 layers, at most 5 per GPU
    with pytest.raises(ValueError):
        layers_for_rank(35, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out):
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parents[1] / "event-aware-sae-trainer_b200"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    from sae_b200.atlas import layers_for_rank, max_over_ranks, sum_over_ranks
    mine = layers_for_rank(35, world, rank)
    slowest = max_over_ranks(10.0 + rank)
    total = sum_over_ranks(len(mine))
    out.put((rank, mine, slowest, total))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_reduce_timing_and_counts():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][1] == list(range(0, 35, 2)) and res[1][1] == list(range(1, 35, 2))
    assert all(r[2] == 11.0 for r in res)     # max over ranks
    assert all(r[3] == 35 for r in res)       # every layer counted once
