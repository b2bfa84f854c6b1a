"""The HBM-resident activation pool (host logic on CPU): the reference's shard
format in, every shard once per epoch in a seeded shuffled order, resumable."""
import pytest
import torch


def _write_pool(tmp_path, n=5, seqs=3, seq_len=8, d=16):
    shards = []
    for i in range(n):
        t = (torch.arange(seqs * seq_len * d, dtype=torch.float32).reshape(seqs, seq_len, d)
             + 1000 * i).to(torch.bfloat16)
        torch.save(t, tmp_path / f"shard_{i:05d}.pt")
        shards.append(t)
    return shards


def test_pool_reads_reference_shards_and_covers_each_once_per_epoch(tmp_path):
    from sae_b200 import DeviceActivationPool
    shards = _write_pool(tmp_path)
    pool = DeviceActivationPool.from_dir(tmp_path, device="cpu", seed=3)
    assert pool.d_in == 16 and pool.tokens == 5 * 24
    for epoch in range(3):
        got = [pool.next_batch() for _ in range(5)]
        firsts = sorted(int(b[0, 0].float()) // 1000 for b in got)
        assert firsts == list(range(5))          # every shard once per epoch
        assert all(b.shape == (24, 16) and b.dtype == torch.bfloat16 for b in got)
    torch.testing.assert_close(
        DeviceActivationPool.from_dir(tmp_path, "cpu", seed=3).shards[2], shards[2].reshape(-1, 16))


def test_pool_order_is_seeded_and_resumable(tmp_path):
    from sae_b200 import DeviceActivationPool
    _write_pool(tmp_path)
    a = DeviceActivationPool.from_dir(tmp_path, "cpu", seed=7)
    seq_a = [int(a.next_batch()[0, 0].float()) for _ in range(7)]
    state = a.get_state()
    after = [int(a.next_batch()[0, 0].float()) for _ in range(6)]
    b = DeviceActivationPool.from_dir(tmp_path, "cpu", seed=7)
    assert [int(b.next_batch()[0, 0].float()) for _ in range(7)] == seq_a
    c = DeviceActivationPool.from_dir(tmp_path, "cpu", seed=7)
    c.restore_state(state)
    assert [int(c.next_batch()[0, 0].float()) for _ in range(6)] == after
    d = DeviceActivationPool.from_dir(tmp_path, "cpu", seed=8)
    assert [int(d.next_batch()[0, 0].float()) for _ in range(7)] != seq_a


@pytest.mark.gpu
def test_device_pool_feeds_the_fused_step(tmp_path):
    """Batches handed out by the HBM pool drive the fused step exactly like the
    same activations copied in from the host."""
    from sae_b200 import B200Adam, DeviceActivationPool, FusedStep, make_sae, reference_param_groups
    d, F, seqs, seq_len = 256, 2048, 8, 128
    gen = torch.Generator().manual_seed(1)
    for i in range(3):
        torch.save((4 * torch.randn(seqs, seq_len, d, generator=gen)).to(torch.bfloat16),
                   tmp_path / f"shard_{i:05d}.pt")
    pool = DeviceActivationPool.from_dir(tmp_path, "cuda", seed=0)
    assert all(s.is_cuda for s in pool.shards)

    def run(batches):
        sae = make_sae(d, F, seed=0).cuda()
        opt = B200Adam(reference_param_groups(sae, 1e-4), lr=1e-4, sae=sae)
        fs = FusedStep(sae, opt, max_tokens=seqs * seq_len)
        out = [fs.step(b, lambda_l0=1e-3, al_mu=1e-2, target_l0=50.0) for b in batches]
        torch.cuda.synchronize()
        return out, sae.W_enc.weight.detach().clone()

    batches = [pool.next_batch() for _ in range(3)]
    host = [b.cpu().pin_memory().cuda(non_blocking=True) for b in batches]
    a, wa = run(batches)
    b, wb = run(host)
    assert a == b
    assert torch.equal(wa, wb)
