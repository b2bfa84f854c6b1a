"""The allocation-free straight-through backward, sae_b200_jumprelu_backward_static.

Some callers of this library cannot give it a workspace: a host framework whose
caching allocator already holds the GPU's memory (an extra cudaMalloc would fail
or fragment it), or a latency-critical caller that must not make the implicitly
synchronising cudaMalloc / cudaFree calls. For them the static variant keeps its
scratch -- the per-slab partial sums of the threshold gradient -- in a fixed
4 MiB array inside the library and allocates nothing.

These tests call it through the C ABI and compare it with the workspace entry
point, sae_b200_jumprelu_backward, on two calls in a row: the second call runs
on the array exactly as the first call left it. The file is named so that
pytest collects it last.
"""
import pytest
import torch


def _lib():
    from sae_b200 import _lib as L
    L.load()
    return L


def _inputs(n_tokens, n_features, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    pre = (torch.randn(n_tokens, n_features, device="cuda", generator=g) * 0.6 + 0.3)
    pre = pre.to(torch.bfloat16)
    log_thr = torch.log(torch.rand(n_features, device="cuda", generator=g) * 0.5 + 0.2)
    gf = torch.randn(n_tokens, n_features, device="cuda", generator=g) * 1e-3
    gg = torch.full((n_tokens, n_features), 3e-4, device="cuda")
    return pre, log_thr, gf, gg


def _run(L, static, pre, log_thr, gf, gg, eps=0.2):
    n, F = pre.shape
    grad_pre = torch.zeros_like(pre)
    g_lt = torch.zeros(F, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    if static:
        L.call("sae_b200_jumprelu_backward_static", pre.data_ptr(), L.DTYPE_BF16,
               log_thr.data_ptr(), n, F, gf.data_ptr(), gg.data_ptr(), eps, grad_pre.data_ptr(),
               g_lt.data_ptr(), stream)
    else:
        ws = torch.empty(((n + 255) // 256) * F, device="cuda")
        L.call("sae_b200_jumprelu_backward", pre.data_ptr(), L.DTYPE_BF16, log_thr.data_ptr(),
               n, F, gf.data_ptr(), gg.data_ptr(), eps, grad_pre.data_ptr(), g_lt.data_ptr(),
               ws.data_ptr(), ws.numel() * 4, stream)
    return grad_pre, g_lt


@pytest.mark.gpu
def test_static_scratch_matches_workspace_entry_point_twice():
    L = _lib()
    # Two calls in a row; the second is smaller (3 slabs x 384 features cover
    # fewer slots than the first call's 12 x 1024), so it runs over partial
    # sums the first call left in the shared array. Both entry points run the
    # same two kernels in the same order, so every output must match bit for
    # bit: a stale partial sum would show up as a difference.
    for n, F, seed in ((3000, 1024, 1), (700, 384, 2)):
        pre, log_thr, gf, gg = _inputs(n, F, seed)
        got_pre, got_lt = _run(L, True, pre, log_thr, gf, gg)
        ref_pre, ref_lt = _run(L, False, pre, log_thr, gf, gg)
        torch.cuda.synchronize()
        assert L.device_status() == 0
        assert torch.equal(got_pre, ref_pre)
        assert ref_lt.abs().max() > 0
        assert torch.equal(got_lt, ref_lt)


def test_static_scratch_rejects_oversize_without_touching_the_device():
    """ceil(n/256) * F above the fixed capacity is refused before any CUDA call."""
    L = _lib()
    n, F = 256 * 512, 4096            # 512 slabs x 4096 features = 2 Mi partial sums
    assert ((n + 255) // 256) * F > L.JUMPRELU_BWD_STATIC_FLOATS
    fake = 1 << 20                    # never dereferenced: the size check comes first
    with pytest.raises(L.SaeB200Error) as err:
        L.call("sae_b200_jumprelu_backward_static", fake, L.DTYPE_BF16, fake, n, F, fake, fake,
               0.2, fake, fake, None)
    assert err.value.code == L.SAE_ERR_UNSUPPORTED_SHAPE
    assert "at most" in str(err.value)


@pytest.mark.parametrize("static", [True, False])
def test_more_token_slabs_than_grid_rows_are_refused(static):
    """A small dictionary with a huge token count fits the static array
    (65536 slabs x 8 features) but not CUDA's 65535 grid rows: both entry
    points refuse it with SAE_ERR_UNSUPPORTED_SHAPE before any CUDA call."""
    L = _lib()
    n, F = 65536 * 256, 8
    assert ((n + 255) // 256) * F <= L.JUMPRELU_BWD_STATIC_FLOATS
    fake = 1 << 20
    with pytest.raises(L.SaeB200Error) as err:
        if static:
            L.call("sae_b200_jumprelu_backward_static", fake, L.DTYPE_BF16, fake, n, F, fake,
                   fake, 0.2, fake, fake, None)
        else:
            L.call("sae_b200_jumprelu_backward", fake, L.DTYPE_BF16, fake, n, F, fake, fake, 0.2,
                   fake, fake, fake, 1 << 40, None)
    assert err.value.code == L.SAE_ERR_UNSUPPORTED_SHAPE
    assert "slabs" in str(err.value)
