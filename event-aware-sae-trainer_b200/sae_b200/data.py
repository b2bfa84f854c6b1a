"""Synthetic residual-stream activations for the benchmark configurations.

No activation corpus or LLM is available offline, so every benchmark uses
seeded superposition data with the shapes and value distributions of the
configurations: each token is the sum of ``k_active`` distinct unit directions
of a fixed Gaussian dictionary (``n_dirs x d``, rows normalised) with
Exponential(1) magnitudes, plus N(0, noise^2) noise, rescaled to a
LogNormal(norm_mu, norm_sigma) norm. The dictionary uses seed ``seed``, the
tokens ``seed + 1``.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def superposition_batch(n_tokens: int, d: int, n_dirs: int, k_active: int, norm_mu: float,
                        norm_sigma: float, seed: int, *, device="cuda", noise: float = 0.05,
                        dtype=torch.bfloat16, chunk: int = 4096) -> torch.Tensor:
    dev = torch.device(device)
    g = torch.Generator(device=dev).manual_seed(int(seed))
    D = torch.randn(n_dirs, d, generator=g, device=dev)
    D /= D.norm(dim=1, keepdim=True).clamp(min=1e-8)
    g.manual_seed(int(seed) + 1)
    out = torch.empty(n_tokens, d, device=dev, dtype=dtype)
    for s in range(0, n_tokens, chunk):
        n = min(chunk, n_tokens - s)
        # k distinct directions per token: top-k of uniform keys.
        keys = torch.rand(n, n_dirs, generator=g, device=dev)
        idx = keys.topk(k_active, dim=1).indices
        coef = torch.empty(n, k_active, device=dev).exponential_(1.0, generator=g)
        x = torch.einsum("tk,tkd->td", coef, D[idx])
        x += noise * torch.randn(n, d, generator=g, device=dev)
        norms = torch.exp(norm_mu + norm_sigma * torch.randn(n, generator=g, device=dev))
        x *= (norms / x.norm(dim=1).clamp(min=1e-8)).unsqueeze(1)
        out[s:s + n] = x.to(dtype)
    return out
