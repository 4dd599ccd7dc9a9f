"""Seeded config-2 inputs shared by the golden generator and the GPU test.

Config 2 at full vocabulary (V = 151936, bf16): target logits N(0, 3^2) plus a
per-row Zipf(1.1) log-prior over a random vocabulary permutation, draft logits
= target + N(0, 1).  The tensors are regenerated from the seed on the CPU with
torch's generator (too large to commit); the fixture stores a checksum of them
so that a generator change shows up as a clear test failure.
"""
import torch

V_QWEN = 151936


def zipf_logits(gen, n, V, noise=3.0, s=1.1):
    """N(0, noise^2) plus a per-row Zipf(s) log-prior over a random permutation."""
    base = torch.randn(n, V, generator=gen) * noise
    ranks = torch.arange(1, V + 1, dtype=torch.float64)
    prior = (-s * torch.log(ranks)).float()
    out = torch.empty(n, V)
    for r in range(n):
        perm = torch.randperm(V, generator=gen)
        out[r] = base[r] + prior[perm]
    return out


def cfg2_rows(rows=8, k=4, V=V_QWEN, seed=2026, sigma=1.0):
    """bf16-valued float32 target [rows, k+1, V] and draft [rows, k, V] logits."""
    g = torch.Generator().manual_seed(seed)
    tgt = zipf_logits(g, rows * (k + 1), V).reshape(rows, k + 1, V)
    tgt = tgt.to(torch.bfloat16).float()
    drf = (tgt[:, :k] + torch.randn(rows, k, V, generator=g) * sigma).to(torch.bfloat16).float()
    return tgt, drf


def checksum(t):
    """Order-fixed float64 checksum of a tensor (detects generator drift)."""
    x = t.double().flatten()
    w = torch.arange(1, x.numel() + 1, dtype=torch.float64) % 977.0
    return float((x * w).sum())
