"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no dataset or checkpoint is involved).

Config 2 (Qwen3 vocabulary): target logits N(0, 3^2) plus a per-row Zipf(1.1)
log-prior added over a random vocabulary permutation, so distributions are
peaked; draft logits = target + N(0, sigma^2) with sigma set for an acceptance
rate near 0.6 at T=0.7, top-p 0.9 (DRAFT_SIGMA, calibrated with the oracle).
"""
import torch

QWEN_VOCAB = 151936
DRAFT_SIGMA = 1.0      # E[sum_j min(p_j, q_j)] = 0.60 at T=0.7, top-p 0.9, V=151936


def zipf_logits(rows, V, generator, device="cpu", noise=3.0, s=1.1):
    """[rows, V] float32: N(0, noise^2) + (-s * log rank) over a random permutation."""
    base = torch.randn(rows, V, generator=generator, device=device) * noise
    prior = -s * torch.log(torch.arange(1, V + 1, device=device, dtype=torch.float64)).float()
    for r in range(rows):
        perm = torch.randperm(V, generator=generator, device=device)
        base[r].index_add_(0, perm, prior)
    return base


def cfg2_logits(B=64, k=4, V=QWEN_VOCAB, sigma=DRAFT_SIGMA, seed=0, device="cuda",
                dtype=torch.bfloat16):
    """Target [B, k+1, V] and draft [B, k, V] logits for config 2."""
    g = torch.Generator(device=device).manual_seed(seed)
    tgt = zipf_logits(B * (k + 1), V, g, device).reshape(B, k + 1, V)
    drf = tgt[:, :k] + torch.randn(B, k, V, generator=g, device=device) * sigma
    return tgt.to(dtype), drf.to(dtype)


def uniforms(B, k, seed=0, device="cuda"):
    g = torch.Generator(device=device).manual_seed(seed + 12345)
    return (torch.rand(B, k, generator=g, device=device),
            torch.rand(B, generator=g, device=device))


def attn_lengths(B=64, lo=512, hi=8192, seed=0):
    """Config 3 context lengths, uniform in [lo, hi]."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (B,), generator=g)


def rope_cos_sin(positions, head_dim, theta=1e6):
    """cos/sin [*, head_dim] for RoPE (rotate-half convention, as Qwen3)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64,
                                        device=positions.device) / head_dim))
    f = positions.double()[..., None] * inv
    emb = torch.cat([f, f], dim=-1)
    return emb.cos().float(), emb.sin().float()


def expected_acceptance(p, q):
    """E[min(1, p/q)] under x ~ q = sum_j min(p_j, q_j)."""
    return float(torch.minimum(p, q).sum(-1).mean())


def bytes_per_verify(B, k, V, elt=2, greedy=False):
    """Algorithmic HBM bytes of one verify call: every logits element read once."""
    n = B * (k + 1) if greedy else B * (2 * k + 1)
    return n * V * elt

