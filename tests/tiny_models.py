"""Tiny random Qwen3 pairs for the engine gates (the reference's tests/tiny.py scale).

V=16 keeps the statistical test's sampling noise (~sqrt(V / 2 pi N)) well under
its gate.  The noisy pair perturbs a copy of the target so greedy decoding
actually exercises rejections.
"""
import copy

import torch
from transformers import Qwen3Config, Qwen3ForCausalLM

VOCAB = 16


def tiny_config(hidden=32, layers=2):
    return Qwen3Config(vocab_size=VOCAB, hidden_size=hidden, intermediate_size=2 * hidden,
                       num_hidden_layers=layers, num_attention_heads=4, num_key_value_heads=2,
                       head_dim=8, max_position_embeddings=256, tie_word_embeddings=True)


def tiny_pair(device="cuda", seed_target=0, seed_draft=1):
    """Target and draft of different depth and width."""
    torch.manual_seed(seed_target)
    target = Qwen3ForCausalLM(tiny_config(32, 2)).eval()
    torch.manual_seed(seed_draft)
    draft = Qwen3ForCausalLM(tiny_config(16, 1)).eval()
    return target.to(device), draft.to(device)


def tiny_pair_noisy(noise=0.35, seed=0, device="cuda"):
    """Draft = target + gaussian noise scaled by each parameter's spread."""
    torch.manual_seed(seed)
    target = Qwen3ForCausalLM(tiny_config(32, 2)).eval()
    draft = copy.deepcopy(target).eval()
    g = torch.Generator().manual_seed(seed + 1)
    with torch.no_grad():
        for prm in draft.parameters():
            prm.add_(torch.randn(prm.shape, generator=g) * noise * prm.std().clamp_min(1e-3))
    return target.to(device), draft.to(device)


class TinyTok:
    eos_token_id = None
