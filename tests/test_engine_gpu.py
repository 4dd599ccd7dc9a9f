"""Engine gates on the kernels (tiny models on the GPU).

G2 (the reference's tests/test_greedy_equivalence.py): greedy speculative
decoding is token-for-token identical to greedy autoregressive decoding, for
every k, for the adaptive controllers, for batch 1 vs batch 4 and for a draft
of a different architecture -- and the rejection path is exercised.

G1 part B (the reference's tests/test_rejection_sampling.py:185-230): the full
engine with k=4, T=1, top-p 0.9 produces a second token whose histogram matches
the exactly enumerated autoregressive marginal within TV 0.02.  The marginal
is computed with the CPU oracle's to_probs from the target's logits.
"""
import numpy as np
import pytest
import torch

from oracle import sampling_oracle as O
from specdec.controller import make_controller
from specdec.engine import SamplingConfig, SpecDecodeEngine
from tests.tiny_models import VOCAB, TinyTok, tiny_pair, tiny_pair_noisy

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
G1_TV_MAX = 0.02


@pytest.fixture(scope="module")
def noisy_engine():
    target, draft = tiny_pair_noisy(noise=4.0)
    return SpecDecodeEngine(target, draft, TinyTok(), device=DEV, capacity=128)


def _prompts():
    torch.manual_seed(0)
    B, P = 4, 6
    ids = torch.randint(0, VOCAB, (B, P))
    plen = torch.tensor([P, P - 1, P - 2, P])
    return ids, plen


@pytest.mark.parametrize("k", [1, 2, 3, 4, 6, 8])
def test_greedy_identical_to_autoregressive(noisy_engine, k):
    ids, plen = _prompts()
    NEW = 24
    sp = SamplingConfig(temperature=0.0)
    ar, _ = noisy_engine.generate_autoregressive(ids, plen, NEW, sampling=sp)
    out, st = noisy_engine.generate(ids, plen, NEW, sampling=sp, k_fixed=k)
    assert [o[:NEW] for o in out] == [o[:NEW] for o in ar], f"k={k} alpha={st.alpha_conditional}"


@pytest.mark.parametrize("spec", ["ewma", "ewma+exit", "ucb"])
def test_greedy_identical_with_controllers(noisy_engine, spec):
    ids, plen = _prompts()
    NEW = 24
    sp = SamplingConfig(temperature=0.0)
    ar, _ = noisy_engine.generate_autoregressive(ids, plen, NEW, sampling=sp)
    out, st = noisy_engine.generate(ids, plen, NEW, sampling=sp,
                                    controller=make_controller(spec, k_max=8, tau=0.5))
    assert [o[:NEW] for o in out] == [o[:NEW] for o in ar], spec


def test_batch_of_one_and_mismatched_draft(noisy_engine):
    ids, plen = _prompts()
    NEW = 24
    sp = SamplingConfig(temperature=0.0)
    ar, _ = noisy_engine.generate_autoregressive(ids, plen, NEW, sampling=sp)
    out1, _ = noisy_engine.generate(ids[:1], plen[:1], NEW, sampling=sp, k_fixed=5)
    assert out1[0][:NEW] == ar[0][:NEW]
    t2, d2 = tiny_pair()
    eng2 = SpecDecodeEngine(t2, d2, TinyTok(), device=DEV, capacity=128)
    ar2, _ = eng2.generate_autoregressive(ids, plen, NEW, sampling=sp)
    sd2, _ = eng2.generate(ids, plen, NEW, sampling=sp, k_fixed=4)
    assert [o[:NEW] for o in sd2] == [o[:NEW] for o in ar2]


def test_rejection_path_exercised(noisy_engine):
    ids, plen = _prompts()
    _, st = noisy_engine.generate(ids, plen, 24, sampling=SamplingConfig(temperature=0.0),
                                  k_fixed=8)
    assert st.alpha_conditional < 0.99
    assert st.rounds > 0 and st.emitted >= 4 * 24


@torch.inference_mode()
def test_engine_is_distributionally_lossless():
    target, draft = tiny_pair()
    eng = SpecDecodeEngine(target, draft, TinyTok(), device=DEV, capacity=64)
    sp = SamplingConfig(temperature=1.0, top_p=0.9)
    torch.manual_seed(0)
    prompt = torch.randint(0, VOCAB, (1, 5))
    lg0 = target(input_ids=prompt.to(DEV)).logits[0, -1].float().cpu().numpy()
    p0 = O.to_probs_row(lg0, 1.0, 0.9)
    marg = np.zeros(VOCAB)
    for t0 in range(VOCAB):
        if p0[t0] <= 0:
            continue
        seq = torch.cat([prompt[0], torch.tensor([t0])]).unsqueeze(0).to(DEV)
        l1 = target(input_ids=seq).logits[0, -1].float().cpu().numpy()
        marg += p0[t0] * O.to_probs_row(l1, 1.0, 0.9)
    B, REPS = 2048, 40
    ids = prompt.expand(B, -1).contiguous()
    plen = torch.full((B,), prompt.shape[1], dtype=torch.long)
    first, second, alphas = [], [], []
    for r in range(REPS):
        out, st = eng.generate(ids, plen, max_new_tokens=2, sampling=sp, k_fixed=4,
                               seed=1000 + r)
        first += [o[0] for o in out]
        second += [o[1] for o in out]
        alphas.append(st.alpha_conditional)
    e0 = np.bincount(first, minlength=VOCAB) / len(first)
    e1 = np.bincount(second, minlength=VOCAB) / len(second)
    tv0 = 0.5 * np.abs(e0 - p0).sum()
    tv1 = 0.5 * np.abs(e1 - marg).sum()
    assert tv0 < G1_TV_MAX, tv0
    assert tv1 < G1_TV_MAX, f"TV={tv1:.4f} mean alpha={np.mean(alphas):.3f}"
