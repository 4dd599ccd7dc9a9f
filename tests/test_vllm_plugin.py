"""The vLLM plugin surface (``vllm_draft_spec``), after the reference's
tests/test_vllm_patches.py: the proposer subclasses vLLM's draft-model
proposer with the parent's method signatures, registration is opt-in, the
adaptive-k telemetry behaves, and (GPU) the draft draw on the kernels samples
from the probabilities it hands to the rejection sampler.
"""
import inspect
import os
import types

import numpy as np
import pytest
import torch

vllm = pytest.importorskip("vllm")

from vllm_draft_spec import proposer as PR  # noqa: E402


def test_subclasses_vllm_draft_model_proposer_with_parent_signatures():
    from vllm.v1.spec_decode.draft_model import DraftModelProposer as Parent
    assert issubclass(PR.DraftModelProposer, Parent)
    for m in ("__init__", "propose", "load_model", "dummy_run", "prepare_inputs_padded",
              "prepare_next_token_ids_cpu", "_sample_from_logits"):
        a = list(inspect.signature(getattr(PR.DraftModelProposer, m)).parameters)
        b = list(inspect.signature(getattr(Parent, m)).parameters)
        assert a == b, (m, a, b)


def test_register_is_opt_in(monkeypatch):
    import vllm_draft_spec
    monkeypatch.delenv("SPECDEC_PLUGIN", raising=False)
    assert vllm_draft_spec.register() is False
    gmr = pytest.importorskip("vllm.v1.worker.gpu_model_runner")
    orig = gmr.DraftModelProposer
    try:
        monkeypatch.setenv("SPECDEC_PLUGIN", "1")
        assert vllm_draft_spec.register() is True
        assert gmr.DraftModelProposer is PR.DraftModelProposer
    finally:
        gmr.DraftModelProposer = orig


def test_fixed_k_without_a_controller():
    ak = PR.AdaptiveK(6, None)
    for step in range(3):
        assert ak.enter(10.0 + step) == 6
        ak.leave(10.0 + step + 0.01, 6)


def test_controller_follows_acceptance():
    ctrl = PR.make_step_controller(8, "ewma")
    ak = PR.AdaptiveK(8, ctrl)
    t = 100.0
    k = ak.enter(t)
    # every drafted token accepted, cheap draft steps: k grows to the cap
    for _ in range(40):
        ak.leave(t + 0.002 * k, k)
        ak.observe_counts(torch.full((16,), k + 1), [k] * 16)
        t += 0.05
        k = ak.enter(t)
    assert k >= 6
    # nothing accepted: k falls to 1
    for _ in range(60):
        ak.leave(t + 0.002 * k, k)
        ak.observe_counts(torch.ones(16), [k] * 16)
        t += 0.05
        k = ak.enter(t)
    assert k <= 2


def test_step_costs_ignore_idle_gaps():
    ak = PR.AdaptiveK(4, None)
    ak.enter(1.0)
    ak.leave(1.004, 4)
    d, tt = ak.step_costs(1.020)
    assert d == pytest.approx(0.001) and tt == pytest.approx(0.016)
    assert ak.step_costs(5.0) == (None, None)           # an idle gap, not a step


def test_uniform_sampling_params():
    md = types.SimpleNamespace(temperature=torch.full((4,), 0.7), top_p=torch.full((4,), 0.9),
                               top_k=None)
    T, tp, tk = PR.uniform_sampling_params(md)
    assert T == pytest.approx(0.7) and tp == pytest.approx(0.9) and tk == 0
    md.top_p = torch.tensor([0.9, 0.9, 0.8, 0.9])
    assert PR.uniform_sampling_params(md) is None
    md = types.SimpleNamespace(temperature=None, top_p=None, top_k=torch.full((3,), 20))
    assert PR.uniform_sampling_params(md) == (1.0, 1.0, 20)


@pytest.mark.gpu
def test_b200_draw_samples_from_the_probabilities_it_returns():
    from oracle import sampling_oracle as O
    g = torch.Generator(device="cuda").manual_seed(0)
    V, n = 64, 20000
    row = (torch.randn(V, generator=g, device="cuda") * 2).to(torch.bfloat16)
    logits = row.expand(n, V).contiguous()
    ids, probs = PR.b200_draw(logits, 0.8, 0.9, 0)
    ref = O.to_probs(row.float().cpu().numpy()[None], 0.8, 0.9)[0]
    np.testing.assert_allclose(probs[0].cpu().numpy(), ref, rtol=2e-6, atol=1e-30)
    assert bool((probs[torch.arange(n, device="cuda"), ids] > 0).all())
    hist = torch.bincount(ids, minlength=V).double().cpu().numpy() / n
    assert 0.5 * np.abs(hist - ref).sum() < 0.02
