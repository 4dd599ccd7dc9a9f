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
from vllm_draft_spec import rejection as RJ  # noqa: E402


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
    orig, orig_rs = gmr.DraftModelProposer, gmr.RejectionSampler
    try:
        monkeypatch.setenv("SPECDEC_PLUGIN", "1")
        assert vllm_draft_spec.register() is True
        assert gmr.DraftModelProposer is PR.DraftModelProposer
        assert gmr.RejectionSampler is RJ.B200RejectionSampler
        gmr.RejectionSampler = orig_rs
        monkeypatch.setenv("SPECDEC_B200_REJECTION", "0")      # vLLM's rejection sampler kept
        assert vllm_draft_spec.register() is True
        assert gmr.RejectionSampler is orig_rs
    finally:
        gmr.DraftModelProposer, gmr.RejectionSampler = orig, orig_rs


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


# ---------------------------------------------------------------------------
# the rejection sampler on the fused kernel
# ---------------------------------------------------------------------------
def test_rejection_sampler_subclasses_vllm_with_parent_signature():
    from vllm.v1.sample.rejection_sampler import RejectionSampler as Parent
    assert issubclass(RJ.B200RejectionSampler, Parent)
    for m in ("__init__", "forward"):
        a = list(inspect.signature(getattr(RJ.B200RejectionSampler, m)).parameters)
        b = list(inspect.signature(getattr(Parent, m)).parameters)
        assert a == b, (m, a, b)


def _sampling_md(B, T=0.7, tp=0.9, tk=None, device="cpu", **over):
    from vllm.v1.sample.logits_processor import LogitsProcessors
    md = dict(temperature=None if T == 0 else torch.full((B,), T, device=device),
              all_greedy=T == 0, all_random=T > 0,
              top_p=None if tp is None else torch.full((B,), tp, device=device),
              top_k=None if tk is None else torch.full((B,), tk, device=device),
              generators={}, max_num_logprobs=None, no_penalties=True,
              allowed_token_ids_mask=None, bad_words_token_ids={},
              logitsprocs=LogitsProcessors(), thinking_budget_state_holder=None)
    md.update(over)
    return types.SimpleNamespace(**md)


def _spec_md(counts, V, device="cpu", seed=0):
    from vllm.v1.spec_decode.metadata import SpecDecodeMetadata
    g = torch.Generator().manual_seed(seed)
    ids = [torch.randint(0, V, (n,), generator=g).tolist() for n in counts]
    return SpecDecodeMetadata.make_dummy(ids, torch.device(device))


def test_b200_plan_takes_uniform_batches_only():
    B, k, V = 4, 3, 4096
    md = _spec_md([k] * B, V)
    logits = torch.zeros(B * (k + 1), V, dtype=torch.bfloat16)
    q = torch.full((B * k, V), 1.0 / V)
    plan = RJ.b200_plan(md, q, logits, _sampling_md(B))
    assert plan[:2] == (B, k) and plan[2][0] == pytest.approx(0.7) and plan[2][2] == 0
    assert RJ.b200_plan(md, None, logits, _sampling_md(B, T=0)) == (B, k, (0.0, 1.0, 0))
    # each of these keeps vLLM's own path
    ragged = _spec_md([k, k, k - 1, k], V)
    assert RJ.b200_plan(ragged, q[:-1], logits[:-1], _sampling_md(B)) is None
    assert RJ.b200_plan(md, q, logits, _sampling_md(B, max_num_logprobs=0)) is None
    assert RJ.b200_plan(md, q, logits, _sampling_md(B, generators={1: torch.Generator()})) is None
    assert RJ.b200_plan(md, q, logits, _sampling_md(B, no_penalties=False)) is None
    assert RJ.b200_plan(md, q, logits, _sampling_md(B, all_random=False)) is None     # mixed
    assert RJ.b200_plan(md, None, logits, _sampling_md(B)) is None          # no draft probs
    assert RJ.b200_plan(md, q, logits.float(), _sampling_md(B)) is None     # fp32 logits
    assert RJ.b200_plan(md, q, logits, _sampling_md(B), synthetic_mode=True) is None
    mixed = _sampling_md(B)
    mixed.top_p = torch.tensor([0.9, 0.9, 0.8, 0.9])
    assert RJ.b200_plan(md, q, logits, mixed) is None
    small = torch.zeros(B * (k + 1), 1024, dtype=torch.bfloat16)
    assert RJ.b200_plan(md, torch.full((B * k, 1024), 1.0 / 1024), small, _sampling_md(B)) is None
    busy = _sampling_md(B)
    busy.logitsprocs.non_argmax_invariant.append(types.SimpleNamespace(min_toks={0: (5, [], set())}))
    assert RJ.b200_plan(md, q, logits, busy) is None


def _make_sampler():
    from vllm.v1.sample.sampler import Sampler
    return RJ.B200RejectionSampler(Sampler(), None, torch.device("cuda"))


@pytest.mark.gpu
@pytest.mark.parametrize("T,tp,tk", [(0.7, 0.9, None), (1.0, 1.0, 40), (0.0, None, None)])
def test_rejection_sampler_forward_runs_the_fused_round(T, tp, tk):
    """forward on a uniform batch: the emitted tokens are the accepted draft
    prefix, then the kernel's residual / bonus token, then -1; the same as a
    direct verify_sample_probs call with the same uniforms."""
    from specdec import sampling as S, workloads as W
    B, k, V = 16, 4, 32000
    g = torch.Generator().manual_seed(3)
    tgt = W.zipf_logits(B * (k + 1), V, g).to("cuda", torch.bfloat16)
    drf = (tgt.view(B, k + 1, V)[:, :k].float() + torch.randn(B, k, V, generator=g).cuda())
    q = S.to_probs(drf.to(torch.bfloat16), T, tp or 1.0, tk or 0).reshape(B * k, V) if T > 0 else None
    am = tgt.float().view(B, k + 1, V).argmax(-1)
    draft = torch.where(torch.rand(B, k, generator=g).cuda() < 0.6, am[:, :k],
                        torch.randint(0, V, (B, k), generator=g).cuda())
    md = _spec_md([k] * B, V, device="cuda")
    md.draft_token_ids = draft.reshape(-1).to(torch.int32).contiguous()
    smd = _sampling_md(B, T=T, tp=tp, tk=tk, device="cuda")
    rs = _make_sampler()
    ua = torch.rand(B, k, generator=g).cuda() if T > 0 else torch.zeros(B, k, device="cuda")
    ur = torch.rand(B, generator=g).cuda() if T > 0 else torch.zeros(B, device="cuda")
    rs.uniforms = lambda *a: (ua, ur)
    out = rs.forward(md, q, tgt, smd).sampled_token_ids
    assert rs.calls == {"b200": 1, "vllm": 0}
    assert out.shape == (B, k + 1) and out.dtype == torch.int32
    plan = RJ.b200_plan(md, q, tgt, smd)
    n, y = S.verify_sample_probs(tgt.view(B, k + 1, V), None if q is None else q.view(B, k, V),
                                 draft, ua, ur, T, tp or 1.0, tk or 0)
    assert plan is not None
    for b in range(B):
        nb = int(n[b])
        row = out[b].tolist()
        assert row[:nb] == draft[b, :nb].tolist()
        assert row[nb] == int(y[b])
        assert all(t == -1 for t in row[nb + 1:])
    if T == 0:                        # greedy: accepted while the draft is the argmax
        match = (draft == am[:, :k]).int()
        want = torch.where(match.all(-1), torch.full_like(n, k), (1 - match).argmax(-1).long())
        assert torch.equal(n, want)
