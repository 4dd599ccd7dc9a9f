"""vLLM's rejection sampler on the fused B200 verify kernel.

vLLM 0.22's ``RejectionSampler.forward`` (vllm/v1/sample/rejection_sampler.py:87)
takes, per engine step, the target logits of every request's draft positions
and bonus position ([num_tokens + batch, V], one block of k + 1 rows per
request), the draft probabilities its drafter drew from ([num_tokens, V] fp32)
and the batch's sampling metadata, and returns the emitted tokens per request
([batch, k + 1], -1 after the first rejection).  ``B200RejectionSampler`` keeps
that contract.  For a batch the fused kernel covers, one call of
``specdec.sampling.verify_sample_probs`` does what the reference's engine does
in engine.py:282-303 and vLLM spreads over several kernels: to_probs on the
target logits (temperature, top-p, top-k), the accept test
u < min(1, p(x)/q(x)) with vLLM's own uniforms, and the residual draw from
norm((p - q)+) at the first rejection or the bonus draw from p_k.  Any other
batch runs vLLM's own path unchanged:

* requests with different numbers of draft tokens, or different
  (temperature, top-p, top-k);
* logprobs requested, seeded requests (per-request generators), penalties,
  bad words, allowed-token masks, active min-tokens, thinking budgets, or the
  synthetic acceptance mode;
* sampling without draft probabilities (an argmax or n-gram drafter);
* fp32 target logits, or sampling with V <= 2048 (the kernel's list path
  takes bf16 / fp16 logits of larger vocabularies).

Semantics: p is the reference's to_probs (its top-p boundary and tie rule),
which is what the drafts' probabilities come from when this package's
``DraftModelProposer`` draws them; vLLM's own path applies its top-k / top-p
masks instead.  The bonus token is drawn from p_k by the kernel rather than by
vLLM's sampler, from the same distribution.
"""
import os

import torch

from vllm.logger import init_logger
from vllm.v1.outputs import SamplerOutput
from vllm.v1.sample.rejection_sampler import RejectionSampler as _VllmRejectionSampler
from vllm.v1.sample.rejection_sampler import generate_uniform_probs

logger = init_logger(__name__)

__all__ = ["B200RejectionSampler", "b200_plan", "install"]

SMALL_V = 2048           # the kernel's sampling path needs V > SMALL_V (list kernels)
K_MAX = 64


def _active_min_tokens(sampling_metadata):
    procs = getattr(getattr(sampling_metadata, "logitsprocs", None), "non_argmax_invariant", ())
    return any(getattr(p, "min_toks", None) for p in procs or ())


def b200_plan(metadata, draft_probs, logits, sampling_metadata, synthetic_mode=False):
    """(B, k, (temperature, top_p, top_k)) when the fused kernel covers this
    batch, else None (vLLM's own path).  Reads host-side metadata only, plus
    one small host copy for the sampling parameters (as vLLM's sampler does)."""
    from vllm_draft_spec.proposer import uniform_sampling_params
    md = sampling_metadata
    if synthetic_mode or md.max_num_logprobs is not None or md.generators:
        return None
    if not md.no_penalties or md.allowed_token_ids_mask is not None or md.bad_words_token_ids:
        return None
    holder = getattr(md, "thinking_budget_state_holder", None)
    if holder is not None and holder.has_tracked_requests():
        return None
    if _active_min_tokens(md):
        return None
    counts = metadata.num_draft_tokens
    B = len(counts)
    if B == 0 or len(set(counts)) != 1:
        return None
    k = counts[0]
    if not 1 <= k <= K_MAX:
        return None
    if logits.dim() != 2 or logits.shape[0] != B * (k + 1) or logits.stride(-1) != 1:
        return None
    if logits.dtype not in (torch.bfloat16, torch.float16):
        return None
    if md.all_greedy:
        params = (0.0, 1.0, 0)          # vLLM may leave the temperature tensor unset here
    elif not md.all_random:
        return None                     # greedy and random requests mixed
    else:
        params = uniform_sampling_params(md)
        if params is None or params[0] <= 0.0:
            return None
    V = logits.shape[1]
    if params[0] > 0.0:
        if draft_probs is None or draft_probs.dtype != torch.float32:
            return None
        if tuple(draft_probs.shape) != (B * k, V) or V <= SMALL_V:
            return None
    return B, k, params


def b200_verify(metadata, draft_probs, logits, plan, u_acc, u_res):
    """The fused round for a planned batch: (output token ids [B, k + 1] int32
    with -1 after each request's emitted token, n_acc [B], y [B])."""
    from specdec import sampling as S
    B, k, (T, tp, tk) = plan
    V = logits.shape[1]
    tgt = logits.view(B, k + 1, V)              # one block of k + 1 rows per request
    xs = metadata.draft_token_ids.view(B, k)
    q = draft_probs.view(B, k, V) if T > 0.0 else None
    n_acc, y = S.verify_sample_probs(tgt, q, xs, u_acc, u_res, T, tp, tk)
    pos = torch.arange(k + 1, device=logits.device)[None, :]
    xs_pad = torch.cat([xs.long(), torch.zeros_like(y)[:, None]], dim=1)
    out = torch.where(pos < n_acc[:, None], xs_pad,
                      torch.where(pos == n_acc[:, None], y[:, None], torch.full_like(y[:, None], -1)))
    return out.to(torch.int32), n_acc, y


class B200RejectionSampler(_VllmRejectionSampler):
    """vLLM's RejectionSampler with the fused B200 verify round for the
    batches it covers (module docstring); ``SPECDEC_B200_REJECTION=0`` turns it
    off.  ``calls`` counts the steps taken by each path."""

    def __init__(self, sampler, spec_config=None, device=None):
        super().__init__(sampler, spec_config, device)
        self.b200 = os.environ.get("SPECDEC_B200_REJECTION", "1").strip().lower() not in (
            "0", "false", "no", "off")
        self.calls = {"b200": 0, "vllm": 0}

    def uniforms(self, metadata, sampling_metadata, B, k, device):
        """u_acc [B, k] from vLLM's own generator of acceptance uniforms (float64,
        rounded to float32 and kept below 1, so that p >= q still accepts), and
        one uniform per request for the residual / bonus draw.  A greedy batch
        draws none: its test is x_i == argmax p_i."""
        if sampling_metadata.all_greedy:
            return (torch.zeros(B, k, device=device), torch.zeros(B, device=device))
        u = generate_uniform_probs(B * k, metadata.num_draft_tokens, sampling_metadata.generators,
                                   device)
        u = u.view(B, k).to(torch.float32).clamp_(max=1.0 - 2.0 ** -24)
        return u, torch.rand(B, device=device)

    def forward(self, metadata, draft_probs, logits, sampling_metadata):
        plan = None
        if self.b200:
            plan = b200_plan(metadata, draft_probs, logits, sampling_metadata,
                             self.synthetic_mode)
        if plan is None:
            self.calls["vllm"] += 1
            return super().forward(metadata, draft_probs, logits, sampling_metadata)
        self.calls["b200"] += 1
        B, k, _ = plan
        u_acc, u_res = self.uniforms(metadata, sampling_metadata, B, k, logits.device)
        out, _, _ = b200_verify(metadata, draft_probs, logits, plan, u_acc, u_res)
        return SamplerOutput(sampled_token_ids=out, logprobs_tensors=None)


def install():
    """Make vLLM's model runner build this rejection sampler."""
    import vllm.v1.worker.gpu_model_runner as gmr
    gmr.RejectionSampler = B200RejectionSampler
    logger.info("adaptive-specdec: B200RejectionSampler installed")
