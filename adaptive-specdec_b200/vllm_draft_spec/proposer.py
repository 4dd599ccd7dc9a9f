"""DraftModelProposer for vLLM V1 (0.22): vLLM's draft-model proposer plus the
adaptive-k controller and the B200 draft draw.

Mirrors the reference's proposer (vllm_draft_spec/proposer.py:56-368):

* k is chosen per engine step by a ``specdec.controller`` controller
  (``SPECDEC_CONTROLLER``; "fixed" keeps k = num_speculative_tokens).  The
  controller learns from the previous step's accepted counts and from the
  per-forward draft / target costs measured between consecutive ``propose``
  calls (wall clock: the drafter is launch bound, and reading CUDA events
  would synchronise the pipeline being measured).  num_speculative_tokens
  stays k_max for vLLM's buffers and scheduler lookahead; ``propose`` drafts
  k <= k_max tokens.
* drafting itself (model loading under its own prefix, the shift-by-one
  input layout, the drafting attention metadata, CUDA graphs) is vLLM's.
* with probabilistic draft sampling, ``_sample_from_logits`` runs the
  reference's ``to_probs`` (temperature, top-p, top-k) and an inverse-CDF
  draw on this package's kernels when every request of the batch shares one
  (temperature, top-p, top-k); a mixed batch keeps vLLM's own draw.
"""
import os
import time

import torch

from vllm.logger import init_logger
from vllm.v1.spec_decode.draft_model import DraftModelProposer as _VllmDraftModelProposer

logger = init_logger(__name__)

__all__ = ["DraftModelProposer", "AdaptiveK", "install", "uniform_sampling_params"]


class AdaptiveK:
    """Host-side k selection and its telemetry (no vLLM types involved).

    ``observe_counts`` takes per-request (1 + accepted) counts of the previous
    step (a device tensor read one step late, so the copy never waits on
    running work) with the numbers of tokens that were drafted for them;
    ``enter`` is called at every propose and returns this step's k.
    """

    MAX_PERIOD_S = 1.0        # a longer gap between steps is idle time, not a step

    def __init__(self, k_max, controller=None):
        self.k_max = int(k_max)
        self.k = self.k_max
        self.controller = controller
        self._pending = None          # (counts tensor, drafted list) of the previous step
        self._t_enter = None
        self._t_draft = None
        self._k_prev = None

    def step_costs(self, now):
        """(draft seconds per forward, target seconds per step) or (None, None)."""
        if self._t_enter is None or self._t_draft is None:
            return None, None
        period = now - self._t_enter
        if period <= 0 or period > self.MAX_PERIOD_S:
            return None, None
        return self._t_draft / max(1, self._k_prev or 1), max(1e-5, period - self._t_draft)

    def observe_counts(self, counts, drafted):
        self._pending = (counts, list(drafted))

    def observe_accepted(self, n_acc, now):
        """Accepted counts already on the host (vLLM's non-padded path)."""
        if self.controller is None or not n_acc:
            return
        t_d, t_t = self.step_costs(now)
        self.controller.update(max(1, self.k), list(n_acc), dt=1.0, t_draft_fwd=t_d,
                               t_target_fwd=t_t)

    def enter(self, now):
        t_d, t_t = self.step_costs(now)
        self._t_enter = now
        if self.controller is None:
            self.k = self.k_max
            return self.k
        if self._pending is not None:
            counts, drafted = self._pending
            self._pending = None
            try:
                c = counts.tolist() if torch.is_tensor(counts) else list(counts)
                n_acc = [max(0, int(x) - 1) for x in c[:len(drafted)]]
                if n_acc:
                    self.controller.update(max(1, max(drafted)), n_acc, dt=1.0,
                                           t_draft_fwd=t_d, t_target_fwd=t_t)
            except Exception as e:       # telemetry must never stop serving
                logger.warning("adaptive-specdec: telemetry read failed: %s", e)
        self.k = max(1, min(self.k_max, int(self.controller.propose_k())))
        return self.k

    def leave(self, now, k):
        self._t_draft = now - self._t_enter
        self._k_prev = k


def make_step_controller(k_max, spec=None):
    """The controller named by ``SPECDEC_CONTROLLER`` (None for fixed k)."""
    spec = (spec if spec is not None else os.environ.get("SPECDEC_CONTROLLER", "fixed"))
    spec = spec.strip().lower()
    if spec in ("", "fixed", "none", "off"):
        return None
    from specdec.controller import make_controller
    # vLLM's drafter rides the target's token stream: no commit-only forward
    return make_controller(spec, k_max=k_max, extra_fwd=0)


def uniform_sampling_params(md):
    """(temperature, top_p, top_k) when every request of the batch shares them,
    else None.  Reads the per-request tensors once (one small host copy)."""
    vals = []
    for t, default in ((md.temperature, 1.0), (md.top_p, 1.0), (md.top_k, 0)):
        if t is None:
            vals.append((default, default))
        else:
            vals.append(torch.stack([t.min().float(), t.max().float()]))
    dev = [v for v in vals if torch.is_tensor(v)]
    host = torch.stack(dev).cpu().tolist() if dev else []
    out, i = [], 0
    for v in vals:
        if torch.is_tensor(v):
            lo, hi = host[i]
            i += 1
        else:
            lo, hi = v
        if lo != hi:
            return None
        out.append(lo)
    T, tp, tk = out
    return float(T), float(tp), int(tk)


class DraftModelProposer(_VllmDraftModelProposer):
    """vLLM's DraftModelProposer with adaptive k and the B200 draft draw."""

    def __init__(self, vllm_config, device, runner=None):
        super().__init__(vllm_config, device, runner)
        self.k_max = int(self.num_speculative_tokens)
        ctrl = None
        try:
            ctrl = make_step_controller(self.k_max)
        except Exception as e:
            logger.warning("adaptive-specdec: controller unavailable (%s); fixed k=%d", e,
                           self.k_max)
        self.adaptive = AdaptiveK(self.k_max, ctrl)
        self.b200_sampling = os.environ.get("SPECDEC_B200_SAMPLING", "1").strip() not in (
            "0", "false", "no", "off")
        logger.info("adaptive-specdec: DraftModelProposer k_max=%d controller=%s b200_draw=%s",
                    self.k_max, getattr(ctrl, "name", "fixed"), self.b200_sampling)

    # ---- telemetry hooks (same signatures as the parent) -------------------
    def prepare_inputs_padded(self, common_attn_metadata, spec_decode_metadata,
                              valid_sampled_tokens_count):
        self.adaptive.observe_counts(valid_sampled_tokens_count,
                                     spec_decode_metadata.num_draft_tokens)
        return super().prepare_inputs_padded(common_attn_metadata, spec_decode_metadata,
                                             valid_sampled_tokens_count)

    def prepare_next_token_ids_cpu(self, sampled_token_ids, requests, gpu_input_batch,
                                   num_scheduled_tokens):
        self.adaptive.observe_accepted([max(0, len(s) - 1) for s in sampled_token_ids],
                                       time.perf_counter())
        return super().prepare_next_token_ids_cpu(sampled_token_ids, requests, gpu_input_batch,
                                                  num_scheduled_tokens)

    # ---- drafting ------------------------------------------------------------
    def propose(self, target_token_ids, target_positions, target_hidden_states, next_token_ids,
                token_indices_to_sample, common_attn_metadata, sampling_metadata,
                mm_embed_inputs=None, num_rejected_tokens_gpu=None, slot_mappings=None):
        k = self.adaptive.enter(time.perf_counter())
        self.num_speculative_tokens = k
        try:
            out = super().propose(target_token_ids, target_positions, target_hidden_states,
                                  next_token_ids, token_indices_to_sample, common_attn_metadata,
                                  sampling_metadata, mm_embed_inputs=mm_embed_inputs,
                                  num_rejected_tokens_gpu=num_rejected_tokens_gpu,
                                  slot_mappings=slot_mappings)
        finally:
            self.num_speculative_tokens = self.k_max
        self.adaptive.leave(time.perf_counter(), k)
        return out

    def _sample_from_logits(self, logits, sampling_metadata):
        if (not self.b200_sampling or not self._enable_probabilistic_draft_probs
                or sampling_metadata.all_greedy):
            return super()._sample_from_logits(logits, sampling_metadata)
        params = uniform_sampling_params(sampling_metadata)
        if params is None or params[0] <= 0.0:
            return super()._sample_from_logits(logits, sampling_metadata)
        return b200_draw(logits, *params)


def b200_draw(logits, temperature, top_p, top_k):
    """x ~ to_probs(logits) on the B200 kernels: (ids [B], probs [B, V] fp32)."""
    from specdec import sampling as S
    probs = S.to_probs(logits, temperature, top_p, top_k)
    u = torch.rand(probs.shape[0], device=probs.device)
    return S.sample_from_probs(probs, u=u), probs


def install():
    """Make vLLM's model runner build this proposer for method="draft_model"."""
    import vllm.v1.worker.gpu_model_runner as gmr
    gmr.DraftModelProposer = DraftModelProposer
    logger.info("adaptive-specdec: DraftModelProposer installed")
