"""vLLM plugin surface of the B200 build: ``DraftModelProposer``.

The reference ships an out-of-tree vLLM plugin (vllm_draft_spec/__init__.py,
proposer.py, patches.py) whose proposer drafts with a separate draft model,
chooses k per step with the adaptive controller, and registers through the
``vllm.general_plugins`` entry point, opt-in with ``SPECDEC_PLUGIN=1``.  The
vLLM installed beside this package (0.22) supports ``method="draft_model"``
itself, so none of the reference's config patches are needed; what this
package adds on top of vLLM's own draft-model proposer is:

* the adaptive-k controller (``SPECDEC_CONTROLLER=ewma|ewma+exit|ucb|fixed``),
  fed with the accepted counts and the measured draft / target step costs;
* the verify round on this package's fused kernel: ``B200RejectionSampler``
  replaces vLLM's rejection sampler (``SPECDEC_B200_REJECTION=0`` keeps
  vLLM's) and runs the accept test and the residual / bonus draw of a uniform
  batch in one call, from vLLM's draft probabilities;
* the draft draw on this package's kernels when vLLM samples drafts
  probabilistically (``draft_sample_method="probabilistic"``): the draft
  distribution is the reference's full ``to_probs`` (temperature, top-p,
  top-k; vLLM's own path applies the temperature only) and the token is an
  inverse-CDF draw from it, so the probabilities handed to vLLM's rejection
  sampler are exactly the ones the token was drawn from.

Usage:
    SPECDEC_PLUGIN=1 SPECDEC_CONTROLLER=ewma vllm serve Qwen/Qwen3-8B \\
      --speculative-config '{"model": "Qwen/Qwen3-0.6B", "method": "draft_model",
                             "num_speculative_tokens": 8}'
"""

__all__ = ["register"]


def register():
    """Entry point for ``vllm.general_plugins``.  Opt-in: nothing happens
    unless ``SPECDEC_PLUGIN`` is set, so installing the package changes no
    other vLLM job in the same environment (the reference's rule)."""
    import os
    if os.environ.get("SPECDEC_PLUGIN", "").strip().lower() not in ("1", "true", "yes", "on"):
        return False
    from vllm_draft_spec import proposer, rejection
    proposer.install()
    if os.environ.get("SPECDEC_B200_REJECTION", "1").strip().lower() not in ("0", "false", "no",
                                                                           "off"):
        rejection.install()
    return True
