"""Host logic of the fused layer installs (no GPU).

specdec.fused_attention.install and specdec.fused_layers.install rewrite a
model's modules in place: the q / k / v (and gate / up) weights become views
of one concatenated tensor and the forwards are replaced.  On CPU tensors
every replaced forward must fall through to the module's own code, so a
model with the installs gives bit-identical logits; the views must hold the
original weights; install is idempotent and uninstall restores the forwards.
"""
import torch

from specdec import fused_attention as FA
from specdec import fused_layers as FL
from tests.tiny_models import VOCAB, tiny_config


def _pair(seed=0):
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(seed)
    a = Qwen3ForCausalLM(tiny_config(32, 2)).eval()
    torch.manual_seed(seed)
    b = Qwen3ForCausalLM(tiny_config(32, 2)).eval()
    return a, b


@torch.inference_mode()
def test_installs_keep_weights_and_cpu_logits():
    ref, m = _pair()
    assert FA.install(m) == 2 and FA.install(m) == 0
    n = FL.install(m)
    assert n == FL.installed_modules(m) and FL.install(m) == 0
    # 2 decoder layers + 4 norms each (input, post, q, k) + 2 MLPs + the final norm
    assert n == 2 + 8 + 2 + 1
    for lr, lm in zip(ref.model.layers, m.model.layers):
        a = lm.self_attn
        nq, nk = a.q_proj.weight.shape[0], a.k_proj.weight.shape[0]
        assert torch.equal(a._sd_qkv_w[:nq], lr.self_attn.q_proj.weight)
        assert torch.equal(a._sd_qkv_w[nq + nk:], lr.self_attn.v_proj.weight)
        assert a.q_proj.weight.data_ptr() == a._sd_qkv_w.data_ptr()      # a view, no copy
        ni = lm.mlp.gate_proj.weight.shape[0]
        assert torch.equal(lm.mlp._sd_gu_w[ni:], lr.mlp.up_proj.weight)
        assert lm.mlp.up_proj.weight.data_ptr() == lm.mlp._sd_gu_w[ni:].data_ptr()
    ids = torch.randint(0, VOCAB, (2, 7), generator=torch.Generator().manual_seed(0))
    assert torch.equal(m(input_ids=ids).logits, ref(input_ids=ids).logits)
    FA.uninstall(m)
    FL.uninstall(m)
    assert FA.installed_layers(m) == 0 and FL.installed_modules(m) == 0
    assert torch.equal(m(input_ids=ids).logits, ref(input_ids=ids).logits)


def test_install_skips_modules_it_cannot_fuse():
    """A q_norm without a k_norm, or an MLP whose activation is not SiLU,
    keeps its own forward."""
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(vocab_size=VOCAB, hidden_size=32, intermediate_size=64,
                      num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=8, hidden_act="gelu", max_position_embeddings=64)
    m = LlamaForCausalLM(cfg).eval()
    assert FA.install(m) == 1                       # Llama attention: no norms, fused
    n = FL.install(m)
    assert n == 1 + 2 + 1                           # the layer, its two norms, the final norm
    assert not hasattr(m.model.layers[0].mlp, "_sd_gu_w")
