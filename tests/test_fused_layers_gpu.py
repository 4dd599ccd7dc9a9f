"""The decoder layers' one-launch RMSNorm and gated MLP against transformers.

sd_rmsnorm follows Qwen3RMSNorm's bf16 sequence with the float32 sum of
squares reduced in another order (a value may move by one bf16 ulp:
ULPS, EXACT_MIN); sd_silu_mul follows act_fn(gate) * up with SiLU.  Installed
on models, the logits stay within bf16 noise of the modules' own forwards, and
greedy speculative decoding through every fused layer still emits exactly
the greedy autoregressive tokens.
"""
import pytest
import torch

from specdec import attention as A
from specdec import fused_layers as FL
from specdec.kvcache import RaggedCache
from tests.tiny_models import VOCAB, TinyTok, tiny_config

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
ULPS = 2
EXACT_MIN = 0.97


def _ulp_check(got, want):
    g, w = got.float(), want.float()
    mag = torch.maximum(w.abs(), g.abs()).clamp_min(2.0 ** -100)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    return bool(((g - w).abs() <= ULPS * ulp).all()), float((g == w).float().mean())


@pytest.mark.parametrize("shape", [(32, 5, 4096), (32, 1, 1024), (3, 7, 32), (2, 3, 5000)])
def test_rmsnorm_matches_transformers(shape):
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm
    g = torch.Generator(device=DEV).manual_seed(0)
    H = shape[-1]
    x = (3 * torch.randn(*shape, generator=g, device=DEV)).to(torch.bfloat16)
    ref = Qwen3RMSNorm(H, eps=1e-6).to(DEV)
    ref.weight.data = (1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    want = ref(x)
    got = FL.rmsnorm(x, ref.weight, 1e-6)
    ok, exact = _ulp_check(got, want)
    assert ok and exact >= EXACT_MIN, (ok, exact)
    # rows H elements apart holding H - 1 (a column slice), and in place
    xs = x[..., 1:]
    w2 = ref.weight[1:].contiguous()
    assert _ulp_check(FL.rmsnorm(xs, w2, 1e-6), _ref_norm(xs, w2, 1e-6))[0]
    y = x.clone()
    FL.rmsnorm(y, ref.weight, 1e-6, out=y)
    assert torch.equal(y, got)


@pytest.mark.parametrize("shape", [(32, 5, 4096), (32, 1, 1024), (2, 3, 8192)])
def test_add_rmsnorm_matches_transformers(shape):
    """residual = residual + h (bf16), then the post-attention norm."""
    g = torch.Generator(device=DEV).manual_seed(2)
    H = shape[-1]
    h = torch.randn(*shape, generator=g, device=DEV).to(torch.bfloat16)
    res = (4 * torch.randn(*shape, generator=g, device=DEV)).to(torch.bfloat16)
    w = (1 + 0.2 * torch.randn(H, generator=g, device=DEV)).to(torch.bfloat16)
    r_got, y_got = FL.add_rmsnorm(h, res, w, 1e-6)
    r_want = res + h
    assert torch.equal(r_got, r_want)
    ok, exact = _ulp_check(y_got, _ref_norm(r_want, w, 1e-6))
    assert ok and exact >= EXACT_MIN, (ok, exact)


def _ref_norm(x, w, eps):
    xf = x.float()
    v = xf.pow(2).mean(-1, keepdim=True)
    return w * (xf * torch.rsqrt(v + eps)).to(torch.bfloat16)


@pytest.mark.parametrize("shape", [(32, 5, 12288), (32, 1, 3072), (3, 7, 64)])
def test_silu_mul_matches_transformers(shape):
    g = torch.Generator(device=DEV).manual_seed(1)
    gu = (2 * torch.randn(*shape[:-1], 2 * shape[-1], generator=g, device=DEV)).to(torch.bfloat16)
    I = shape[-1]
    want = torch.nn.functional.silu(gu[..., :I]) * gu[..., I:]
    got = FL.silu_mul(gu)
    ok, exact = _ulp_check(got, want)
    assert ok and exact >= 0.999, (ok, exact)


def _models(llama):
    torch.manual_seed(0)
    if llama:
        from transformers import LlamaConfig, LlamaForCausalLM
        cfg = LlamaConfig(vocab_size=VOCAB, hidden_size=64, intermediate_size=128,
                          num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                          head_dim=16, max_position_embeddings=256, tie_word_embeddings=True)
        mk = lambda: LlamaForCausalLM(cfg)       # noqa: E731
    else:
        from transformers import Qwen3ForCausalLM
        mk = lambda: Qwen3ForCausalLM(tiny_config(32, 2))     # noqa: E731
    torch.manual_seed(0)
    a = mk().eval().to(DEV, torch.bfloat16)
    torch.manual_seed(0)
    b = mk().eval().to(DEV, torch.bfloat16)
    return a, b


@pytest.mark.parametrize("llama", [False, True])
@torch.inference_mode()
def test_installed_layers_match_module_forwards(llama):
    A.register()
    ref, fused = _models(llama)
    for m in (ref, fused):
        m.set_attn_implementation(A.IMPL)
    n = FL.install(fused)
    assert n == FL.installed_modules(fused) and n >= 2 * 2 + 2 + 1     # norms, MLPs, final norm
    assert FL.install(fused) == 0
    B, P = 3, 9
    ids = torch.randint(0, VOCAB, (B, P), generator=torch.Generator().manual_seed(0)).to(DEV)
    outs = []
    for m in (ref, fused):
        c = RaggedCache(2, B, 64, DEV, attn_impl=A.IMPL)
        q = ids.shape[1]
        outs.append(m(input_ids=ids, position_ids=c.positions(q), attention_mask=None,
                      past_key_values=c, cache_position=c.cache_position(q), use_cache=True).logits)
    torch.testing.assert_close(outs[1].float(), outs[0].float(), atol=3e-2, rtol=3e-2)
    FL.uninstall(fused)
    assert FL.installed_modules(fused) == 0


@torch.inference_mode()
def test_engine_greedy_through_every_fused_layer():
    """Gate G2 with the fused attention, norms and MLPs (the engine's
    defaults) on bf16 models."""
    from specdec.engine import SamplingConfig, SpecDecodeEngine
    from tests.test_fused_attention_gpu import _bf16_tiny
    target, draft = _bf16_tiny(0), _bf16_tiny(5)
    eng = SpecDecodeEngine(target, draft, TinyTok(), device=DEV, capacity=128)
    assert FL.installed_modules(target) > 0 and FL.installed_modules(draft) > 0
    torch.manual_seed(0)
    ids = torch.randint(0, VOCAB, (4, 6))
    plen = torch.tensor([6, 5, 4, 6])
    sp = SamplingConfig(temperature=0.0)
    ar, _ = eng.generate_autoregressive(ids, plen, 24, sampling=sp)
    for k in (1, 3):
        out, _ = eng.generate(ids, plen, 24, sampling=sp, k_fixed=k)
        assert [o[:24] for o in out] == [o[:24] for o in ar], k
