"""The fused QK-norm + RoPE + KV-append step against transformers' own ops.

sd_qkv_norm_rope_append replaces, per attention layer, Qwen3RMSNorm on the q
and k heads, apply_rotary_pos_emb and the cache update of the reference's
_RaggedLayer.update (specdec/kvcache.py:61-74).  Without the norms (Llama /
Qwen2 layers) the arithmetic is the same bf16 operations in the same order,
so the outputs must be bit-identical; with the norms the float32 sum of
squares is reduced in another order, which may move a value by one bf16 ulp
(NORM_ULPS), and almost every element must still match exactly
(NORM_EXACT_MIN).
"""
import pytest
import torch

from specdec import attention as A
from specdec import fused_attention as FA
from specdec.kvcache import RaggedCache
from tests.tiny_models import VOCAB, TinyTok, tiny_config

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
NORM_ULPS = 2               # |fused - transformers| <= 2 bf16 ulps of the larger term
NORM_EXACT_MIN = 0.97       # share of elements that match bit for bit


def _rope_tables(B, Lq, D, pos0, theta=1e6):
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    cfg = Qwen3Config(head_dim=D, hidden_size=D * 4, num_attention_heads=4, rope_theta=theta,
                      max_position_embeddings=1 << 16)
    rot = Qwen3RotaryEmbedding(cfg).to(DEV)
    pos = pos0[:, None] + torch.arange(Lq, device=DEV)[None, :]
    x = torch.empty(1, dtype=torch.bfloat16, device=DEV)
    return rot(x, pos)


def _reference(q, k, v, qw, kw, eps, cos, sin, kc, vc, lens, D):
    """transformers' ops: Qwen3RMSNorm per head, apply_rotary_pos_emb, then
    the cache write at each row's offset."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
    B, Lq, _ = q.shape
    qs = q.view(B, Lq, -1, D)
    ks = k.view(B, Lq, -1, D)
    if qw is not None:
        nq, nk = Qwen3RMSNorm(D, eps).to(DEV), Qwen3RMSNorm(D, eps).to(DEV)
        nq.weight.data, nk.weight.data = qw.clone(), kw.clone()
        qs, ks = nq(qs), nk(ks)
    qs, ks = qs.transpose(1, 2), ks.transpose(1, 2)
    vs = v.view(B, Lq, -1, D).transpose(1, 2)
    qe, ke = apply_rotary_pos_emb(qs, ks, cos, sin)
    kc, vc = kc.clone(), vc.clone()
    for b in range(B):
        s = int(lens[b])
        kc[b, :, s:s + Lq] = ke[b]
        vc[b, :, s:s + Lq] = vs[b]
    return qe.contiguous(), kc, vc


def _close_in_ulps(got, want, ulps):
    g, w = got.float(), want.float()
    mag = torch.maximum(w.abs(), g.abs()).clamp_min(2.0 ** -100)
    ulp = torch.exp2(torch.floor(torch.log2(mag)) - 7)
    return bool(((g - w).abs() <= ulps * ulp).all()), float((g == w).float().mean())


def _inputs(B, Lq, Hq, Hkv, D, C, lens, seed, norm=True, fused_rows=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    bf = torch.bfloat16
    if fused_rows:                     # q, k, v as column slices of one QKV GEMM output
        qkv = torch.randn(B, Lq, (Hq + 2 * Hkv) * D, generator=g, device=DEV).to(bf)
        q, k, v = qkv[..., :Hq * D], qkv[..., Hq * D:(Hq + Hkv) * D], qkv[..., (Hq + Hkv) * D:]
    else:
        q = torch.randn(B, Lq, Hq * D, generator=g, device=DEV).to(bf)
        k = torch.randn(B, Lq, Hkv * D, generator=g, device=DEV).to(bf)
        v = torch.randn(B, Lq, Hkv * D, generator=g, device=DEV).to(bf)
    qw = (1 + 0.3 * torch.randn(D, generator=g, device=DEV)).to(bf) if norm else None
    kw = (1 + 0.3 * torch.randn(D, generator=g, device=DEV)).to(bf) if norm else None
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(bf)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(bf)
    lens = torch.tensor(lens, dtype=torch.long, device=DEV)
    cos, sin = _rope_tables(B, Lq, D, lens)
    return q, k, v, qw, kw, cos, sin, kc, vc, lens


@pytest.mark.parametrize("shape", [
    # B, L, Hq, Hkv, D, C, lengths
    (4, 5, 32, 8, 128, 64, [0, 17, 40, 59]),        # Qwen3-8B heads, k = 4 verify forward
    (3, 1, 16, 8, 128, 32, [3, 0, 31]),             # Qwen3-0.6B heads, one draft step
    (2, 7, 4, 2, 8, 16, [9, 2]),                    # the tiny test models
    (2, 3, 6, 2, 256, 8, [1, 5]),                   # largest head dimension
    (1, 70, 8, 2, 64, 80, [0]),                     # prefill-sized
])
@pytest.mark.parametrize("fused_rows", [False, True])
def test_qk_norm_rope_append_matches_transformers(shape, fused_rows):
    B, Lq, Hq, Hkv, D, C, lens = shape
    eps = 1e-6
    q, k, v, qw, kw, cos, sin, kc, vc, lens = _inputs(B, Lq, Hq, Hkv, D, C, lens, 1,
                                                     fused_rows=fused_rows)
    want_q, want_k, want_v = _reference(q, k, v, qw, kw, eps, cos, sin, kc, vc, lens, D)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got_q = FA.qkv_norm_rope_append(q, k, v, qw, kw, eps, cos, sin, kc, vc, lens, D, err=err)
    torch.cuda.synchronize()
    assert int(err) == 0
    assert torch.equal(vc, want_v)                  # v is a copy
    for got, want in ((got_q, want_q), (kc, want_k)):
        ok, exact = _close_in_ulps(got, want, NORM_ULPS)
        assert ok and exact >= NORM_EXACT_MIN, (ok, exact)


@pytest.mark.parametrize("shape", [(4, 5, 32, 8, 128, 64, [0, 17, 40, 59]),
                                   (2, 7, 4, 2, 8, 16, [9, 2])])
def test_rope_append_without_norm_is_bit_exact(shape):
    B, Lq, Hq, Hkv, D, C, lens = shape
    q, k, v, _, _, cos, sin, kc, vc, lens = _inputs(B, Lq, Hq, Hkv, D, C, lens, 2, norm=False)
    want_q, want_k, want_v = _reference(q, k, v, None, None, 0.0, cos, sin, kc, vc, lens, D)
    got_q = FA.qkv_norm_rope_append(q, k, v, None, None, 0.0, cos, sin, kc, vc, lens, D)
    torch.cuda.synchronize()
    assert torch.equal(got_q, want_q)
    assert torch.equal(kc, want_k)
    assert torch.equal(vc, want_v)


def test_rows_past_capacity_set_the_flag_and_write_nothing():
    B, Lq, Hq, Hkv, D, C = 3, 4, 4, 2, 16, 10
    q, k, v, qw, kw, cos, sin, kc, vc, lens = _inputs(B, Lq, Hq, Hkv, D, C, [2, 7, 6], 3)
    want_q, want_k, want_v = _reference(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc,
                                        torch.tensor([2, 0, 6]), D)
    kc0, vc0 = kc.clone(), vc.clone()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got_q = FA.qkv_norm_rope_append(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc, lens, D, err=err)
    torch.cuda.synchronize()
    assert int(err) == 1                              # row 1: 7 + 4 > 10
    assert torch.equal(kc[1], kc0[1]) and torch.equal(vc[1], vc0[1])
    for b in (0, 2):
        assert _close_in_ulps(kc[b], want_k[b], NORM_ULPS)[0]
        assert torch.equal(vc[b], want_v[b])
    assert _close_in_ulps(got_q, want_q, NORM_ULPS)[0]   # q is written for every row


def test_argument_checks():
    q, k, v, qw, kw, cos, sin, kc, vc, lens = _inputs(2, 3, 4, 2, 8, 16, [0, 1], 4)
    with pytest.raises(Exception):
        FA.qkv_norm_rope_append(q, k, v, qw, None, 1e-6, cos, sin, kc, vc, lens, 8)
    with pytest.raises(Exception):
        FA.qkv_norm_rope_append(q.float(), k, v, qw, kw, 1e-6, cos, sin, kc, vc, lens, 8)
    with pytest.raises(Exception):
        FA.qkv_norm_rope_append(q, k[:, :2], v, qw, kw, 1e-6, cos, sin, kc, vc, lens, 8)


# ---------------------------------------------------------------------------
# installed on a model: the same logits and cache as the layers' own forward
# ---------------------------------------------------------------------------
def _bf16_tiny(seed, llama=False):
    torch.manual_seed(seed)
    if llama:
        from transformers import LlamaConfig, LlamaForCausalLM
        cfg = LlamaConfig(vocab_size=VOCAB, hidden_size=64, intermediate_size=128,
                          num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                          head_dim=16, max_position_embeddings=256, tie_word_embeddings=True)
        m = LlamaForCausalLM(cfg)
    else:
        from transformers import Qwen3ForCausalLM
        m = Qwen3ForCausalLM(tiny_config(32, 2))
    return m.eval().to(DEV, torch.bfloat16)


def _fwd(m, cache, tokens, valid=None):
    q = tokens.shape[1]
    return m(input_ids=tokens, position_ids=cache.positions(q),
             attention_mask=cache.attn_mask(q, torch.bfloat16, valid=valid),
             past_key_values=cache, cache_position=cache.cache_position(q), use_cache=True).logits


@pytest.mark.parametrize("llama", [False, True])
@torch.inference_mode()
def test_installed_forward_matches_layer_forward(llama):
    A.register()
    ref, fused = _bf16_tiny(0, llama), _bf16_tiny(0, llama)
    for m in (ref, fused):
        m.set_attn_implementation(A.IMPL)
    assert FA.install(fused) == 2 and FA.install(fused) == 0
    B, P = 3, 9
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, VOCAB, (B, P), generator=g).to(DEV)
    plen = torch.tensor([9, 6, 7], device=DEV)
    caches = [RaggedCache(2, B, 64, DEV, attn_impl=A.IMPL) for _ in range(2)]
    outs = []
    for m, c in zip((ref, fused), caches):
        lg = [_fwd(m, c, ids, valid=plen)]
        c.set_lengths(plen.cpu())
        spec = torch.randint(0, VOCAB, (B, 5), generator=torch.Generator().manual_seed(1)).to(DEV)
        lg.append(_fwd(m, c, spec))
        c.advance(5)
        c.rollback([2, 0, 4])
        lg.append(_fwd(m, c, spec[:, :1]))
        outs.append(lg)
    for a, b in zip(*outs):
        torch.testing.assert_close(b.float(), a.float(), atol=3e-2, rtol=3e-2)
    for la, lb in zip(caches[0].layers, caches[1].layers):
        for b in range(B):
            n = int(caches[0].lengths[b]) + 1
            torch.testing.assert_close(lb.keys[b, :, :n].float(), la.keys[b, :, :n].float(),
                                       atol=3e-2, rtol=3e-2)
            torch.testing.assert_close(lb.values[b, :, :n].float(), la.values[b, :, :n].float(),
                                       atol=3e-2, rtol=3e-2)
    assert int(caches[1]._err) == 0


@torch.inference_mode()
def test_installed_forward_leaves_other_calls_alone():
    """fp32 models and calls without a RaggedCache go through the layer's own
    forward, bit for bit."""
    A.register()
    from transformers import Qwen3ForCausalLM
    torch.manual_seed(0)
    ref = Qwen3ForCausalLM(tiny_config(32, 2)).eval().to(DEV)
    torch.manual_seed(0)
    fused = Qwen3ForCausalLM(tiny_config(32, 2)).eval().to(DEV)
    FA.install(fused)
    ids = torch.randint(0, VOCAB, (2, 6), generator=torch.Generator().manual_seed(0)).to(DEV)
    assert torch.equal(fused(input_ids=ids).logits, ref(input_ids=ids).logits)
    for m in (ref, fused):
        m.set_attn_implementation(A.IMPL)
    outs = []
    for m in (ref, fused):
        c = RaggedCache(2, 2, 32, DEV, attn_impl=A.IMPL)
        outs.append(_fwd(m, c, ids))
    assert torch.equal(outs[0], outs[1])
    FA.uninstall(fused)
    assert FA.installed_layers(fused) == 0


@torch.inference_mode()
def test_engine_greedy_with_fused_layers_matches_autoregressive():
    """Gate G2 on bf16 models with the fused layers: greedy speculative
    decoding emits exactly the tokens of greedy autoregressive decoding
    through the same layers."""
    from specdec.engine import SamplingConfig, SpecDecodeEngine
    target, draft = _bf16_tiny(0), _bf16_tiny(5)
    eng = SpecDecodeEngine(target, draft, TinyTok(), device=DEV, capacity=128, fused_qkv=True)
    assert FA.installed_layers(target) == 2 and FA.installed_layers(draft) == 2
    torch.manual_seed(0)
    ids = torch.randint(0, VOCAB, (4, 6))
    plen = torch.tensor([6, 5, 4, 6])
    sp = SamplingConfig(temperature=0.0)
    NEW = 24
    ar, _ = eng.generate_autoregressive(ids, plen, NEW, sampling=sp)
    for k in (1, 3):
        out, st = eng.generate(ids, plen, NEW, sampling=sp, k_fixed=k)
        assert [o[:NEW] for o in out] == [o[:NEW] for o in ar], k
        assert st.rounds > 0
