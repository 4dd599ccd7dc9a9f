"""Paged KV cache on the kernels: the same results as the contiguous cache.

A paged layer holds the very values of the contiguous [B, Hkv, C, D] cache,
only scattered over pages of PAGE slots in a shared pool.  With C = W * PAGE
the verify attention runs the same schedule and arithmetic on both, so every
comparison here is bit for bit: attention (tensor-core and CUDA-core paths),
the append, the fused norm / RoPE / append, a tiny model through
PagedRaggedCache, and whole engine runs.
"""
import pytest
import torch

from specdec import attention as A
from specdec import fused_attention as FA
from specdec.kvcache import PAGE, PagedRaggedCache, RaggedCache
from tests.tiny_models import VOCAB, TinyTok, tiny_config, tiny_pair_noisy

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _to_pages(cache, W, n_pages, seed):
    """Scatter a contiguous [B, H, W*PAGE, D] cache over a pool in a random
    page order; returns (pool, block table)."""
    B, H, C, D = cache.shape
    assert C == W * PAGE
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(n_pages, generator=g)[:B * W].view(B, W)
    pool = torch.randn(n_pages, H, PAGE, D, generator=g).to(cache.dtype).to(DEV)
    for b in range(B):
        for j in range(W):
            pool[perm[b, j]] = cache[b, :, j * PAGE:(j + 1) * PAGE]
    return pool, perm.to(torch.int32).to(DEV).contiguous()


def _from_pages(pool, bt):
    B, W = bt.shape
    return torch.stack([torch.cat([pool[int(bt[b, j])] for j in range(W)], dim=1)
                        for b in range(B)])


@pytest.mark.parametrize("case", [
    # dtype, B, Hq, Hkv, D, W, qlen, lengths, valid
    (torch.bfloat16, 4, 32, 8, 128, 8, 5, [0, 300, 700, 1010], None),    # tcgen05 path
    (torch.bfloat16, 3, 16, 8, 128, 4, 1, [127, 128, 500], None),        # one draft query
    (torch.bfloat16, 2, 32, 8, 128, 4, 20, [0, 0], [20, 13]),            # short prefill
    (torch.float32, 3, 4, 2, 64, 3, 4, [5, 200, 300], None),              # CUDA-core path
    (torch.bfloat16, 2, 4, 2, 8, 2, 7, [9, 120], None),                   # tiny head dim
])
def test_paged_attention_matches_contiguous(case):
    dt, B, Hq, Hkv, D, W, qlen, lens, valid = case
    C = W * PAGE
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(B, Hq, qlen, D, generator=g, device=DEV).to(dt)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(dt)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(dt)
    lens = torch.tensor(lens, device=DEV)
    val = None if valid is None else torch.tensor(valid, device=DEV)
    want = A.verify_attention(q, kc, vc, lens, valid=val).clone()
    kp, bt = _to_pages(kc, W, B * W + 3, 1)
    vp, _ = _to_pages(vc, W, B * W + 3, 1)
    got = A.verify_attention(q, kp, vp, lens, valid=val, block_table=bt)
    torch.cuda.synchronize()
    assert torch.equal(got, want)


def _bf(x):
    return x.to(torch.bfloat16)


def test_paged_append_matches_contiguous_and_flags_missing_pages():
    B, H, D, W, q = 3, 2, 128, 3, 5
    C = W * PAGE
    g = torch.Generator(device=DEV).manual_seed(5)
    kc = _bf(torch.randn(B, H, C, D, generator=g, device=DEV))
    vc = _bf(torch.randn(B, H, C, D, generator=g, device=DEV))
    kp, bt = _to_pages(kc, W, B * W + 1, 2)
    vp, _ = _to_pages(vc, W, B * W + 1, 2)
    nk = _bf(torch.randn(B, H, q, D, generator=g, device=DEV))
    nv = _bf(torch.randn(B, H, q, D, generator=g, device=DEV))
    lens = torch.tensor([0, PAGE - 2, 2 * PAGE + 7], device=DEV)   # row 1 crosses a page
    ref = RaggedCache(1, B, C, DEV, attn_impl=A.IMPL)
    ref.lengths.copy_(lens)
    ref.layers[0].keys, ref.layers[0].values = kc.clone(), vc.clone()
    ref.layers[0].is_initialized = True
    ref.layers[0].update(nk, nv, 0)
    pc = PagedRaggedCache(1, B, C, DEV, n_pages=B * W + 1)
    pc.lengths.copy_(lens)
    pc.block_table.copy_(bt)
    lay = pc.layers[0]
    lay.keys, lay.values, lay.is_initialized = kp, vp, True
    lay.update(nk, nv, 0)
    torch.cuda.synchronize()
    assert torch.equal(_from_pages(lay.keys, bt), ref.layers[0].keys)
    assert torch.equal(_from_pages(lay.values, bt), ref.layers[0].values)
    assert int(pc._err) == 0
    # a slot whose page is not assigned: nothing written, bit 1 set
    bt2 = bt.clone()
    bt2[1, 1] = -1
    pc.block_table.copy_(bt2)
    before = lay.keys.clone()
    lay.update(nk + 1, nv + 1, 0)
    torch.cuda.synchronize()
    assert int(pc._err) & 2
    # row 1's two slots in page bt[1, 0] are written, its three past the page
    # bound are not; row 0 is written
    assert torch.equal(lay.keys[int(bt[1, 1])], before[int(bt[1, 1])])
    assert torch.equal(lay.keys[int(bt[1, 0]), :, PAGE - 2:], _bf(nk[1, :, :2].float() + 1))
    assert torch.equal(lay.keys[int(bt[0, 0]), :, :q], _bf(nk[0].float() + 1))
    with pytest.raises(RuntimeError):
        pc.check_errors()


def test_fused_append_paged_matches_contiguous():
    from tests.test_fused_attention_gpu import _inputs
    B, Lq, Hq, Hkv, D, W = 3, 5, 32, 8, 128, 3
    C = W * PAGE
    q, k, v, qw, kw, cos, sin, kc, vc, lens = _inputs(B, Lq, Hq, Hkv, D, C,
                                                     [0, PAGE - 3, 2 * PAGE + 1], 7)
    kp, bt = _to_pages(kc, W, B * W + 2, 4)
    vp, _ = _to_pages(vc, W, B * W + 2, 4)
    q1 = FA.qkv_norm_rope_append(q, k, v, qw, kw, 1e-6, cos, sin, kc, vc, lens, D).clone()
    q2 = FA.qkv_norm_rope_append(q, k, v, qw, kw, 1e-6, cos, sin, kp, vp, lens, D,
                                 block_table=bt)
    torch.cuda.synchronize()
    assert torch.equal(q1, q2)
    assert torch.equal(_from_pages(kp, bt), kc)
    assert torch.equal(_from_pages(vp, bt), vc)


def _fwd(m, cache, tokens, valid=None):
    q = tokens.shape[1]
    return m(input_ids=tokens, position_ids=cache.positions(q),
             attention_mask=cache.attn_mask(q, torch.float32, valid=valid),
             past_key_values=cache, cache_position=cache.cache_position(q), use_cache=True).logits


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@torch.inference_mode()
def test_tiny_model_through_paged_cache(dtype):
    """Prefill, a k = 4 verify forward, a rollback and the next forward: the
    same logits from PagedRaggedCache as from RaggedCache (bf16: through the
    fused layers)."""
    from transformers import Qwen3ForCausalLM
    A.register()
    torch.manual_seed(0)
    m = Qwen3ForCausalLM(tiny_config(32, 2)).eval().to(DEV, dtype)
    m.set_attn_implementation(A.IMPL)
    if dtype == torch.bfloat16:
        FA.install(m)
    B, P = 3, 9
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, VOCAB, (B, P), generator=g).to(DEV)
    plen = torch.tensor([9, 6, 7])
    spec = torch.randint(0, VOCAB, (B, 5), generator=g).to(DEV)
    outs = []
    for paged in (False, True):
        c = PagedRaggedCache(2, B, 2 * PAGE, DEV, n_pages=8) if paged else \
            RaggedCache(2, B, 2 * PAGE, DEV, attn_impl=A.IMPL)
        lg = []
        if paged:
            c.reserve_prefill(P, plen)
        lg.append(_fwd(m, c, ids, valid=plen.to(DEV)))
        c.set_lengths(plen)
        for step in range(40):                       # crosses the first page bound
            if paged:
                c.reserve(5)
            lg.append(_fwd(m, c, spec))
            c.advance(5)
            c.rollback([2, 0, 4])
        c.check_errors()
        outs.append((lg, c.lengths.tolist()))
    assert outs[0][1] == outs[1][1] and max(outs[0][1]) > PAGE
    for a, b in zip(outs[0][0], outs[1][0]):
        assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@torch.inference_mode()
def test_long_prefill_through_paged_cache(dtype):
    """A right-padded prefill longer than 64 tokens on a fresh cache runs
    torch's SDPA over the first P slots; the paged cache gathers them from
    its pages (the padding from the sink page).  The last real token's
    logits and the next forward match the contiguous cache."""
    from transformers import Qwen3ForCausalLM
    A.register()
    torch.manual_seed(0)
    m = Qwen3ForCausalLM(tiny_config(32, 2)).eval().to(DEV, dtype)
    m.set_attn_implementation(A.IMPL)
    if dtype == torch.bfloat16:
        FA.install(m)
    B, P = 3, 150
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, VOCAB, (B, P), generator=g).to(DEV)
    plen = torch.tensor([150, 90, 131])
    nxt = torch.randint(0, VOCAB, (B, 2), generator=g).to(DEV)
    outs = []
    for paged in (False, True):
        c = PagedRaggedCache(2, B, 3 * PAGE, DEV, n_pages=10) if paged else \
            RaggedCache(2, B, 3 * PAGE, DEV, attn_impl=A.IMPL)
        if paged:
            c.reserve_prefill(P, plen)
        lg = _fwd(m, c, ids, valid=plen.to(DEV))
        last = lg[torch.arange(B, device=DEV), (plen - 1).to(DEV)].clone()
        c.set_lengths(plen)
        if paged:
            c.reserve(2)
        lg2 = _fwd(m, c, nxt).clone()
        c.check_errors()
        outs.append((last, lg2))
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    for a, b in zip(*outs):
        torch.testing.assert_close(b.float(), a.float(), atol=tol, rtol=tol)


@torch.inference_mode()
def test_engine_paged_matches_contiguous():
    """The engine with paged caches emits the same tokens as with contiguous
    ones, greedy and sampled (same seed), and the pools hold less memory."""
    from specdec.engine import SamplingConfig, SpecDecodeEngine
    target, draft = tiny_pair_noisy(noise=4.0)
    torch.manual_seed(0)
    B = 4
    ids = torch.randint(0, VOCAB, (B, 6))
    plen = torch.tensor([6, 5, 4, 6])
    runs = {}
    for paged in (False, True):
        eng = SpecDecodeEngine(target, draft, TinyTok(), device=DEV, capacity=512,
                               paged_kv=paged)
        for T in (0.0, 1.0):
            out, st = eng.generate(ids, plen, 150, sampling=SamplingConfig(temperature=T),
                                   seed=3, k_fixed=4)
            runs[(paged, T)] = out
    for T in (0.0, 1.0):
        assert runs[(False, T)] == runs[(True, T)], T
    assert max(len(o) for o in runs[(True, 0.0)]) >= 150


def test_paged_pool_is_sized_by_row_lengths():
    """Config-5-like prompts: the paged pool is a fraction of the
    capacity-padded cache (bytes of one bf16 layer of Qwen3-8B heads)."""
    g = torch.Generator().manual_seed(0)
    B, new, k = 64, 512, 8
    plen = torch.randint(128, 4097, (B,), generator=g)
    cap = 4096 + 2 * new + 2 * (k + 1)
    per = plen + 2 * new + 2 * (k + 1)
    n_pages = int(((per + PAGE - 1) // PAGE).sum()) + 1
    c = PagedRaggedCache(1, B, cap, DEV, n_pages=n_pages)
    c.reserve_prefill(int(plen.max()), plen)
    c.layers[0].lazy_initialization(torch.empty(B, 8, 1, 128, dtype=torch.bfloat16, device=DEV))
    contiguous = 2 * B * 8 * c.capacity * 128 * 2
    assert c.kv_bytes < 0.75 * contiguous
    assert c.free_pages == n_pages - 1 - int(((plen + PAGE - 1) // PAGE).sum())
