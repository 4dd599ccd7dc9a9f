"""Ragged KV cache (K2) and verify attention (K3) on the GPU.

* lengths bookkeeping replays the reference RaggedCache trace (fixture from
  reference specdec/kvcache.py) and must match exactly;
* KV append is checked element-for-element against a torch scatter;
* verify attention is checked against a plain fp32 torch implementation of the
  reference mask rule s <= lengths[b] + j (bf16: 2e-2 abs / rel, fp32: 1e-4);
* the reference invariant (tests/test_kv_rollback.py in the reference): after a
  rollback the cache is indistinguishable from one that only saw the accepted
  prefix, and a poisoned stale tail never leaks -- run through a tiny Qwen3
  whose attention is the kernel.
"""
import json

import pytest
import torch

from specdec import attention as A
from specdec import workloads as W
from specdec.kvcache import RaggedCache
from tests.golden import GOLDEN

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def test_lengths_trace_matches_reference():
    g = json.loads((GOLDEN / "kvcache.json").read_text())
    c = RaggedCache(2, 3, 32, DEV)
    for op, arg, want in g["trace"]:
        if op == "set_lengths":
            c.set_lengths(torch.tensor(arg))
        elif op == "advance":
            c.advance(arg)
        elif isinstance(arg, list) and op == "rollback" and arg == [1, 0, 1]:
            c.rollback(torch.tensor(arg, device=DEV))          # device path, no sync
        else:
            c.rollback(arg)
        assert c.lengths.tolist() == want, op
    assert c.positions(3).tolist() == g["positions"]
    assert c.cache_position(3).tolist() == g["cache_position"]
    assert c.kv_len_for(3) == g["kv_len_for_3"]
    assert (c.attn_mask(3, torch.float32) == 0).squeeze(1).tolist() == \
        [m[0] for m in g["mask_allowed"]]
    mv = c.attn_mask(3, torch.float32, valid=torch.tensor([9, 4, 6]))
    assert (mv == 0).squeeze(1).tolist() == [m[0] for m in g["mask_valid_allowed"]]
    with pytest.raises(RuntimeError):
        c.rollback([100, 0, 0])
    c2 = RaggedCache(1, 2, 16, DEV)
    c2.set_lengths([4, 4])
    assert (c2.attn_mask(2, torch.float32) is None) == g["uniform_mask_is_none"]


def test_commit_and_device_errors():
    c = RaggedCache(1, 4, 64, DEV)
    c.set_lengths([10, 20, 30, 40])
    c.advance(5)
    c.commit(torch.tensor([0, 4, 2, 3], device=DEV), 4)
    assert c.lengths.tolist() == [11, 25, 33, 44]
    c.rollback(torch.tensor([0, 0, 100, 0], device=DEV))      # below zero: refused on device
    with pytest.raises(RuntimeError):
        c.check_errors()
    assert c.lengths.tolist() == [11, 25, 33, 44]
    c.advance(30)                        # row 3 would pass capacity: that row is refused
    with pytest.raises(RuntimeError):
        c.check_errors()
    assert c.lengths.tolist() == [41, 55, 63, 44]
    c.set_lengths([60, 0, 0, 0])
    with pytest.raises(RuntimeError):
        c.advance(5)                                           # host-known: raises at once


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_append_matches_scatter(dt):
    g = torch.Generator(device=DEV).manual_seed(0)
    B, H, C, D, q = 5, 3, 40, 16, 4
    c = RaggedCache(1, B, C, DEV)
    lens = torch.tensor([0, 3, 7, 20, 36])
    c.set_lengths(lens)
    k = torch.randn(B, H, q, D, generator=g, device=DEV).to(dt)
    v = torch.randn(B, H, q, D, generator=g, device=DEV).to(dt)
    c.layers[0].update(k, v)
    ref = torch.zeros(B, H, C, D, dtype=dt, device=DEV)
    idx = (lens.to(DEV).view(B, 1) + torch.arange(q, device=DEV)).view(B, 1, q, 1).expand(B, H, q, D)
    ref.scatter_(2, idx, k)
    assert torch.equal(c.layers[0].keys, ref)
    ref.zero_().scatter_(2, idx, v)
    assert torch.equal(c.layers[0].values, ref)


def _ref_attention(q, kc, vc, lens, valid, scale):
    """fp32 attention with the reference mask rule s <= len[b] + j (and s < valid[b])."""
    B, Hq, ql, D = q.shape
    Hkv, C = kc.shape[1], kc.shape[2]
    g = Hq // Hkv
    kf = kc.float().repeat_interleave(g, dim=1)
    vf = vc.float().repeat_interleave(g, dim=1)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float(), kf) * scale
    pos = torch.arange(C, device=q.device).view(1, 1, 1, C)
    lim = lens.view(B, 1, 1, 1) + torch.arange(ql, device=q.device).view(1, 1, ql, 1)
    allowed = pos <= lim
    if valid is not None:
        allowed = allowed & (pos < valid.view(B, 1, 1, 1))
    s = s.masked_fill(~allowed, float("-inf"))
    p = torch.softmax(s, -1).nan_to_num(0.0)
    return torch.einsum("bhqk,bhkd->bqhd", p, vf)


@pytest.mark.parametrize("dt,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-4)])
def test_verify_attention_matches_reference_rule(dt, tol):
    g = torch.Generator(device=DEV).manual_seed(1)
    B, Hq, Hkv, D, C, ql = 6, 32, 8, 128, 2304, 5
    lens = torch.tensor([16, 300, 1, 1024, 2000, 777], device=DEV)
    q = torch.randn(B, Hq, ql, D, generator=g, device=DEV).to(dt)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(dt)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(dt)
    out = A.verify_attention(q, kc, vc, lens, scale=D ** -0.5)
    ref = _ref_attention(q, kc, vc, lens, None, D ** -0.5)
    torch.testing.assert_close(out.float(), ref, atol=tol, rtol=tol)
    # stale tail beyond each row's live window is unreachable
    kc2, vc2 = kc.clone(), vc.clone()
    for b in range(B):
        kc2[b, :, int(lens[b]) + ql:] = 99.0
        vc2[b, :, int(lens[b]) + ql:] = 99.0
    out2 = A.verify_attention(q, kc2, vc2, lens, scale=D ** -0.5)
    assert torch.equal(out, out2)


def test_verify_attention_tensor_core_splits_and_caps():
    """bf16, head_dim 128 (the tensor-core path): rows with no live key, one
    split, several splits and a 6-key last split; repeated calls reuse the
    per-call split counters."""
    g = torch.Generator(device=DEV).manual_seed(3)
    B, Hq, Hkv, D, C, ql = 5, 32, 8, 128, 3000, 5
    lens = torch.tensor([0, 1020, 2500, 7, 1500], device=DEV)
    valid = torch.tensor([0, 1022, 3000, 3, 1030], device=DEV)
    q = torch.randn(B, Hq, ql, D, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(torch.bfloat16)
    ref = _ref_attention(q, kc, vc, lens, valid, D ** -0.5)
    out = A.verify_attention(q, kc, vc, lens, valid=valid, scale=D ** -0.5)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
    assert torch.count_nonzero(out[0]) == 0
    for _ in range(3):
        again = A.verify_attention(q, kc, vc, lens, valid=valid, scale=D ** -0.5)
        assert torch.equal(again, out)
    # NaN in every slot outside the live windows (never-written cache memory)
    # must not reach the output
    kc2, vc2 = kc.clone(), vc.clone()
    for b in range(B):
        n = min(int(lens[b]) + ql, int(valid[b]))
        kc2[b, :, n:] = float("nan")
        vc2[b, :, n:] = float("nan")
    out2 = A.verify_attention(q, kc2, vc2, lens, valid=valid, scale=D ** -0.5)
    assert torch.equal(out2, out)


def _ref_rows(q, kc, vc, lens, scale, rows):
    """fp32 attention of the reference's mask rule (key s visible to query j
    of row b iff s <= lens[b] + j), one row at a time (config-3 sized caches
    do not fit a dense [B, Hq, q, C] score tensor comfortably)."""
    B, Hq, ql, D = q.shape
    g = Hq // kc.shape[1]
    out = {}
    for b in rows:
        n = int(lens[b]) + ql
        kf = kc[b, :, :n].float().repeat_interleave(g, dim=0)
        vf = vc[b, :, :n].float().repeat_interleave(g, dim=0)
        s = torch.einsum("hqd,hkd->hqk", q[b].float(), kf) * scale
        pos = torch.arange(n, device=q.device).view(1, 1, n)
        lim = int(lens[b]) + torch.arange(ql, device=q.device).view(1, ql, 1)
        s = s.masked_fill(pos > lim, float("-inf"))
        out[b] = torch.einsum("hqk,hkd->qhd", torch.softmax(s, -1), vf)
    return out


def test_verify_attention_config3_shape():
    """The headline shape of config 3: B = 64 rows, 32 query / 8 kv heads x
    128, 5 queries, context lengths uniform in [512, 8192] (the bench's
    seeded lengths), one layer, every row checked against the fp32 rule.
    This is the stream-K schedule, piece merge and cost-aware split at the
    size they are timed at."""
    B, Hq, Hkv, D, ql = 64, 32, 8, 128, 5
    lens = W.attn_lengths(B, seed=0).to(DEV)
    C = int(lens.max()) + ql + 3
    g = torch.Generator(device=DEV).manual_seed(0)
    q = torch.randn(B, Hq, ql, D, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(torch.bfloat16)
    out = A.verify_attention(q, kc, vc, lens, scale=D ** -0.5)
    ref = _ref_rows(q, kc, vc, lens, D ** -0.5, range(B))
    for b in range(B):
        torch.testing.assert_close(out[b].float(), ref[b], atol=2e-2, rtol=2e-2,
                                   msg=lambda m: f"row {b} (len {int(lens[b])}): {m}")
    again = A.verify_attention(q, kc, vc, lens, scale=D ** -0.5)
    assert torch.equal(again, out)


def test_prefill_valid_cap():
    g = torch.Generator(device=DEV).manual_seed(2)
    B, Hq, Hkv, D, C, ql = 3, 4, 2, 8, 16, 7
    q = torch.randn(B, Hq, ql, D, generator=g, device=DEV)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV)
    lens = torch.zeros(B, dtype=torch.long, device=DEV)
    valid = torch.tensor([7, 5, 6], device=DEV)
    out = A.verify_attention(q, kc, vc, lens, valid=valid)
    ref = _ref_attention(q, kc, vc, lens, valid, D ** -0.5)
    for b in range(B):
        n = int(valid[b])
        torch.testing.assert_close(out[b, :n], ref[b, :n], atol=1e-4, rtol=1e-4)


# ---------------------------------------------------------------------------
# the reference's rollback invariant, through a tiny Qwen3 on the kernels
# ---------------------------------------------------------------------------
def _tiny(seed=0):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=16, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=8,
                      max_position_embeddings=256, tie_word_embeddings=True)
    return Qwen3ForCausalLM(cfg).eval().to(DEV)


def _fwd(m, cache, tokens, valid=None):
    q = tokens.shape[1]
    return m(input_ids=tokens, position_ids=cache.positions(q),
             attention_mask=cache.attn_mask(q, torch.float32, valid=valid),
             past_key_values=cache, cache_position=cache.cache_position(q), use_cache=True).logits


@torch.inference_mode()
def test_rollback_invariant_tiny_qwen3():
    A.register()
    m = _tiny()
    m.set_attn_implementation(A.IMPL)
    ref = _tiny()
    ref.set_attn_implementation("eager")
    B, P = 3, 7
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 16, (B, P), generator=g).to(DEV)
    plen = torch.tensor([7, 5, 6], device=DEV)
    c = RaggedCache(2, B, 128, DEV, attn_impl=A.IMPL)
    lg = _fwd(m, c, ids, valid=plen)
    c.set_lengths(plen.cpu())
    for b in range(B):
        want = ref(input_ids=ids[b:b + 1, :int(plen[b])]).logits[0, -1]
        torch.testing.assert_close(lg[b, int(plen[b]) - 1], want, atol=1e-4, rtol=1e-4)
    spec = torch.randint(0, 16, (B, 4), generator=g).to(DEV)
    keep = torch.tensor([4, 1, 2])
    _fwd(m, c, spec)
    c.advance(4)
    c.rollback((4 - keep).tolist())
    assert c.lengths.tolist() == (plen.cpu() + keep).tolist()
    nxt = torch.randint(0, 16, (B, 1), generator=g).to(DEV)
    got = _fwd(m, c, nxt)
    for b in range(B):
        seq = torch.cat([ids[b, :int(plen[b])], spec[b, :int(keep[b])], nxt[b]]).unsqueeze(0)
        want = ref(input_ids=seq).logits[0, -1]
        torch.testing.assert_close(got[b, -1], want, atol=1e-4, rtol=1e-4)
    # poisoned stale tail
    outs = []
    for corrupt in (False, True):
        cc = RaggedCache(2, B, 128, DEV, attn_impl=A.IMPL)
        _fwd(m, cc, ids, valid=plen)
        cc.set_lengths(plen.cpu())
        _fwd(m, cc, spec)
        cc.advance(4)
        cc.rollback((4 - keep).tolist())
        if corrupt:
            for layer in cc.layers:
                for b in range(B):
                    layer.keys[b, :, int(cc.lengths[b]):] = 99.0
                    layer.values[b, :, int(cc.lengths[b]):] = 99.0
        outs.append(_fwd(m, cc, nxt).clone())
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("case", [
    # B, Hq, Hkv, qlen, lengths (None: U[512, 640]), valid, C
    (32, 16, 8, 1, None, None, 1040),                 # a config-4 draft step (2 rows / kv head)
    (4, 32, 8, 2, [0, 127, 128, 1000], None, 1200),   # 8 rows per kv head, page bounds
    (3, 8, 8, 8, [5, 300, 0], [9, 303, 4], 320),      # group 1, 8 queries, a capped prefill
    (2, 16, 8, 1, [7000, 8100], None, 8200),          # long rows: 64 chunks each
])
def test_attention_few_query_rows_matches_reference_rule(case):
    """<= 8 query rows per kv head (a draft step, group-1 layers, short
    prefills) against the fp32 mask rule, rows of every length class."""
    B, Hq, Hkv, ql, lens, valid, C = case
    g = torch.Generator(device=DEV).manual_seed(4)
    D = 128
    if lens is None:
        lens = torch.randint(512, 641, (B,), generator=torch.Generator().manual_seed(0)).tolist()
    q = torch.randn(B, Hq, ql, D, generator=g, device=DEV).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=DEV).to(torch.bfloat16)
    lens_d = torch.tensor(lens, device=DEV)
    val = None if valid is None else torch.tensor(valid, device=DEV)
    out = A.verify_attention(q, kc, vc, lens_d, valid=val)
    ref = _ref_attention(q, kc, vc, lens_d, val, D ** -0.5)
    torch.testing.assert_close(out.float(), ref, atol=2e-2, rtol=2e-2)
