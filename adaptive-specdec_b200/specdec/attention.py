"""Verify attention over the ragged cache, and its transformers hook.

``verify_attention`` is the Python face of sd_verify_attn: grouped-query
attention where query j of row b reads cache slots s <= lengths[b] + j (and
s < valid[b] in a right-padded prefill).  It replaces the reference's HF SDPA
over ``_RaggedLayer.update``'s max-width view plus the additive mask
(specdec/kvcache.py:61-74 and :138-162, called at specdec/engine.py:274): each
row reads only its own live keys.

``register()`` installs it as the transformers attention implementation
"specdec_b200" (with a mask function that builds no mask); a model loaded with
``attn_implementation="specdec_b200"`` and run against a
``RaggedCache(..., attn_impl="specdec_b200")`` then attends through the kernel.
"""
import torch

from specdec import _lib as L

IMPL = "specdec_b200"
PREFILL_SDPA_MIN = 64          # prefills longer than this (fresh cache) use torch SDPA
_ATTN_DTYPES = {torch.bfloat16: 2, torch.float32: 0}


class _WS:
    def __init__(self):
        self.t = {}

    def get(self, n, device):
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        cur = self.t.get(key)
        if cur is None or cur.numel() < n:
            cur = torch.empty(max(int(n), 1 << 20), dtype=torch.uint8, device=device)
            self.t[key] = cur
        return cur


_ws = _WS()


def verify_attention(q, k_cache, v_cache, lengths, valid=None, scale=None, out=None,
                     block_table=None):
    """q [B, Hq, qlen, D], caches [B, Hkv, C, D] -> out [B, qlen, Hq, D].

    ``lengths`` [B] int64 on the device are the lengths before this forward's
    advance (the new keys were already appended at lengths[b] + j).  With
    ``block_table`` [B, W] int32 the caches are page pools
    [n_pages, Hkv, PAGE, D] (PagedRaggedCache) and C = W * PAGE.
    """
    L.require_cuda(q, k_cache, v_cache, lengths)
    if q.dtype not in _ATTN_DTYPES or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise L.SpecdecError(f"verify_attention supports bf16 / fp32, got {q.dtype}")
    B, Hq, qlen, D = q.shape
    if block_table is not None:
        return _verify_attention_paged(q, k_cache, v_cache, lengths, valid, scale, out,
                                       block_table)
    _, Hkv, C, _ = k_cache.shape
    if q.stride(-1) != 1:
        q = q.contiguous()
    kc = k_cache if k_cache.is_contiguous() else k_cache.contiguous()
    vc = v_cache if v_cache.is_contiguous() else v_cache.contiguous()
    if out is None:
        out = torch.empty(B, qlen, Hq, D, dtype=q.dtype, device=q.device)
    sc = float(scale) if scale is not None else D ** -0.5
    lens = lengths.to(torch.long).contiguous()
    val = None if valid is None else valid.to(q.device, torch.long).contiguous()
    lib = L.lib()
    with torch.cuda.device(q.device):
        nws = lib.sd_verify_attn_workspace_bytes(B, Hq, Hkv, D, C, qlen)
        ws = _ws.get(nws, q.device)
        L.check(lib.sd_verify_attn(L.ptr(q), q.stride(0), q.stride(1), q.stride(2), L.ptr(kc),
                                   L.ptr(vc), L.ptr(lens), L.ptr(val), B, Hq, Hkv, D, C, qlen, sc,
                                   L.ptr(out), out.stride(0), out.stride(1), out.stride(2),
                                   _ATTN_DTYPES[q.dtype], L.ptr(ws), ws.numel(),
                                   L.stream_ptr(q.device)), "verify_attn")
    return out


def _verify_attention_paged(q, kpool, vpool, lengths, valid, scale, out, bt):
    from specdec.kvcache import PAGE
    B, Hq, qlen, D = q.shape
    npages, Hkv, page, _ = kpool.shape
    if page != PAGE or vpool.shape != kpool.shape or not (kpool.is_contiguous()
                                                          and vpool.is_contiguous()):
        raise L.SpecdecError("paged caches must be contiguous [n_pages, Hkv, PAGE, D] pools")
    if bt.dtype != torch.int32 or bt.dim() != 2 or bt.shape[0] != B or not bt.is_contiguous():
        raise L.SpecdecError("block_table must be a contiguous [B, W] int32 tensor")
    W = bt.shape[1]
    if q.stride(-1) != 1:
        q = q.contiguous()
    if out is None:
        out = torch.empty(B, qlen, Hq, D, dtype=q.dtype, device=q.device)
    sc = float(scale) if scale is not None else D ** -0.5
    lens = lengths.to(torch.long).contiguous()
    val = None if valid is None else valid.to(q.device, torch.long).contiguous()
    lib = L.lib()
    with torch.cuda.device(q.device):
        nws = lib.sd_verify_attn_workspace_bytes(B, Hq, Hkv, D, W * PAGE, qlen)
        ws = _ws.get(nws, q.device)
        L.check(lib.sd_verify_attn_paged(
            L.ptr(q), q.stride(0), q.stride(1), q.stride(2), L.ptr(kpool), L.ptr(vpool), L.ptr(bt),
            W, npages, L.ptr(lens), L.ptr(val), B, Hq, Hkv, D, qlen, sc, L.ptr(out), out.stride(0),
            out.stride(1), out.stride(2), _ATTN_DTYPES[q.dtype], L.ptr(ws), ws.numel(),
            L.stream_ptr(q.device)), "verify_attn_paged")
    return out


def gather_pages(pool, block_table, n):
    """The first n slots of every row of a page pool as [B, Hkv, n, D]."""
    from specdec.kvcache import PAGE
    npg = -(-n // PAGE)
    idx = block_table[:, :npg].long().clamp_min(0)
    B = idx.shape[0]
    g = pool[idx]                                     # [B, npg, Hkv, PAGE, D]
    return g.permute(0, 2, 1, 3, 4).reshape(B, pool.shape[1], npg * PAGE, pool.shape[3])[:, :, :n]


def hf_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None, **kwargs):
    """transformers AttentionInterface function for RaggedCache buffers."""
    cache = getattr(key, "_sd_cache", None)
    if cache is not None:
        q_len = query.shape[2]
        if (cache.valid is not None and q_len > PREFILL_SDPA_MIN and cache._host_valid
                and int(cache._host.max()) == 0):
            # right-padded prefill of a fresh cache (every row at length 0):
            # plain causal attention over the q new keys; a real token i < valid[b]
            # only sees keys s <= i, so the padding never reaches it.  Prefill is
            # outside the verify round; torch's SDPA (flash / cuDNN) runs it.
            bt = getattr(cache, "block_table", None)
            if bt is not None:
                ks, vs = gather_pages(key, bt, q_len), gather_pages(value, bt, q_len)
            else:
                ks, vs = key[:, :, :q_len], value[:, :, :q_len]
            out = torch.nn.functional.scaled_dot_product_attention(
                query, ks, vs, is_causal=True, scale=scaling, enable_gqa=True)
            return out.transpose(1, 2), None
        out = verify_attention(query, key, value, cache.lengths, valid=cache.valid, scale=scaling,
                               block_table=getattr(cache, "block_table", None))
        return out, None
    # a forward without a RaggedCache: causal self-attention over the given
    # K/V, i.e. the same kernel with every row starting at length 0
    if attention_mask is not None and attention_mask.dim() == 4 and not bool(
            (attention_mask == 0).all()):
        raise L.SpecdecError("specdec_b200 attention without a RaggedCache supports plain "
                             "causal masks only")
    if key.shape[2] != query.shape[2]:
        raise L.SpecdecError("specdec_b200 attention without a RaggedCache needs q_len == kv_len")
    lens = torch.zeros(query.shape[0], dtype=torch.long, device=query.device)
    out = verify_attention(query, key.contiguous(), value.contiguous(), lens, scale=scaling)
    return out, None


def _no_mask(*args, **kwargs):
    return None


def register():
    """Register the kernel as attention implementation "specdec_b200"."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface
    AttentionInterface.register(IMPL, hf_attention)
    AttentionMaskInterface.register(IMPL, _no_mask)
    return IMPL
