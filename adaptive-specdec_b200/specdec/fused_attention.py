"""One kernel between an attention layer's projections and its attention.

transformers' Qwen3Attention.forward (and Llama's, without the norms) runs,
per layer and forward, the q / k / v projections, then RMSNorm on each q and
k head, the rotary embedding on q and k, the cache update (the reference's
_RaggedLayer.update, specdec/kvcache.py:61-74) and the attention.  Between
the projections and the attention that is a dozen small elementwise kernels
per tensor plus the append.  ``install(model)`` replaces that stretch, for
the layers run against a ``RaggedCache(..., attn_impl="specdec_b200")``, with

* one projection GEMM over the concatenated q / k / v weights (the three
  modules' weights become views into it: no extra memory), and
* one launch of sd_qkv_norm_rope_append: norm, rotary embedding, q out in the
  attention's [B, Hq, L, D] layout, k and v into the cache at each row's own
  offset,

after which the verify-attention kernel and o_proj run as before.  Any other
call (another cache, another attention implementation, a dtype other than
bf16, sliding-window layers) goes through the layer's original forward.

Numerics: the same bf16 operations in the same order as transformers'; the
float32 sum of squares of the norm is reduced in another order, so a
normalised value can differ by one bf16 ulp.
"""
import types

import torch

from specdec import _lib as L
from specdec import attention as A
from specdec.kvcache import RaggedCache

__all__ = ["qkv_norm_rope_append", "install", "uninstall", "installed_layers"]

D_MAX = 256


def _row_stride(x, name):
    """Element stride between consecutive (b, l) rows of a [B, L, H*D] tensor
    whose rows are evenly spaced and whose last dimension is contiguous."""
    if x.dim() != 3 or x.stride(-1) != 1:
        raise L.SpecdecError(f"{name}: [B, L, H*D] with a contiguous last dimension expected")
    B, Lq, _ = x.shape
    if Lq == 1:
        return x.stride(0) if B > 1 else 0
    if B > 1 and x.stride(0) != Lq * x.stride(1):
        raise L.SpecdecError(f"{name}: rows must be evenly spaced (stride(0) == L * stride(1))")
    return x.stride(1)


def qkv_norm_rope_append(q, k, v, q_norm_w, k_norm_w, eps, cos, sin, k_cache, v_cache, lengths,
                         head_dim, q_out=None, err=None, block_table=None):
    """q [B, L, Hq*D], k / v [B, L, Hkv*D] (bf16 projection outputs) ->
    q_out [B, Hq, L, D]; k and v are written to k_cache / v_cache
    [B, Hkv, C, D] at slots lengths[b] + l, or, with ``block_table`` [B, W]
    int32, to the page pools [n_pages, Hkv, PAGE, D] of a PagedRaggedCache
    (C = W * PAGE).

    q_norm_w / k_norm_w [D] (or both None: no norm) and eps are the heads'
    RMSNorm; cos / sin [B or 1, L, D] the rotary tables of the positions.
    ``err`` ([1] int32) gets bit 0 when a row's slots would pass C and bit 1
    when a paged slot has no page (those k / v are not written)."""
    L.require_cuda(q, k, v, cos, sin, k_cache, v_cache, lengths)
    ts = [q, k, v, cos, sin, k_cache, v_cache] + [w for w in (q_norm_w, k_norm_w) if w is not None]
    if any(t.dtype != torch.bfloat16 for t in ts):
        raise L.SpecdecError("qkv_norm_rope_append takes bf16 tensors")
    if (q_norm_w is None) != (k_norm_w is None):
        raise L.SpecdecError("give both norm weights or neither")
    D = int(head_dim)
    B, Lq, nq = q.shape
    Bc, Hkv, C, Dc = k_cache.shape
    bts = npages = 0
    if block_table is not None:
        if block_table.dtype != torch.int32 or block_table.dim() != 2 or \
                block_table.shape[0] != B or not block_table.is_contiguous():
            raise L.SpecdecError("block_table must be a contiguous [B, W] int32 tensor")
        npages, bts = Bc, block_table.shape[1]
        Bc, C = B, bts * C
    if Dc != D or nq % D or k.shape != (B, Lq, Hkv * D) or v.shape != k.shape or Bc != B:
        raise L.SpecdecError(f"shape mismatch: q {tuple(q.shape)}, k {tuple(k.shape)}, "
                             f"cache {tuple(k_cache.shape)}, head_dim {D}")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous() and v_cache.shape == k_cache.shape):
        raise L.SpecdecError("the caches must be contiguous [B, Hkv, C, D]")
    Hq = nq // D
    if cos.shape[-2:] != (Lq, D) or sin.shape != cos.shape or cos.shape[0] not in (1, B):
        raise L.SpecdecError(f"cos / sin must be [B or 1, L, D], got {tuple(cos.shape)}")
    if cos.stride() != sin.stride() or cos.stride(-1) != 1:
        cos, sin = cos.contiguous(), sin.contiguous()
    cs_bs = cos.stride(0) if cos.shape[0] > 1 else 0
    cs_ls = cos.stride(1)
    for w in (q_norm_w, k_norm_w):
        if w is not None and (w.numel() != D or not w.is_contiguous()):
            raise L.SpecdecError("norm weights must be contiguous [D]")
    lens = lengths if lengths.dtype == torch.long and lengths.is_contiguous() else \
        lengths.to(torch.long).contiguous()
    if q_out is None:
        q_out = torch.empty(B, Hq, Lq, D, dtype=q.dtype, device=q.device)
    elif q_out.shape != (B, Hq, Lq, D) or not q_out.is_contiguous():
        raise L.SpecdecError("q_out must be contiguous [B, Hq, L, D]")
    with torch.cuda.device(q.device):
        L.check(L.lib().sd_qkv_norm_rope_append(
            L.ptr(q), _row_stride(q, "q"), L.ptr(k), _row_stride(k, "k"), L.ptr(v),
            _row_stride(v, "v"), L.ptr(q_norm_w), L.ptr(k_norm_w), float(eps), L.ptr(cos),
            L.ptr(sin), cs_bs, cs_ls, L.ptr(k_cache), L.ptr(v_cache), L.ptr(block_table), bts,
            npages, L.ptr(lens), B, Lq, Hq, Hkv, D, C, L.ptr(q_out), L.ptr(err),
            L.stream_ptr(q.device)), "qkv_norm_rope_append")
    return q_out


def _is_attention(m):
    return all(hasattr(m, a) for a in ("q_proj", "k_proj", "v_proj", "o_proj", "head_dim",
                                       "layer_idx", "scaling"))


def _norm_of(m, name):
    n = getattr(m, name, None)
    if n is None:
        return None, None
    eps = getattr(n, "variance_epsilon", getattr(n, "eps", None))
    if eps is None or getattr(n, "weight", None) is None:
        raise L.SpecdecError(f"{type(m).__name__}.{name} is not an RMSNorm with a weight")
    return n.weight, float(eps)


def _fuse_qkv_weights(m):
    """Concatenate the three projections' weights (and biases) into one tensor
    and make the modules' parameters views into it."""
    projs = (m.q_proj, m.k_proj, m.v_proj)
    W = torch.cat([p.weight.detach() for p in projs], 0)
    has_bias = [p.bias is not None for p in projs]
    if any(has_bias) and not all(has_bias):
        return None, None
    bias = torch.cat([p.bias.detach() for p in projs], 0) if all(has_bias) else None
    o = 0
    for p in projs:
        n = p.weight.shape[0]
        p.weight = torch.nn.Parameter(W[o:o + n], requires_grad=False)
        if bias is not None:
            p.bias = torch.nn.Parameter(bias[o:o + n], requires_grad=False)
        o += n
    return W, bias


def _fused_forward(self, hidden_states, position_embeddings=None, attention_mask=None,
                   past_key_values=None, **kwargs):
    cache = past_key_values
    D = self.head_dim
    if (not isinstance(cache, RaggedCache) or cache.attn_impl != A.IMPL
            or self.config._attn_implementation != A.IMPL or position_embeddings is None
            or hidden_states.dtype != torch.bfloat16 or D % 2 or D > D_MAX
            or position_embeddings[0].dtype != torch.bfloat16
            or getattr(self, "sliding_window", None) is not None):
        return self._sd_orig_forward(hidden_states, position_embeddings, attention_mask,
                                     past_key_values=past_key_values, **kwargs)
    B, Lq, _ = hidden_states.shape
    nq, nk = self.q_proj.weight.shape[0], self.k_proj.weight.shape[0]
    if self._sd_qkv_w is not None:
        qkv = torch.nn.functional.linear(hidden_states, self._sd_qkv_w, self._sd_qkv_b)
        q, k, v = qkv[..., :nq], qkv[..., nq:nq + nk], qkv[..., nq + nk:]
    else:
        q, k, v = self.q_proj(hidden_states), self.k_proj(hidden_states), self.v_proj(hidden_states)
    layer = cache.layers[self.layer_idx]
    Hkv = nk // D
    if not layer.is_initialized:
        layer.lazy_initialization(torch.empty(B, Hkv, 1, D, dtype=q.dtype, device=q.device))
    qw, eps = _norm_of(self, "q_norm")
    kw, _ = _norm_of(self, "k_norm")
    cos, sin = position_embeddings
    q_out = qkv_norm_rope_append(q, k, v, qw, kw, eps if eps is not None else 0.0, cos, sin,
                                 layer.keys, layer.values, cache.lengths, D, err=cache._err,
                                 block_table=getattr(cache, "block_table", None))
    cache._last_q = Lq
    out, w = A.hf_attention(self, q_out, layer.keys, layer.values, attention_mask,
                            scaling=self.scaling)
    out = out.reshape(B, Lq, -1)
    return self.o_proj(out), w


def install(model, fuse_qkv_gemm=True):
    """Put the fused forward on every attention layer of ``model`` whose norms
    (if any) are RMSNorms over the head dimension.  Returns the number of
    layers changed; calling it again changes nothing."""
    n = 0
    for m in model.modules():
        if not _is_attention(m) or hasattr(m, "_sd_orig_forward"):
            continue
        qn, kn = getattr(m, "q_norm", None), getattr(m, "k_norm", None)
        if (qn is None) != (kn is None):
            continue
        if qn is not None:
            _norm_of(m, "q_norm")
            _norm_of(m, "k_norm")
            if qn.weight.numel() != m.head_dim or kn.weight.numel() != m.head_dim:
                continue
        W = bias = None
        if fuse_qkv_gemm:
            W, bias = _fuse_qkv_weights(m)
        m._sd_qkv_w, m._sd_qkv_b = W, bias
        m._sd_orig_forward = m.forward
        m.forward = types.MethodType(_fused_forward, m)
        n += 1
    return n


def _installed(m):
    return getattr(m.forward, "__func__", None) is _fused_forward


def uninstall(model):
    """Restore the original forwards (the projections keep their views)."""
    for m in model.modules():
        if _installed(m):
            m.forward = m._sd_orig_forward
            del m._sd_orig_forward, m._sd_qkv_w, m._sd_qkv_b


def installed_layers(model):
    return sum(1 for m in model.modules() if _installed(m))
