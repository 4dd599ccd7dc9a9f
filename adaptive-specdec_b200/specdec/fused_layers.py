"""The decoder layers' RMSNorm and gated MLP as single launches.

In every draft and verify forward of the engine (the reference's
specdec/engine.py:245-274 run HF models), each decoder layer calls two
RMSNorms (transformers' Qwen3RMSNorm / LlamaRMSNorm: about eight small
kernels each) and a gated MLP (gate GEMM, up GEMM, SiLU, product, down
GEMM).  At the engine's batch sizes these forwards are launch-bound, so
``install(model)`` gives

* every RMSNorm module one launch of sd_rmsnorm (bf16 inputs; anything else
  runs the module's own forward),
* every SiLU-gated MLP one GEMM over the concatenated gate / up weights (the
  two modules' weights become views into it: no extra memory), one launch of
  sd_silu_mul and the down GEMM, and
* every pre-norm decoder layer (Qwen3, Qwen2, Llama, Mistral) its residual
  add and post-attention norm as one launch of sd_add_rmsnorm.

Numerics are transformers' bf16 sequence; the norm's float32 sum of squares is
reduced in another order, so a value can differ by one bf16 ulp.
"""
import types

import torch

from specdec import _lib as L

__all__ = ["rmsnorm", "add_rmsnorm", "silu_mul", "install", "uninstall", "installed_modules"]


def _rows(x, H):
    """x [..., H] as a 2-D view with one row stride (a copy if it has none)."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    try:
        x2 = x.view(-1, H)
    except RuntimeError:
        x2 = x.contiguous().view(-1, H)
    return x2


def rmsnorm(x, weight, eps, out=None):
    """bf16 RMSNorm over the last dimension: rn(w * rn(x * rsqrt(mean(x^2) + eps)))."""
    L.require_cuda(x, weight)
    if x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise L.SpecdecError("rmsnorm takes bf16 tensors")
    H = x.shape[-1]
    if weight.numel() != H or not weight.is_contiguous():
        raise L.SpecdecError(f"rmsnorm weight must be contiguous [{H}]")
    x2 = _rows(x, H)
    if out is None:
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    o2 = _rows(out, H)
    if o2.data_ptr() != out.data_ptr() or o2.shape != x2.shape:
        raise L.SpecdecError("rmsnorm out must be viewable as rows of H elements")
    with torch.cuda.device(x.device):
        L.check(L.lib().sd_rmsnorm(L.ptr(x2), x2.stride(0), L.ptr(weight), float(eps), L.ptr(o2),
                                   o2.stride(0), x2.shape[0], H, L.stream_ptr(x.device)),
                "rmsnorm")
    return out


def add_rmsnorm(x, res, weight, eps):
    """(rn(x + res), rmsnorm(rn(x + res))): a decoder layer's residual add and
    the norm after it in one launch (bf16, H <= 8192)."""
    L.require_cuda(x, res, weight)
    if x.dtype != torch.bfloat16 or res.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise L.SpecdecError("add_rmsnorm takes bf16 tensors")
    H = x.shape[-1]
    if res.shape != x.shape or weight.numel() != H or not weight.is_contiguous():
        raise L.SpecdecError("add_rmsnorm: x, res [..., H] and a contiguous weight [H]")
    x2, r2 = _rows(x, H), _rows(res, H)
    res_out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    o2, ro2 = out.view(-1, H), res_out.view(-1, H)
    with torch.cuda.device(x.device):
        L.check(L.lib().sd_add_rmsnorm(L.ptr(x2), x2.stride(0), L.ptr(r2), r2.stride(0),
                                       L.ptr(weight), float(eps), L.ptr(o2), o2.stride(0),
                                       L.ptr(ro2), ro2.stride(0), x2.shape[0], H,
                                       L.stream_ptr(x.device)), "add_rmsnorm")
    return res_out, out


def silu_mul(gu, out=None):
    """gu [..., 2I] bf16 = [gate | up] -> rn(rn(silu(gate)) * up) [..., I]."""
    L.require_cuda(gu)
    if gu.dtype != torch.bfloat16 or gu.shape[-1] % 2:
        raise L.SpecdecError("silu_mul takes bf16 [..., 2I]")
    I2 = gu.shape[-1]
    g2 = _rows(gu, I2)
    if out is None:
        out = torch.empty(*gu.shape[:-1], I2 // 2, dtype=gu.dtype, device=gu.device)
    o2 = _rows(out, I2 // 2)
    with torch.cuda.device(gu.device):
        L.check(L.lib().sd_silu_mul(L.ptr(g2), g2.stride(0), L.ptr(o2), o2.stride(0),
                                    g2.shape[0], I2 // 2, L.stream_ptr(gu.device)), "silu_mul")
    return out


def _is_rmsnorm(m):
    w = getattr(m, "weight", None)
    return (type(m).__name__.endswith("RMSNorm") and isinstance(w, torch.Tensor) and w.dim() == 1
            and hasattr(m, "variance_epsilon") and not hasattr(m, "_sd_orig_forward"))


def _norm_forward(self, hidden_states):
    x = hidden_states
    if (x.is_cuda and x.dtype == torch.bfloat16 and self.weight.dtype == torch.bfloat16
            and x.shape[-1] == self.weight.numel()):
        return rmsnorm(x, self.weight, self.variance_epsilon)
    return self._sd_orig_forward(hidden_states)


def _is_silu_mlp(m):
    if not all(hasattr(m, a) for a in ("gate_proj", "up_proj", "down_proj", "act_fn")):
        return False
    if hasattr(m, "_sd_orig_forward"):
        return False
    act = m.act_fn
    return isinstance(act, torch.nn.SiLU) or type(act).__name__ == "SiLUActivation"


def _mlp_forward(self, x):
    if x.is_cuda and x.dtype == torch.bfloat16 and self._sd_gu_w is not None and \
            self._sd_gu_w.dtype == torch.bfloat16:
        gu = torch.nn.functional.linear(x, self._sd_gu_w, self._sd_gu_b)
        return self.down_proj(silu_mul(gu))
    return self._sd_orig_forward(x)


def _fuse_gate_up(m):
    g, u = m.gate_proj, m.up_proj
    if (g.bias is None) != (u.bias is None):
        return None, None
    W = torch.cat([g.weight.detach(), u.weight.detach()], 0)
    bias = torch.cat([g.bias.detach(), u.bias.detach()], 0) if g.bias is not None else None
    n = g.weight.shape[0]
    g.weight = torch.nn.Parameter(W[:n], requires_grad=False)
    u.weight = torch.nn.Parameter(W[n:], requires_grad=False)
    if bias is not None:
        g.bias = torch.nn.Parameter(bias[:n], requires_grad=False)
        u.bias = torch.nn.Parameter(bias[n:], requires_grad=False)
    return W, bias


# decoder layers whose forward is the pre-norm sequence
#   r = x; h = attn(input_layernorm(x)); r = r + h; h = mlp(post_norm(r)); r + h
_PRE_NORM_LAYERS = ("Qwen3DecoderLayer", "Qwen2DecoderLayer", "LlamaDecoderLayer",
                    "MistralDecoderLayer")


def _is_pre_norm_layer(m):
    return (type(m).__name__ in _PRE_NORM_LAYERS and not hasattr(m, "_sd_orig_forward")
            and all(hasattr(m, a) for a in ("self_attn", "mlp", "input_layernorm",
                                            "post_attention_layernorm")))


def _layer_forward(self, hidden_states, attention_mask=None, position_ids=None,
                   past_key_values=None, use_cache=False, position_embeddings=None, **kwargs):
    pn = self.post_attention_layernorm
    if not (hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16
            and pn.weight.dtype == torch.bfloat16 and hidden_states.shape[-1] <= 8192):
        return self._sd_orig_forward(hidden_states, attention_mask=attention_mask,
                                     position_ids=position_ids, past_key_values=past_key_values,
                                     use_cache=use_cache, position_embeddings=position_embeddings,
                                     **kwargs)
    residual = hidden_states
    h = self.input_layernorm(hidden_states)
    h, _ = self.self_attn(hidden_states=h, attention_mask=attention_mask,
                          position_ids=position_ids, past_key_values=past_key_values,
                          use_cache=use_cache, position_embeddings=position_embeddings, **kwargs)
    residual, h = add_rmsnorm(h, residual, pn.weight, pn.variance_epsilon)
    h = self.mlp(h)
    return residual + h


def install(model):
    """Put the one-launch forwards on every RMSNorm, SiLU-gated MLP and
    pre-norm decoder layer (residual add fused into its second norm) of
    ``model``; returns how many modules changed (again: none)."""
    n = 0
    for m in model.modules():
        if _is_pre_norm_layer(m):
            m._sd_orig_forward = m.forward
            m.forward = types.MethodType(_layer_forward, m)
            n += 1
            continue
        if _is_rmsnorm(m):
            m._sd_orig_forward = m.forward
            m.forward = types.MethodType(_norm_forward, m)
            n += 1
        elif _is_silu_mlp(m):
            W, b = _fuse_gate_up(m)
            if W is None:
                continue
            m._sd_gu_w, m._sd_gu_b = W, b
            m._sd_orig_forward = m.forward
            m.forward = types.MethodType(_mlp_forward, m)
            n += 1
    return n


def uninstall(model):
    """Restore the modules' own forwards (the projections keep their views)."""
    for m in model.modules():
        if hasattr(m, "_sd_orig_forward") and (_is_norm_installed(m) or _is_mlp_installed(m)):
            m.forward = m._sd_orig_forward
            del m._sd_orig_forward
            for a in ("_sd_gu_w", "_sd_gu_b"):
                if hasattr(m, a):
                    delattr(m, a)


def _is_norm_installed(m):
    f = getattr(m.forward, "__func__", None)
    return f is _norm_forward or f is _layer_forward


def _is_mlp_installed(m):
    f = getattr(m.forward, "__func__", None)
    return f is _mlp_forward


def installed_modules(model):
    return sum(1 for m in model.modules() if _is_norm_installed(m) or _is_mlp_installed(m))
