"""Sampling transforms and rejection sampling on B200 kernels.

Drop-in for the reference's specdec/sampling.py (to_probs, sample_from_probs,
residual_probs, gather_prob at lines 34-95), with the same names, argument
meaning and output dtypes, plus the two fused entry points the engine uses:

* ``verify_sample`` -- one launch sequence for engine.py:282-303: to_probs on
  the k+1 target and k draft vectors, the accept test, and the residual or
  bonus draw;
* ``draft_sample``  -- one draft step, engine.py:250-251 and :256.

Draws are inverse-CDF with uniforms: either passed in (``u=...``) or drawn
from ``generator`` on the device.  Given the same uniforms, results match the
reference's arithmetic as restated in oracle/sampling_oracle.py.

Tie rule at the top-p boundary: among equal probabilities, lower vocabulary
index first (the reference's ``torch.sort`` is unstable, so any order is a
valid reading of it; this one is deterministic).
"""
import torch

from specdec import _lib as L

__all__ = ["to_probs", "sample_from_probs", "residual_probs", "gather_prob",
           "verify_sample", "verify_sample_probs", "draft_sample"]


def _knobs(temperature, top_p, top_k):
    T = 0.0 if temperature is None or temperature <= 0.0 else float(temperature)
    tp = 1.0 if top_p is None else float(top_p)
    tk = 0 if not top_k else int(top_k)
    return T, tp, tk


def _rows(x):
    """View x [..., V] as [N, V] with unit stride along V."""
    V = x.shape[-1]
    x2 = x.reshape(-1, V)
    if x2.stride(-1) != 1 or (x2.shape[0] > 1 and x2.stride(0) < V):
        x2 = x2.contiguous()
    return x2


def to_probs(logits, temperature=1.0, top_p=1.0, top_k=0):
    """Logits -> float32 probabilities over the full vocabulary.

    Same contract as reference specdec/sampling.py:34-67: temperature <= 0 is a
    one-hot at the first maximum; otherwise softmax(logits / T), then top-k
    (ties at the k-th value kept), then top-p (smallest prefix of the sorted
    probabilities reaching top_p, first entry always kept), renormalised.
    """
    L.require_cuda(logits)
    T, tp, tk = _knobs(temperature, top_p, top_k)
    x = _rows(logits)
    n, V = x.shape
    out = torch.empty((n, V), dtype=torch.float32, device=x.device)
    code = L.dtype_code(x.dtype)
    lib = L.lib()
    with torch.cuda.device(x.device):
        ws = L.workspaces.get(lib.sd_sampling_workspace_bytes(n, n, V, code), x.device)
        L.check(lib.sd_to_probs(L.ptr(x), x.stride(0), code, n, V, T, tp, tk, L.ptr(out),
                                out.stride(0), L.ptr(ws), ws.numel(), L.stream_ptr(x.device)),
                "to_probs")
    return out.reshape(logits.shape)


def sample_from_probs(probs, generator=None, u=None):
    """Inverse-CDF draw per row: probs [..., V] -> ids [...] (int64).

    Replaces reference specdec/sampling.py:70-74 (torch.multinomial).  The
    uniforms are ``u`` if given, else drawn from ``generator`` on the device.
    """
    L.require_cuda(probs)
    p = _rows(probs.float())
    n, V = p.shape
    if u is None:
        u = torch.rand(n, generator=generator, device=p.device)
    u = u.reshape(-1).float().contiguous()
    out = torch.empty(n, dtype=torch.long, device=p.device)
    with torch.cuda.device(p.device):
        L.check(L.lib().sd_sample_from_probs(L.ptr(p.contiguous()), n, V, L.ptr(u), L.ptr(out),
                                             L.stream_ptr(p.device)), "sample_from_probs")
    return out.reshape(probs.shape[:-1])


def residual_probs(p, q):
    """norm((p - q)_+), p itself where that sums to <= 1e-9 (sampling.py:77-90)."""
    L.require_cuda(p, q)
    p2 = _rows(p.float()).contiguous()
    q2 = _rows(q.float()).contiguous()
    n, V = p2.shape
    out = torch.empty_like(p2)
    with torch.cuda.device(p2.device):
        L.check(L.lib().sd_residual_probs(L.ptr(p2), L.ptr(q2), n, V, L.ptr(out),
                                          L.stream_ptr(p2.device)), "residual_probs")
    return out.reshape(p.shape)


def gather_prob(probs, ids):
    """probs [..., V], ids [...] -> probs at ids (sampling.py:93-95)."""
    L.require_cuda(probs, ids)
    p2 = _rows(probs.float()).contiguous()
    i2 = ids.reshape(-1).long().contiguous()
    out = torch.empty(i2.shape[0], dtype=torch.float32, device=p2.device)
    with torch.cuda.device(p2.device):
        L.check(L.lib().sd_gather_prob(L.ptr(p2), p2.shape[0], p2.shape[1], L.ptr(i2), L.ptr(out),
                                       L.stream_ptr(p2.device)), "gather_prob")
    return out.reshape(ids.shape)


def _vocab_rows(x, name):
    if x.stride(-1) != 1:
        raise L.SpecdecError(f"{name} must be contiguous along the vocabulary")
    return x


def verify_sample(target_logits, draft_logits, draft_ids, u_acc, u_res, temperature=1.0,
                  top_p=1.0, top_k=0, alive=None, return_probs=False):
    """The fused verify round (reference engine.py:282-303).

    target_logits [B, k+1, V] (p_1..p_{k+1}), draft_logits [B, k, V] (q_1..q_k;
    ignored when temperature <= 0), draft_ids [B, k], u_acc [B, k] and u_res [B]
    float uniforms, alive [B] bool or None.  Returns (n_acc [B], y [B]) int64,
    plus (p_i(x_i), q_i(x_i)) [B, k] float32 when return_probs.
    """
    L.require_cuda(target_logits, draft_ids, u_acc, u_res)
    B, k1, V = target_logits.shape
    k = k1 - 1
    greedy = temperature is None or temperature <= 0.0
    T, tp, tk = _knobs(temperature, top_p, top_k)
    tgt = _vocab_rows(target_logits, "target_logits")
    if greedy:
        drf = None
        dbs = dps = 0
    else:
        L.require_cuda(draft_logits)
        drf = _vocab_rows(draft_logits, "draft_logits")
        if drf.shape != (B, k, V) or drf.dtype != tgt.dtype:
            raise L.SpecdecError("draft_logits must be [B, k, V] with the target's dtype")
        dbs, dps = drf.stride(0), drf.stride(1)
    xs = draft_ids.long()
    if xs.stride(-1) != 1:
        xs = xs.contiguous()
    ua = u_acc.float()
    if ua.stride(-1) != 1:
        ua = ua.contiguous()
    ur = u_res.float().contiguous()
    al = None if alive is None else alive.to(torch.uint8).contiguous()
    dev = tgt.device
    n_acc = torch.empty(B, dtype=torch.long, device=dev)
    y = torch.empty(B, dtype=torch.long, device=dev)
    px = torch.empty(B, k, dtype=torch.float32, device=dev) if return_probs else None
    qx = torch.empty(B, k, dtype=torch.float32, device=dev) if return_probs else None
    code = L.dtype_code(tgt.dtype)
    lib = L.lib()
    nvec = B * (k + 1) if greedy else B * (2 * k + 1)
    with torch.cuda.device(dev):
        ws = L.workspaces.get(lib.sd_sampling_workspace_bytes(B, nvec, V, code), dev)
        L.check(lib.sd_verify_sample(L.ptr(tgt), tgt.stride(0), tgt.stride(1), L.ptr(drf), dbs,
                                     dps, code, L.ptr(xs), xs.stride(0), L.ptr(ua), ua.stride(0),
                                     L.ptr(ur), L.ptr(al), B, k, V, T, tp, tk, L.ptr(n_acc),
                                     L.ptr(y), L.ptr(px), L.ptr(qx), L.ptr(ws), ws.numel(),
                                     L.stream_ptr(dev)), "verify_sample")
    if return_probs:
        return n_acc, y, px, qx
    return n_acc, y


def verify_sample_probs(target_logits, draft_probs, draft_ids, u_acc, u_res, temperature=1.0,
                        top_p=1.0, top_k=0, alive=None, return_probs=False):
    """The fused verify round with the draft distributions given as
    probabilities: q_i = draft_probs[:, i] (fp32 [B, k, V], used as given),
    as a serving engine's rejection sampler holds them.  Otherwise as
    ``verify_sample``: to_probs (temperature, top-p, top-k) on the target
    logits [B, k+1, V], the accept test u < min(1, p(x)/max(q(x), 1e-10)), the
    residual draw from norm((p - q)+) at the first rejection or the bonus draw
    from p_k (reference engine.py:282-303).  Returns (n_acc, y) int64, plus
    (p_i(x_i), q_i(x_i)) when return_probs.
    """
    L.require_cuda(target_logits, draft_ids, u_acc, u_res)
    B, k1, V = target_logits.shape
    k = k1 - 1
    T, tp, tk = _knobs(temperature, top_p, top_k)
    tgt = _vocab_rows(target_logits, "target_logits")
    q = None
    if T > 0.0:
        L.require_cuda(draft_probs)
        if draft_probs.shape != (B, k, V) or draft_probs.dtype != torch.float32:
            raise L.SpecdecError("draft_probs must be float32 [B, k, V]")
        q = _vocab_rows(draft_probs, "draft_probs")
    xs = draft_ids.long()
    if xs.stride(-1) != 1:
        xs = xs.contiguous()
    ua = u_acc.float()
    if ua.stride(-1) != 1:
        ua = ua.contiguous()
    ur = u_res.float().contiguous()
    al = None if alive is None else alive.to(torch.uint8).contiguous()
    dev = tgt.device
    n_acc = torch.empty(B, dtype=torch.long, device=dev)
    y = torch.empty(B, dtype=torch.long, device=dev)
    px = torch.empty(B, k, dtype=torch.float32, device=dev) if return_probs else None
    qx = torch.empty(B, k, dtype=torch.float32, device=dev) if return_probs else None
    code = L.dtype_code(tgt.dtype)
    lib = L.lib()
    with torch.cuda.device(dev):
        ws = L.workspaces.get(lib.sd_sampling_workspace_bytes(B, B * (k + 1), V, code), dev)
        L.check(lib.sd_verify_sample_qprobs(
            L.ptr(tgt), tgt.stride(0), tgt.stride(1), code, L.ptr(q),
            0 if q is None else q.stride(0), 0 if q is None else q.stride(1), L.ptr(xs),
            xs.stride(0), L.ptr(ua), ua.stride(0), L.ptr(ur), L.ptr(al), B, k, V, T, tp, tk,
            L.ptr(n_acc), L.ptr(y), L.ptr(px), L.ptr(qx), L.ptr(ws), ws.numel(),
            L.stream_ptr(dev)), "verify_sample_probs")
    if return_probs:
        return n_acc, y, px, qx
    return n_acc, y


def draft_sample(logits, u, temperature=1.0, top_p=1.0, top_k=0):
    """x ~ to_probs(logits) by inverse CDF with uniforms u; returns (x, q(x)).

    logits [B, V] (row stride free, vocabulary contiguous), u [B].
    """
    L.require_cuda(logits, u)
    x2 = _vocab_rows(logits, "logits")
    if x2.dim() != 2:
        raise L.SpecdecError("draft_sample expects [B, V] logits")
    B, V = x2.shape
    T, tp, tk = _knobs(temperature, top_p, top_k)
    uu = u.reshape(-1).float().contiguous()
    x = torch.empty(B, dtype=torch.long, device=x2.device)
    qx = torch.empty(B, dtype=torch.float32, device=x2.device)
    code = L.dtype_code(x2.dtype)
    lib = L.lib()
    with torch.cuda.device(x2.device):
        ws = L.workspaces.get(lib.sd_sampling_workspace_bytes(B, B, V, code), x2.device)
        L.check(lib.sd_draft_sample(L.ptr(x2), x2.stride(0), code, B, V, L.ptr(uu), T, tp, tk,
                                    L.ptr(x), L.ptr(qx), L.ptr(ws), ws.numel(),
                                    L.stream_ptr(x2.device)), "draft_sample")
    return x, qx
