"""Generate the golden fixtures that pin the CPU oracle to the real reference.

Run in a container where the reference checkout is available:

    python tests/golden/make_golden.py --ref <path to adaptive-specdec checkout>

It imports the reference's own ``specdec`` package read-only and calls its
``to_probs`` / ``residual_probs`` / ``gather_prob`` (specdec/sampling.py:34-95),
``RaggedCache`` (specdec/kvcache.py:98-202) and controllers
(specdec/controller.py:47-251) on seeded inputs, and stores inputs plus outputs
as small ``.npz`` / ``.json`` files next to this script.  Nothing at test time
reads the reference; the tests only read these fixtures.

Two harness shims, applied to the imported modules only (no file is changed):

* ``torch.sort`` inside the reference's sampling module is forced to
  ``stable=True`` for the "stable" fixtures, which defines the tie order at the
  nucleus boundary (ascending vocabulary index).  Fixtures from the unmodified
  module are stored too, with a flag per vector telling whether the two differ.
* ``sample_from_probs`` (torch.multinomial) is replaced in the verify harness by
  an inverse-CDF draw with the uniform passed in, in float64 and vocabulary
  order, so the draw is a function of the stored uniforms.
"""
import argparse
import importlib
import json
import pathlib
import sys
import types

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent


def load_reference(ref):
    sys.path.insert(0, str(ref))
    sampling = importlib.import_module("specdec.sampling")
    controller = importlib.import_module("specdec.controller")
    kvcache = importlib.import_module("specdec.kvcache")
    return sampling, controller, kvcache


class _StableTorch(types.ModuleType):
    """Proxy for the torch module that forces stable sorting."""

    def __init__(self):
        super().__init__("torch_stable_proxy")

    def __getattr__(self, name):
        if name == "sort":
            def sort(x, dim=-1, descending=False, stable=None):
                return torch.sort(x, dim=dim, descending=descending, stable=True)
            return sort
        return getattr(torch, name)


def bf16r(t):
    return t.to(torch.bfloat16).to(torch.float32)


def zipf_logits(gen, n, V, noise=3.0, s=1.1):
    """N(0, noise^2) plus a per-row Zipf(s) log-prior over a random permutation."""
    base = torch.randn(n, V, generator=gen) * noise
    ranks = torch.arange(1, V + 1, dtype=torch.float64)
    prior = (-s * torch.log(ranks)).float()
    out = torch.empty(n, V)
    for r in range(n):
        perm = torch.randperm(V, generator=gen)
        out[r] = base[r] + prior[perm]
    return out


def icdf(probs, u):
    """Inverse CDF over float32 probs with float64 running sum, vocabulary order."""
    p = probs.double()
    c = p.cumsum(-1)
    t = u.double().unsqueeze(-1) * p.sum(-1, keepdim=True)
    j = (c <= t).sum(-1)
    last_nz = (p > 0).long().cumsum(-1).argmax(-1)
    return torch.where(j >= p.shape[-1], last_nz, j)


def ref_verify(S, tgt, drf, xs, u_acc, u_res, T, top_p, top_k):
    """reference specdec/engine.py:282-303, uniforms as tensors."""
    B, k1, V = tgt.shape
    k = k1 - 1
    ps = [S.to_probs(tgt[:, i], T, top_p, top_k) for i in range(k + 1)]
    qs = [S.to_probs(drf[:, i], T, top_p, top_k) for i in range(k)]
    n_acc = torch.zeros(B, dtype=torch.long)
    alive = torch.ones(B, dtype=torch.bool)
    for i in range(k):
        ratio = S.gather_prob(ps[i], xs[:, i]) / S.gather_prob(qs[i], xs[:, i]).clamp_min(1e-10)
        ok = (u_acc[:, i] < ratio.clamp(max=1.0)) & alive & (n_acc == i)
        n_acc = n_acc + ok.long()
        alive = alive & ok
    all_acc = n_acc == k
    pick = n_acc.clamp(max=k - 1)
    p_stop = torch.stack(ps[:k], 1)[torch.arange(B), pick]
    q_stop = torch.stack(qs, 1)[torch.arange(B), pick]
    y_res = icdf(S.residual_probs(p_stop, q_stop), u_res)
    y_bonus = icdf(ps[k], u_res)
    y = torch.where(all_acc, y_bonus, y_res)
    return n_acc, y, torch.stack(ps, 1), torch.stack(qs, 1)


def make_to_probs(S_stable, S_plain):
    g = torch.Generator().manual_seed(1234)
    cases = []
    cases.append(("v16_t1", torch.randn(4, 16, generator=g) * 1.5, 1.0, 1.0, 0))
    cases.append(("v32_t1_tp09", torch.randn(8, 32, generator=g) * 2.0, 1.0, 0.9, 0))
    cases.append(("v32_t07_tp05_tk5", torch.randn(8, 32, generator=g) * 2.0, 0.7, 0.5, 5))
    cases.append(("v1000_bf16_t07_tp09", bf16r(torch.randn(6, 1000, generator=g) * 3.0), 0.7, 0.9, 0))
    cases.append(("v1000_bf16_t13_tp08_tk50", bf16r(torch.randn(6, 1000, generator=g) * 3.0), 1.3, 0.8, 50))
    cases.append(("v1000_bf16_tk7", bf16r(torch.randn(4, 1000, generator=g) * 2.0), 1.0, 1.0, 7))
    gr = bf16r(torch.randn(6, 64, generator=g))
    gr[0, 10] = gr[0, 40] = gr[0].max() + 1.0          # tied maximum: first index wins
    cases.append(("v64_greedy_ties", gr, 0.0, 0.9, 5))
    cases.append(("v4096_bf16_zipf_t07_tp09", bf16r(zipf_logits(g, 8, 4096)), 0.7, 0.9, 0))
    cases.append(("v4096_bf16_zipf_t1_tp095_tk100", bf16r(zipf_logits(g, 4, 4096)), 1.0, 0.95, 100))
    out = {}
    for name, x, T, tp, tk in cases:
        st = S_stable.to_probs(x, T, tp, tk)
        pl = S_plain.to_probs(x, T, tp, tk)
        out[name + "__x"] = x.numpy()
        out[name + "__stable"] = st.numpy()
        out[name + "__plain"] = pl.numpy()
        out[name + "__params"] = np.array([T, tp, tk], dtype=np.float64)
        out[name + "__tiediff"] = ((st > 0) != (pl > 0)).any(-1).numpy()
    np.savez_compressed(HERE / "to_probs.npz", names=np.array([c[0] for c in cases]), **out)


def make_residual(S):
    g = torch.Generator().manual_seed(99)
    p = S.to_probs(torch.randn(6, 32, generator=g) * 2, 1.0, 0.9)
    q = S.to_probs(torch.randn(6, 32, generator=g) * 2, 1.0, 0.9)
    q[0] = p[0]                                          # degenerate row: falls back to p
    oh = torch.zeros(1, 32)
    oh[0, 7] = 1.0
    p = torch.cat([p, oh])
    q = torch.cat([q, oh])                               # one-hot equal pair (greedy)
    r = S.residual_probs(p, q)
    ids = torch.randint(0, 32, (7,), generator=g)
    np.savez_compressed(HERE / "residual.npz", p=p.numpy(), q=q.numpy(), r=r.numpy(),
                        ids=ids.numpy(), gathered=S.gather_prob(p, ids).numpy())


def make_verify(S_stable, S_plain):
    cases = {}

    def one(name, tgt, drf, T, tp, tk, seed):
        g = torch.Generator().manual_seed(seed)
        B, k1, V = tgt.shape
        k = k1 - 1
        q_for_draw = torch.stack([S_stable.to_probs(drf[:, i], T, tp, tk) for i in range(k)], 1)
        xs = torch.multinomial(q_for_draw.reshape(-1, V), 1, generator=g).reshape(B, k)
        u_acc = torch.rand(B, k, generator=g)
        u_res = torch.rand(B, generator=g)
        n_acc, y, P, Q = ref_verify(S_stable, tgt, drf, xs, u_acc, u_res, T, tp, tk)
        n_acc_p, y_p, _, _ = ref_verify(S_plain, tgt, drf, xs, u_acc, u_res, T, tp, tk)
        cases[name] = dict(tgt=tgt.numpy(), drf=drf.numpy(), xs=xs.numpy(), u_acc=u_acc.numpy(),
                           u_res=u_res.numpy(), n_acc=n_acc.numpy(), y=y.numpy(),
                           n_acc_plain=n_acc_p.numpy(), y_plain=y_p.numpy(),
                           params=np.array([T, tp, tk], dtype=np.float64),
                           P=P.numpy(), Q=Q.numpy())

    # Config 1: B=8, k=4, V=32 fp32, N(0, 2^2) from seed 0, T=1.0, top-p 1.0.
    torch.manual_seed(0)
    tgt = torch.randn(8, 5, 32) * 2.0
    drf = torch.randn(8, 4, 32) * 2.0
    one("cfg1_v32", tgt, drf, 1.0, 1.0, 0, seed=7)
    # tests/tiny.py scale (V=16)
    torch.manual_seed(0)
    one("cfg1_v16", torch.randn(8, 5, 16) * 2.0, torch.randn(8, 4, 16) * 2.0, 1.0, 1.0, 0, seed=8)
    # sampling knobs on the tiny shape
    torch.manual_seed(1)
    t1 = torch.randn(8, 5, 32) * 2.0
    one("v32_t07_tp09", t1, t1[:, :4] + 0.5 * torch.randn(8, 4, 32), 0.7, 0.9, 0, seed=9)
    # greedy
    torch.manual_seed(2)
    t2 = bf16r(torch.randn(8, 5, 64) * 2.0)
    one("v64_greedy", t2, bf16r(t2[:, :4] + 0.7 * torch.randn(8, 4, 64)), 0.0, 1.0, 0, seed=10)
    # bf16 Zipf-peaked medium case with nucleus ties
    g = torch.Generator().manual_seed(3)
    zt = bf16r(zipf_logits(g, 16 * 5, 4096)).reshape(16, 5, 4096)
    zd = bf16r(zt[:, :4] + torch.randn(16, 4, 4096, generator=g) * 1.0)
    one("v4096_bf16_zipf_t07_tp09", zt, zd, 0.7, 0.9, 0, seed=11)
    flat = {}
    for name, d in cases.items():
        for key, val in d.items():
            flat[f"{name}__{key}"] = val
    np.savez_compressed(HERE / "verify.npz", names=np.array(list(cases)), **flat)


def make_verify_cfg2(S_stable, S_plain):
    """Config 2 at the full Qwen3 vocabulary (V = 151936), 8 rows: sampling at
    T = 0.7 / top-p 0.9 and greedy, through the reference's own functions.
    Inputs are regenerated by tests/golden/cfg2_inputs.py from the seed; only
    draws, uniforms, outputs and a checksum are stored."""
    sys.path.insert(0, str(HERE))
    import cfg2_inputs as CI
    tgt, drf = CI.cfg2_rows()
    B, k1, V = tgt.shape
    k = k1 - 1
    g = torch.Generator().manual_seed(77)
    out = {"tgt_sum": np.float64(CI.checksum(tgt)), "drf_sum": np.float64(CI.checksum(drf))}
    for name, T, tp in (("t07_tp09", 0.7, 0.9), ("greedy", 0.0, 1.0)):
        q_draw = torch.stack([S_stable.to_probs(drf[:, i], max(T, 0.7), 0.9) for i in range(k)], 1)
        xs = torch.multinomial(q_draw.reshape(-1, V), 1, generator=g).reshape(B, k)
        if T == 0.0:                                   # greedy rows: half the drafts are the argmax
            am = tgt[:, :k].argmax(-1)
            xs = torch.where(torch.rand(B, k, generator=g) < 0.5, am, xs)
        u_acc = torch.rand(B, k, generator=g)
        u_res = torch.rand(B, generator=g)
        n_acc, y, P, Q = ref_verify(S_stable, tgt, drf, xs, u_acc, u_res, T, tp, 0)
        n_acc_p, y_p, _, _ = ref_verify(S_plain, tgt, drf, xs, u_acc, u_res, T, tp, 0)
        bi = torch.arange(B)[:, None]
        pi = torch.arange(k)[None, :]
        out.update({f"{name}__xs": xs.numpy(), f"{name}__u_acc": u_acc.numpy(),
                    f"{name}__u_res": u_res.numpy(), f"{name}__n_acc": n_acc.numpy(),
                    f"{name}__y": y.numpy(), f"{name}__n_acc_plain": n_acc_p.numpy(),
                    f"{name}__y_plain": y_p.numpy(),
                    f"{name}__px": P[bi, pi, xs].numpy(), f"{name}__qx": Q[bi, pi, xs].numpy(),
                    f"{name}__nkeep_p": (P > 0).sum(-1).numpy(),
                    f"{name}__nkeep_q": (Q > 0).sum(-1).numpy()})
    np.savez_compressed(HERE / "verify_cfg2.npz", **out)


def make_kvcache(K):
    """RaggedCache length bookkeeping (kvcache.py:165-202) and mask (:138-162)."""
    c = K.RaggedCache(2, 3, 32, torch.device("cpu"))
    trace = []
    c.set_lengths(torch.tensor([7, 5, 6]))
    trace.append(("set_lengths", [7, 5, 6], c.lengths.tolist()))
    c.advance(4)
    trace.append(("advance", 4, c.lengths.tolist()))
    c.rollback([0, 3, 2])
    trace.append(("rollback", [0, 3, 2], c.lengths.tolist()))
    c.rollback(1)
    trace.append(("rollback", 1, c.lengths.tolist()))
    c.rollback(torch.tensor([1, 0, 1]))
    trace.append(("rollback", [1, 0, 1], c.lengths.tolist()))
    pos = c.positions(3).tolist()
    cpos = c.cache_position(3).tolist()
    mask = c.attn_mask(3, torch.float32)
    mask_valid = c.attn_mask(3, torch.float32, valid=torch.tensor([9, 4, 6]))
    raised = False
    try:
        c.rollback([100, 0, 0])
    except RuntimeError:
        raised = True
    out = dict(trace=trace, positions=pos, cache_position=cpos, kv_len_for_3=c.kv_len_for(3),
               mask_allowed=(mask == 0).tolist(), mask_valid_allowed=(mask_valid == 0).tolist(),
               raises_below_zero=raised)
    c2 = K.RaggedCache(1, 2, 16, torch.device("cpu"))
    c2.set_lengths([4, 4])
    out["uniform_mask_is_none"] = c2.attn_mask(2, torch.float32) is None
    (HERE / "kvcache.json").write_text(json.dumps(out, indent=1))


def make_controller(C):
    grid = []
    for a in (0.05, 0.3, 0.45, 0.55, 0.7, 0.78, 0.9, 0.98):
        for c in (0.05, 0.12, 0.15, 0.25, 0.5, 1.0, 1.6):
            for ef in (0, 1):
                grid.append([a, c, ef, C.best_k(a, c, 8, ef),
                             [C.expected_speedup(k, a, c, ef) for k in range(1, 9)]])
    rng = np.random.default_rng(5)
    ew = C.EWMAAnalytic(k_max=8, beta=0.95, warmup=3)
    ew_trace = []
    for r in range(60):
        k = ew.propose_k()
        n_acc = [int(v) for v in rng.integers(0, k + 1, size=3)]
        dt = float(rng.uniform(0.5, 1.5))
        tdf, ttf = float(rng.uniform(0.05, 0.3)), 1.0
        ew.update(k, n_acc, dt, t_draft_fwd=tdf, t_target_fwd=ttf)
        ew_trace.append([k, n_acc, dt, tdf, ttf, ew.alpha, ew.c])
    ucb = C.UCBBandit(k_max=5)
    ucb_trace = []
    for r in range(40):
        k = ucb.propose_k()
        n_acc = [int(v) for v in rng.integers(0, k + 1, size=2)]
        dt = float(rng.uniform(0.5, 1.5))
        ucb.update(k, n_acc, dt)
        ucb_trace.append([k, n_acc, dt, {str(kk): v for kk, v in ucb.mu.items()}])
    ee = C.ConfidenceEarlyExit(C.FixedK(6), tau=0.4, min_k=2)
    ee_cases = [[i, conf, ee.should_stop_drafting(i, torch.tensor(conf))]
                for i in (0, 1, 2, 3) for conf in ([0.1, 0.2], [0.5, 0.6], [0.39], [0.41])]
    specs = {s: C.make_controller(s).state()["name"] for s in ("fixed3", "ewma", "ewma+exit", "ucb")}
    (HERE / "controller.json").write_text(json.dumps(dict(
        best_k_grid=grid, ewma_trace=ew_trace, ucb_trace=ucb_trace, early_exit=ee_cases,
        make_controller_names=specs), indent=1))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to the reference checkout")
    args = ap.parse_args()
    sampling, controller, kvcache = load_reference(pathlib.Path(args.ref))
    stable = types.ModuleType("ref_sampling_stable")
    stable.__dict__.update(sampling.__dict__)
    stable.torch = _StableTorch()
    for fn in ("to_probs", "sample_from_probs", "residual_probs", "gather_prob"):
        f = getattr(sampling, fn)
        setattr(stable, fn, types.FunctionType(f.__code__, stable.__dict__, fn, f.__defaults__))
    torch.set_num_threads(4)
    make_to_probs(stable, sampling)
    make_residual(sampling)
    make_verify(stable, sampling)
    make_verify_cfg2(stable, sampling)
    make_kvcache(kvcache)
    make_controller(controller)
    for p in sorted(HERE.glob("*.*")):
        print(f"{p.name:24s} {p.stat().st_size:>9d} B")


if __name__ == "__main__":
    main()
