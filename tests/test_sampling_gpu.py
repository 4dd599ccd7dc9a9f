"""GPU parity of the verify-round sampling kernels against the CPU oracle.

Bar (from the task's parity contract):
* accept counts and emitted tokens bit-exact, except rows whose decision sits
  within 1e-6 of a boundary: |u - min(1, p/q)| < 1e-6 at a tested position, an
  inverse-CDF crossing within 1e-6 * total of u * total, or a top-p edge
  |fl32(cum - p) - top_p| < 1e-6 on a vector the row used;
* probabilities within 1e-5 relative (the contract asks 1e-3);
* the statistical rejection-rule test (TV <= 0.02, here 0.01) on the kernels.

Inputs are seeded; the oracle is oracle/sampling_oracle.py, itself pinned to
the reference by tests/test_oracle_golden.py.
"""
import numpy as np
import pytest
import torch

from oracle import sampling_oracle as O
from specdec import sampling as S
from specdec import workloads as W
from tests.golden import GOLDEN

pytestmark = pytest.mark.gpu
EPS = 1e-6
PREL = 1e-5
DEV = "cuda"


def _np(t):
    return t.detach().float().cpu().numpy()


def _ok(d):
    return (d["acc_margin"] > EPS) & (d["cdf_margin"] > EPS) & (d["topp_margin"] > EPS)


def _check_verify(tgt, drf, xs, ua, ur, T, tp, tk, max_exempt=0.1, tag=""):
    """Kernel vs oracle on the same (already device-resident) inputs."""
    n_k, y_k, px_k, qx_k = S.verify_sample(tgt, drf, xs, ua, ur, T, tp, tk, return_probs=True)
    n_o, y_o, d = O.verify(_np(tgt), _np(drf), xs.cpu().numpy(), _np(ua), _np(ur), T, tp, tk,
                           return_details=True)
    ok = _ok(d)
    assert ok.mean() >= 1.0 - max_exempt, f"{tag}: too many boundary rows {(~ok).sum()}"
    n_k, y_k = n_k.cpu().numpy(), y_k.cpu().numpy()
    bad = np.nonzero(ok & ((n_k != n_o) | (y_k != y_o)))[0]
    assert bad.size == 0, (f"{tag}: rows {bad[:8]} differ: kernel n/y "
                           f"{n_k[bad[:8]]}/{y_k[bad[:8]]} oracle {n_o[bad[:8]]}/{y_o[bad[:8]]}")
    if T is not None and T > 0:
        px_k, qx_k = px_k.cpu().numpy(), qx_k.cpu().numpy()
        sel = ok[:, None] & np.ones_like(px_k, dtype=bool)
        np.testing.assert_allclose(px_k[sel], d["px"][sel], rtol=2e-6, atol=1e-30, err_msg=tag)
        np.testing.assert_allclose(qx_k[sel], d["qx"][sel], rtol=2e-6, atol=1e-30, err_msg=tag)
    return n_k, y_k, ok


# ---------------------------------------------------------------------------
# golden cases (pinned to the reference)
# ---------------------------------------------------------------------------
_VZ = np.load(GOLDEN / "verify.npz")


@pytest.mark.parametrize("case", [str(n) for n in _VZ["names"]])
def test_verify_golden(case):
    g = {k: _VZ[f"{case}__{k}"] for k in ("tgt", "drf", "xs", "u_acc", "u_res", "n_acc", "y",
                                          "params")}
    T, tp, tk = (float(g["params"][0]), float(g["params"][1]), int(g["params"][2]))
    dt = torch.bfloat16 if "bf16" in case or "greedy" in case else torch.float32
    tgt = torch.from_numpy(g["tgt"]).to(DEV, dt)
    drf = torch.from_numpy(g["drf"]).to(DEV, dt)
    xs = torch.from_numpy(g["xs"]).to(DEV)
    ua = torch.from_numpy(g["u_acc"]).to(DEV)
    ur = torch.from_numpy(g["u_res"]).to(DEV)
    n_k, y_k, ok = _check_verify(tgt, drf, xs, ua, ur, T, tp, tk, max_exempt=0.25, tag=case)
    # and directly against the reference's own outputs
    np.testing.assert_array_equal(n_k[ok], g["n_acc"][ok])
    np.testing.assert_array_equal(y_k[ok], g["y"][ok])


_TZ = np.load(GOLDEN / "to_probs.npz")


@pytest.mark.parametrize("case", [str(n) for n in _TZ["names"]])
def test_to_probs_golden(case):
    x = _TZ[case + "__x"]
    T, tp, tk = _TZ[case + "__params"]
    dt = torch.bfloat16 if "bf16" in case or "greedy" in case else torch.float32
    got = _np(S.to_probs(torch.from_numpy(x).to(DEV, dt), float(T), float(tp), int(tk)))
    infos = []
    want = O.to_probs(x, float(T), float(tp), int(tk), infos=infos)
    ref = _TZ[case + "__stable"]
    for r in range(x.shape[0]):
        if infos[r].topp_margin < EPS:
            continue
        np.testing.assert_array_equal(got[r] > 0, want[r] > 0, err_msg=f"{case} row {r}")
        np.testing.assert_allclose(got[r], want[r], rtol=PREL, atol=0, err_msg=f"{case} row {r}")
        np.testing.assert_allclose(got[r], ref[r], rtol=PREL, atol=1e-12, err_msg=f"{case} ref")


# ---------------------------------------------------------------------------
# config 2 at full size (B=64, k=4, V=151936 bf16) and the greedy case
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg2():
    tgt, drf = W.cfg2_logits(seed=0)
    ua, ur = W.uniforms(64, 4, seed=0)
    xs, _ = S.draft_sample(drf.reshape(-1, drf.shape[-1]), torch.rand(
        256, generator=torch.Generator(device=DEV).manual_seed(3), device=DEV), 0.7, 0.9)
    return tgt, drf, xs.reshape(64, 4), ua, ur


def test_cfg2_reference_golden_full_vocab():
    """Config 2 at V = 151936 against outputs the reference's own to_probs and
    accept loop produced (tests/golden/verify_cfg2.npz, 8 rows; sampling at
    T = 0.7 / top-p 0.9 and greedy).  Rows inside the contract's 1e-6
    exemption margins (computed by the oracle) may differ."""
    from tests.golden import cfg2_inputs as CI
    z = np.load(GOLDEN / "verify_cfg2.npz")
    tgt, drf = CI.cfg2_rows()
    assert CI.checksum(tgt) == float(z["tgt_sum"]), "input generator changed"
    td, dd = tgt.to(DEV, torch.bfloat16), drf.to(DEV, torch.bfloat16)
    for name, T, tp in (("t07_tp09", 0.7, 0.9), ("greedy", 0.0, 1.0)):
        xs = torch.from_numpy(z[name + "__xs"]).to(DEV)
        ua = torch.from_numpy(z[name + "__u_acc"]).to(DEV)
        ur = torch.from_numpy(z[name + "__u_res"]).to(DEV)
        n_k, y_k, px_k, qx_k = S.verify_sample(td, dd, xs, ua, ur, T, tp, return_probs=True)
        _, _, d = O.verify(tgt.numpy(), drf.numpy(), z[name + "__xs"], z[name + "__u_acc"],
                           z[name + "__u_res"], T, tp, 0, return_details=True)
        ok = _ok(d)
        assert ok.mean() >= 0.75, name
        n_k, y_k = n_k.cpu().numpy(), y_k.cpu().numpy()
        np.testing.assert_array_equal(n_k[ok], z[name + "__n_acc"][ok], err_msg=name)
        np.testing.assert_array_equal(y_k[ok], z[name + "__y"][ok], err_msg=name)
        if T > 0:
            np.testing.assert_allclose(px_k.cpu().numpy()[ok], z[name + "__px"][ok], rtol=2e-6,
                                       atol=1e-30, err_msg=name)
            np.testing.assert_allclose(qx_k.cpu().numpy()[ok], z[name + "__qx"][ok], rtol=2e-6,
                                       atol=1e-30, err_msg=name)


def test_cfg2_sampling_parity(cfg2):
    tgt, drf, xs, ua, ur = cfg2
    n_k, y_k, ok = _check_verify(tgt, drf, xs, ua, ur, 0.7, 0.9, 0, max_exempt=0.05, tag="cfg2")
    assert len(set(n_k.tolist())) >= 3, "instance should exercise several accept lengths"


def test_cfg2_greedy_parity(cfg2):
    tgt, drf, xs, ua, ur = cfg2
    am = tgt.float().argmax(-1)                    # [64, 5]
    xs_g = torch.where(torch.rand(64, 4, device=DEV) < 0.7, am[:, :4], xs)
    _check_verify(tgt, drf, xs_g, ua, ur, 0.0, 1.0, 0, max_exempt=0.0, tag="greedy")


def _check_verify_probs(tgt, drf, xs, ua, ur, T, tp, tk, max_exempt=0.1, tag=""):
    """verify_sample_probs with q = to_probs(draft logits) on the kernels vs the
    oracle's verify from the draft logits: the same q, so the same results."""
    B, k, V = drf.shape
    q = S.to_probs(drf, T, tp, tk).reshape(B, k, V)
    n_k, y_k, px_k, qx_k = S.verify_sample_probs(tgt, q, xs, ua, ur, T, tp, tk, return_probs=True)
    n_o, y_o, d = O.verify(_np(tgt), _np(drf), xs.cpu().numpy(), _np(ua), _np(ur), T, tp, tk,
                           return_details=True)
    ok = _ok(d)
    assert ok.mean() >= 1.0 - max_exempt, f"{tag}: too many boundary rows {(~ok).sum()}"
    n_k, y_k = n_k.cpu().numpy(), y_k.cpu().numpy()
    bad = np.nonzero(ok & ((n_k != n_o) | (y_k != y_o)))[0]
    assert bad.size == 0, (f"{tag}: rows {bad[:8]} differ: kernel n/y "
                           f"{n_k[bad[:8]]}/{y_k[bad[:8]]} oracle {n_o[bad[:8]]}/{y_o[bad[:8]]}")
    px_k, qx_k = px_k.cpu().numpy(), qx_k.cpu().numpy()
    sel = ok[:, None] & np.ones_like(px_k, dtype=bool)
    np.testing.assert_allclose(px_k[sel], d["px"][sel], rtol=2e-6, atol=1e-30, err_msg=tag)
    np.testing.assert_allclose(qx_k[sel], d["qx"][sel], rtol=2e-6, atol=1e-30, err_msg=tag)
    return n_k, y_k, ok


def test_cfg2_verify_with_draft_probabilities(cfg2):
    """The draft distributions given as probabilities (as a serving engine's
    rejection sampler holds them): config 2 at T = 0.7 / top-p 0.9."""
    tgt, drf, xs, ua, ur = cfg2
    n_k, _, _ = _check_verify_probs(tgt, drf, xs, ua, ur, 0.7, 0.9, 0, max_exempt=0.05,
                                    tag="cfg2 probs")
    assert len(set(n_k.tolist())) >= 3


@pytest.mark.parametrize("T,tp,tk,V", [(1.0, 1.0, 0, 32000), (1.2, 0.95, 50, 32000),
                                       (0.8, 1.0, 0, 151936)])
def test_verify_with_draft_probabilities_modes(T, tp, tk, V):
    """No truncation (every element kept), top-k with top-p, and the full
    vocabulary untruncated: each draws through the row pass from q as given."""
    g = torch.Generator().manual_seed(17)
    B, k = 12, 4
    tgt = W.zipf_logits(B * (k + 1), V, g).reshape(B, k + 1, V)
    drf = tgt[:, :k] + torch.randn(B, k, V, generator=g)
    tgt, drf = tgt.to(DEV, torch.bfloat16), drf.to(DEV, torch.bfloat16)
    am = tgt.float().argmax(-1)
    xs = torch.where(torch.rand(B, k, generator=g).to(DEV) < 0.5, am[:, :k],
                     torch.randint(0, V, (B, k), generator=g).to(DEV)).contiguous()
    ua = torch.rand(B, k, generator=g).to(DEV)
    ur = torch.rand(B, generator=g).to(DEV)
    _check_verify_probs(tgt, drf, xs, ua, ur, T, tp, tk, max_exempt=0.25, tag=f"probs {T} {tp} {tk}")


def test_verify_with_draft_probabilities_greedy(cfg2):
    """T = 0: the greedy round, the draft probabilities unused."""
    tgt, drf, xs, ua, ur = cfg2
    am = tgt.float().argmax(-1)
    xs_g = torch.where(torch.rand(64, 4, device=DEV) < 0.7, am[:, :4], xs)
    n_p, y_p = S.verify_sample_probs(tgt, None, xs_g, ua, ur, 0.0)
    n_l, y_l = S.verify_sample(tgt, None, xs_g, ua, ur, 0.0)
    assert torch.equal(n_p, n_l) and torch.equal(y_p, y_l)


def test_cfg2_topk_and_topp(cfg2):
    tgt, drf, xs, ua, ur = cfg2
    _check_verify(tgt[:16], drf[:16], xs[:16], ua[:16], ur[:16], 1.0, 0.8, 40, tag="topk40+topp")


def test_cfg2_to_probs_full_rows(cfg2):
    tgt = cfg2[0]
    x = tgt[:3].reshape(-1, tgt.shape[-1])[:8]
    got = _np(S.to_probs(x, 0.7, 0.9))
    infos = []
    want = O.to_probs(_np(x), 0.7, 0.9, infos=infos)
    for r in range(x.shape[0]):
        if infos[r].topp_margin < EPS:
            continue
        np.testing.assert_array_equal(got[r] > 0, want[r] > 0)
        np.testing.assert_allclose(got[r], want[r], rtol=PREL, atol=0)


# ---------------------------------------------------------------------------
# histogram-path edge cases
# ---------------------------------------------------------------------------
def _to_probs_case(x, T, tp, tk, dt=torch.bfloat16):
    xd = x.to(DEV, dt)
    got = _np(S.to_probs(xd, T, tp, tk))
    infos = []
    want = O.to_probs(_np(xd), T, tp, tk, infos=infos)
    for r in range(x.shape[0]):
        if infos[r].topp_margin < EPS:
            continue
        np.testing.assert_array_equal(got[r] > 0, want[r] > 0, err_msg=f"row {r}")
        np.testing.assert_allclose(got[r], want[r], rtol=PREL, atol=0, err_msg=f"row {r}")


def test_odd_vocab_unaligned_rows():
    g = torch.Generator().manual_seed(1)
    x = W.zipf_logits(6, 5003, g)                     # rows start off 16-byte boundaries
    _to_probs_case(x, 0.8, 0.9, 0)
    _to_probs_case(x, 1.0, 1.0, 17)


def test_counter_overflow_many_equal_values():
    """>65535 equal logits (e.g. masked vocabulary) take the wrap-logging path."""
    g = torch.Generator().manual_seed(2)
    V = 150000
    x = torch.full((3, V), -30.0)
    x[:, :2000] = torch.randn(3, 2000, generator=g) * 2
    x[1, 5000:] = -0.0
    x[1, 2000:5000] = 0.0
    _to_probs_case(x, 1.0, 0.95, 0)
    _to_probs_case(x, 0.7, 0.5, 100)


def test_signed_zero_is_one_tie_class():
    V = 8192
    x = torch.zeros(2, V)
    x[:, ::2] = -0.0
    x[0, 7] = 3.0
    _to_probs_case(x, 1.0, 0.5, 0)


def test_fp16_logits():
    g = torch.Generator().manual_seed(4)
    x = W.zipf_logits(4, 32000, g)
    _to_probs_case(x, 0.7, 0.9, 0, dt=torch.float16)


def test_boundary_tie_class_index_order():
    """Many equal values at the nucleus edge: kept members are the lowest indices."""
    V = 10000
    x = torch.full((1, V), 1.0)
    x[0, 100] = 8.0
    _to_probs_case(x, 1.0, 0.5, 0)
    p = _np(S.to_probs(x.to(DEV, torch.bfloat16), 1.0, 0.5))[0]
    idx = np.nonzero(p > 0)[0]
    assert 100 in idx
    others = idx[idx != 100]
    expect = np.array([i for i in range(V) if i != 100][:others.size])
    assert others.size > 0 and np.array_equal(others, expect)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_greedy_argmax_ties_nan_and_alignment(dt):
    """Greedy (T = 0) picks the first index of the maximum, NaN counting as the
    maximum and -0 equal to +0, on rows whose starts fall at different 16-byte
    alignments (unaligned head and tail elements)."""
    V = 50000
    g = torch.Generator().manual_seed(9)
    base = torch.randn(7, V + 5, generator=g) * 3
    x = base[:, 3:3 + V]                              # row stride V + 5: varied alignment
    x[1, [40000, 17, 30000]] = 50.0                   # ties in different chunks
    x[2, 25000] = float("nan"); x[2, 30000] = float("nan"); x[2, 100] = 60.0
    x[3] = 0.0; x[3, ::3] = -0.0                      # one tie class of zeros
    x[4] = float("-inf")
    x[5, 0] = 70.0; x[5, V - 1] = 70.0                # head / tail tie
    x[6, V - 2] = 80.0                                # maximum in the tail
    xd = base.to(DEV, dt)[:, 3:3 + V]
    got = _np(S.to_probs(xd, 0.0)).argmax(-1)
    want = np.argmax(xd.float().cpu().numpy(), -1)
    np.testing.assert_array_equal(got, want)
    assert list(want[1:]) == [17, 25000, 0, 0, 0, V - 2]


def _greedy_ref(tgt, xs, ua, alive=None):
    """Greedy verify on torch: first-index argmax per vector, accepted prefix
    (x_i equal to the argmax and u_i < 1, while alive), emitted token."""
    am = tgt.float().argmax(-1)
    k = xs.shape[1]
    ok = (xs == am[:, :k]) & (ua < 1.0)
    if alive is not None:
        ok &= alive[:, None]
    n = torch.where(ok.all(-1), torch.full_like(xs[:, 0], k), (~ok).int().argmax(-1).long())
    return n, am.gather(1, n[:, None])[:, 0]


def _greedy_inputs(B, k, V, g, p_match=0.7):
    tgt = (torch.randn(B, k + 1, V, generator=g, device=DEV) * 3).to(torch.bfloat16)
    am = tgt.float().argmax(-1)
    xs = torch.where(torch.rand(B, k, generator=g, device=DEV) < p_match, am[:, :k],
                     torch.randint(0, V, (B, k), generator=g, device=DEV)).contiguous()
    return tgt, xs, torch.rand(B, k, generator=g, device=DEV), torch.rand(B, generator=g, device=DEV)


def _verify_ws(tgt, drf, xs, ua, ur, T, ws):
    """sd_verify_sample through the C ABI on a caller-given workspace."""
    from specdec import _lib as L
    B, k1, V = tgt.shape
    n = torch.full((B,), -1, dtype=torch.long, device=DEV)
    y = torch.full((B,), -1, dtype=torch.long, device=DEV)
    rc = L.lib().sd_verify_sample(
        L.ptr(tgt), tgt.stride(0), tgt.stride(1), L.ptr(drf), 0 if drf is None else drf.stride(0),
        0 if drf is None else drf.stride(1), L.dtype_code(tgt.dtype), L.ptr(xs), xs.stride(0),
        L.ptr(ua), ua.stride(0), L.ptr(ur), None, B, k1 - 1, V, T, 0.9, 0, L.ptr(n), L.ptr(y),
        None, None, L.ptr(ws), ws.numel(), L.stream_ptr(tgt.device))
    assert rc == 0
    return n, y


def test_greedy_workspace_needs_no_initialisation():
    """The greedy calls keep no counters: a workspace full of random bytes,
    shared by greedy calls of several shapes with sampling calls (which write
    stats, lists and their own counters there) in between, gives the results
    of a fresh one."""
    from specdec import _lib as L
    g = torch.Generator(device=DEV).manual_seed(11)
    shapes = [(64, 4, 151936), (7, 2, 32003), (3, 64, 4096), (33, 8, 4096), (64, 4, 151936)]
    nbytes = max(L.lib().sd_sampling_workspace_bytes(B, B * (2 * k + 1), V, 2) for B, k, V in shapes)
    ws = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=torch.Generator(
        device=DEV).manual_seed(5), device=DEV)
    for i, (B, k, V) in enumerate(shapes):
        tgt, xs, ua, ur = _greedy_inputs(B, k, V, g, p_match=0.97 if k > 32 else 0.7)
        for _ in range(2):                             # the same shape twice in a row
            n, y = _verify_ws(tgt, None, xs, ua, ur, 0.0, ws)
            n_r, y_r = _greedy_ref(tgt, xs, ua)
            assert torch.equal(n, n_r) and torch.equal(y, y_r), (i, B, k, V)
        drf = (tgt[:, :k].float() + torch.randn(B, k, V, generator=g, device=DEV)).to(tgt.dtype)
        _verify_ws(tgt, drf, xs, ua, ur, 0.7, ws)     # a sampling call in between
    torch.cuda.synchronize()


def test_greedy_long_rows():
    """k = 64 (65 vectors per row): accepted prefixes across the 32-lane groups
    of the row decision."""
    g = torch.Generator(device=DEV).manual_seed(13)
    B, k, V = 6, 64, 2048
    tgt, xs, ua, ur = _greedy_inputs(B, k, V, g, p_match=1.0)
    ua[:, :] = 0.5
    xs[1, 40] = (xs[1, 40] + 1) % V                    # rejected at 40
    xs[2, 31] = (xs[2, 31] + 1) % V                    # at 31, the first group's last lane
    xs[3, 32] = (xs[3, 32] + 1) % V                    # at 32, the second group's first lane
    ua[4, 0] = 1.0                                     # u = 1 rejects even a match
    alive = torch.ones(B, dtype=torch.bool, device=DEV)
    alive[5] = False
    n, y = S.verify_sample(tgt, None, xs, ua, ur, 0.0, alive=alive)
    n_r, y_r = _greedy_ref(tgt, xs, ua, alive)
    assert n.tolist() == [64, 40, 31, 32, 0, 0] and torch.equal(n, n_r)
    assert torch.equal(y, y_r)


def test_greedy_graph_replay():
    """A captured greedy call (two kernels, no memset) replays on new inputs."""
    B, k, V = 16, 4, 151936
    g = torch.Generator(device=DEV).manual_seed(12)
    bufs = _greedy_inputs(B, k, V, g)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        S.verify_sample(bufs[0], None, *bufs[1:], 0.0)  # the stream's workspace exists before capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        n, y = S.verify_sample(bufs[0], None, *bufs[1:], 0.0)
    for rep in range(4):
        new = _greedy_inputs(B, k, V, g)
        for dst, src in zip(bufs, new):
            dst.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        n_r, y_r = _greedy_ref(bufs[0], bufs[1], bufs[2])
        assert torch.equal(n, n_r) and torch.equal(y, y_r), rep
    del graph


# ---------------------------------------------------------------------------
# draft step and the fp32-probability utilities
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("T,tp,tk,V", [(0.7, 0.9, 0, 151936), (1.0, 1.0, 0, 32), (0.0, 1.0, 0, 4096),
                                       (1.2, 0.95, 50, 32000)])
def test_draft_sample_parity(T, tp, tk, V):
    g = torch.Generator().manual_seed(5)
    x = W.zipf_logits(16, V, g).to(DEV, torch.bfloat16 if V > 32 else torch.float32)
    u = torch.rand(16, generator=g).to(DEV)
    xk, qk = S.draft_sample(x, u, T, tp, tk)
    xo, qo, d = O.draft_sample(_np(x), _np(u), T, tp, tk, return_details=True)
    ok = (d["cdf_margin"] > EPS) & (d["topp_margin"] > EPS)
    assert ok.mean() > 0.8
    np.testing.assert_array_equal(xk.cpu().numpy()[ok], xo[ok])
    np.testing.assert_allclose(qk.cpu().numpy()[ok], qo[ok], rtol=2e-6)


def test_prob_utilities():
    z = np.load(GOLDEN / "residual.npz")
    p = torch.from_numpy(z["p"]).to(DEV)
    q = torch.from_numpy(z["q"]).to(DEV)
    np.testing.assert_allclose(_np(S.residual_probs(p, q)), z["r"], rtol=1e-6, atol=1e-9)
    ids = torch.from_numpy(z["ids"]).to(DEV)
    np.testing.assert_array_equal(_np(S.gather_prob(p, ids)), z["gathered"])
    u = torch.rand(p.shape[0], generator=torch.Generator().manual_seed(0)).to(DEV)
    np.testing.assert_array_equal(S.sample_from_probs(p, u=u).cpu().numpy(),
                                  O.sample_inverse_cdf(z["p"], _np(u)))


def test_cpu_tensors_are_rejected():
    with pytest.raises(RuntimeError):
        S.to_probs(torch.randn(2, 8), 1.0)


# ---------------------------------------------------------------------------
# gate G1 part A on the kernels: the rule reproduces p; broken rules do not
# ---------------------------------------------------------------------------
def _tv(a, b):
    return 0.5 * float(np.abs(a - b).sum())


def test_rejection_rule_is_lossless():
    """G1 part A on the kernels (reference tests/test_rejection_sampling.py:82-126):
    the first emitted token follows p (TV < 0.01 over 200k trials), and the
    three negative controls are detected (TV > 0.02): skipping the accept
    test, resampling from p instead of the residual, and drafting with a
    different top-p than the one the accept test uses."""
    V, N = 16, 200_000
    g = torch.Generator().manual_seed(0)
    lp = torch.randn(1, V, generator=g) * 1.5
    lq = torch.randn(1, V, generator=g) * 1.5
    lq_close = lp + torch.randn(1, V, generator=g) * 0.8     # a plausible draft model
    for (tp, lq_use) in ((1.0, lq), (0.9, lq_close)):
        p = O.to_probs(lp.numpy(), 1.0, tp)[0]
        tgt = torch.cat([lp, lp]).unsqueeze(0).expand(N, 2, V).contiguous().to(DEV)
        drf = lq_use.unsqueeze(0).expand(N, 1, V).contiguous().to(DEV)
        gd = torch.Generator(device=DEV).manual_seed(7)
        x, _ = S.draft_sample(drf[:, 0], torch.rand(N, generator=gd, device=DEV), 1.0, tp)
        ua = torch.rand(N, 1, generator=gd, device=DEV)
        ur = torch.rand(N, generator=gd, device=DEV)
        n, y = S.verify_sample(tgt, drf, x.view(N, 1), ua, ur, 1.0, tp)
        first = torch.where(n == 1, x, y).cpu().numpy()
        emp = np.bincount(first, minlength=V) / N
        assert _tv(emp, p) < 0.01, f"top_p={tp}: TV={_tv(emp, p):.4f}"
        # control 1: skipping the accept test emits x ~ q
        bad = np.bincount(x.cpu().numpy(), minlength=V) / N
        assert _tv(bad, p) > 0.02, f"top_p={tp}: skip-accept control TV={_tv(bad, p):.4f}"
        # control 2: on a rejection, resample from p instead of the residual
        yp, _ = S.draft_sample(tgt[:, 0], ur, 1.0, tp)
        bad2 = np.bincount(torch.where(n == 1, x, yp).cpu().numpy(), minlength=V) / N
        assert _tv(bad2, p) > 0.02, f"top_p={tp}: resample-from-p control TV={_tv(bad2, p):.4f}"
    # control 3: draft drawn with top-p 0.5, accept test and residual with 0.9
    p = O.to_probs(lp.numpy(), 1.0, 0.9)[0]
    q_right = O.to_probs(lq_close.numpy(), 1.0, 0.9)[0]
    assert np.minimum(p, q_right).sum() > 0.2, "control instance must be non-degenerate"
    tgt = torch.cat([lp, lp]).unsqueeze(0).expand(N, 2, V).contiguous().to(DEV)
    drf = lq_close.unsqueeze(0).expand(N, 1, V).contiguous().to(DEV)
    gd = torch.Generator(device=DEV).manual_seed(11)
    xm, _ = S.draft_sample(drf[:, 0], torch.rand(N, generator=gd, device=DEV), 1.0, 0.5)
    ua = torch.rand(N, 1, generator=gd, device=DEV)
    ur = torch.rand(N, generator=gd, device=DEV)
    n, y = S.verify_sample(tgt, drf, xm.view(N, 1), ua, ur, 1.0, 0.9)
    emp = np.bincount(torch.where(n == 1, xm, y).cpu().numpy(), minlength=V) / N
    assert _tv(emp, p) > 0.02, f"mismatched top-p control TV={_tv(emp, p):.4f}"


def _vec_stats(B, nvec, V, dev):
    """The per-vector stats records the last sampling call on this stream
    left at the start of its workspace (48-byte records after the 256-byte
    status word): fb_why is the 11th int32."""
    from specdec import _lib as L
    ws = L.workspaces.get(L.lib().sd_sampling_workspace_bytes(B, nvec, V, 2), dev)
    return ws[256:256 + nvec * 48].cpu().numpy().view(np.int32).reshape(nvec, 12)


def test_histogram_fallback_runs_and_is_exact():
    """Flat distributions (T = 2, top-p 0.9 on N(0, 1) logits, V = 4096) put
    more elements inside the list window than the list holds, so every vector
    must take the exact histogram path (VecStats.fb_why != 0); the results
    stay bit-exact against the oracle.  Inputs come from the CPU generator
    (an instance checked to have no row inside the exemption margins)."""
    B, k, V, T, tp = 8, 2, 4096, 2.0, 0.9
    g = torch.Generator().manual_seed(21)
    tgt = (torch.randn(B, k + 1, V, generator=g)).bfloat16()
    drf = (tgt[:, :k].float() + 1.0 * torch.randn(B, k, V, generator=g)).bfloat16()
    q = O.to_probs(drf.float().reshape(-1, V).numpy(), T, tp)
    u = np.random.default_rng(3).random(B * k, dtype=np.float32)
    xs = O.sample_inverse_cdf(q, u).reshape(B, k)
    ua = torch.from_numpy(np.random.default_rng(5).random((B, k), dtype=np.float32))
    ur = torch.from_numpy(np.random.default_rng(6).random(B, dtype=np.float32))
    _check_verify(tgt.to(DEV), drf.to(DEV), torch.from_numpy(xs).to(DEV), ua.to(DEV), ur.to(DEV),
                  T, tp, 0, max_exempt=0.25, tag="flat")
    st = _vec_stats(B, B * (2 * k + 1), V, torch.device(DEV, torch.cuda.current_device()))
    assert (st[:, 10] != 0).all(), f"fallback reasons {st[:, 10].tolist()}"
