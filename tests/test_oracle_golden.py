"""Pin the CPU oracle to the real reference, through the committed fixtures.

The fixtures were produced by tests/golden/make_golden.py, which imported the
reference's specdec/sampling.py (to_probs / residual_probs / gather_prob,
lines 34-95) and restated engine.py:282-303 with uniforms as tensors.

Tolerances: the reference computes exp with torch's vectorised CPU exp and sums
with fp32 lane accumulators, while the oracle uses float64 exp/sums rounded to
float32.  Probabilities therefore agree to ~1e-6 relative, and decisions agree
exactly except where a row sits within that noise of a decision boundary.
"""
import numpy as np
import pytest

from oracle import sampling_oracle as O
from tests.golden import GOLDEN

REL = 1e-6      # oracle vs reference fp32 probabilities (measured max 2.4e-7)


def _load(name):
    return np.load(GOLDEN / name, allow_pickle=False)


def _cases(z):
    return [str(n) for n in z["names"]]


@pytest.mark.parametrize("case", _cases(_load("to_probs.npz")))
def test_to_probs_matches_reference_stable(case):
    z = _load("to_probs.npz")
    x = z[case + "__x"]
    T, tp, tk = z[case + "__params"]
    want = z[case + "__stable"]
    infos = []
    got = O.to_probs(x, float(T), float(tp), int(tk), infos=infos)
    for r in range(x.shape[0]):
        if infos[r].topp_margin < 1e-5:
            continue     # nucleus edge inside the reference's own rounding noise
        np.testing.assert_array_equal(got[r] > 0, want[r] > 0, err_msg=f"{case} row {r} support")
        np.testing.assert_allclose(got[r], want[r], rtol=REL, atol=1e-12, err_msg=f"{case} row {r}")


def test_tie_policy_is_the_only_difference_from_unstable_sort():
    """The unmodified reference (unstable sort) may pick different members of the
    boundary tie class; the kept COUNT and the probabilities of every kept
    token outside that class are the same."""
    z = _load("to_probs.npz")
    saw_tie = False
    for case in _cases(z):
        st, pl = z[case + "__stable"], z[case + "__plain"]
        np.testing.assert_array_equal((st > 0).sum(-1), (pl > 0).sum(-1))
        np.testing.assert_allclose(np.sort(st, -1), np.sort(pl, -1), rtol=1e-6, atol=0)
        saw_tie |= bool(z[case + "__tiediff"].any())
    assert saw_tie, "fixtures should contain at least one boundary tie class"


def test_residual_and_gather():
    z = _load("residual.npz")
    r = O.residual_probs(z["p"], z["q"])
    np.testing.assert_allclose(r, z["r"], rtol=REL, atol=1e-9)
    np.testing.assert_array_equal(O.gather_prob(z["p"], z["ids"]), z["gathered"])


@pytest.mark.parametrize("case", _cases(_load("verify.npz")))
def test_verify_matches_reference(case):
    z = _load("verify.npz")
    g = {k: z[f"{case}__{k}"] for k in ("tgt", "drf", "xs", "u_acc", "u_res", "n_acc", "y",
                                        "params", "P", "Q")}
    T, tp, tk = g["params"]
    n_acc, y, d = O.verify(g["tgt"], g["drf"], g["xs"], g["u_acc"], g["u_res"], float(T),
                           float(tp), int(tk), return_details=True)
    ok = (d["acc_margin"] > 1e-5) & (d["cdf_margin"] > 1e-5) & (d["topp_margin"] > 1e-5)
    assert ok.mean() >= 0.75, f"too many boundary rows: {ok.sum()}/{ok.size}"
    np.testing.assert_array_equal(n_acc[ok], g["n_acc"][ok])
    np.testing.assert_array_equal(y[ok], g["y"][ok])
    sup = (d["P"] > 0) == (g["P"] > 0)
    assert sup.mean() > 0.999
    np.testing.assert_allclose(np.where(sup, d["P"], 0), np.where(sup, g["P"], 0), rtol=REL, atol=1e-9)


def test_cfg1_exact_and_nontrivial():
    """Config 1 (B=8, k=4, V=32, T=1, top-p 1): every row decided identically,
    and the instance exercises both rejections and full acceptance paths."""
    z = _load("verify.npz")
    c = "cfg1_v32"
    n_acc, y = O.verify(z[c + "__tgt"], z[c + "__drf"], z[c + "__xs"], z[c + "__u_acc"],
                        z[c + "__u_res"], 1.0, 1.0, 0)
    np.testing.assert_array_equal(n_acc, z[c + "__n_acc"])
    np.testing.assert_array_equal(y, z[c + "__y"])
    assert len(set(n_acc.tolist())) >= 2


def test_inverse_cdf_definition():
    p = np.array([[0.1, 0.0, 0.6, 0.3]], dtype=np.float32)
    assert O.sample_inverse_cdf(p, np.array([0.0]))[0] == 0
    assert O.sample_inverse_cdf(p, np.array([0.1]))[0] == 2      # cumsum 0.1 is not > 0.1
    assert O.sample_inverse_cdf(p, np.array([0.69]))[0] == 2
    assert O.sample_inverse_cdf(p, np.array([0.71]))[0] == 3
    assert O.sample_inverse_cdf(p, np.array([1.0]))[0] == 3      # u*sum beyond the end: last nonzero


def test_bf16_helpers_round_trip():
    x = np.array([1.0, -2.5, 3.14159, 1e-3, -0.0], dtype=np.float32)
    b = O.f32_to_bf16_bits(x)
    y = O.bf16_bits_to_f32(b)
    assert np.all(np.abs(y - x) <= np.abs(x) * 2 ** -8)
    np.testing.assert_array_equal(O.f32_to_bf16_bits(y), b)


def test_verify_matches_reference_at_full_vocab():
    """Config 2 at V = 151936 (8 rows): the oracle against the reference's own
    to_probs / accept loop outputs (tests/golden/verify_cfg2.npz)."""
    from tests.golden import cfg2_inputs as CI
    z = _load("verify_cfg2.npz")
    tgt, drf = CI.cfg2_rows()
    assert CI.checksum(tgt) == float(z["tgt_sum"]) and CI.checksum(drf) == float(z["drf_sum"]), \
        "config-2 input generator changed: regenerate the fixture"
    tgt, drf = tgt.numpy(), drf.numpy()
    for name, T, tp in (("t07_tp09", 0.7, 0.9), ("greedy", 0.0, 1.0)):
        xs, ua, ur = z[name + "__xs"], z[name + "__u_acc"], z[name + "__u_res"]
        n, y, d = O.verify(tgt, drf, xs, ua, ur, T, tp, 0, return_details=True)
        ok = (d["acc_margin"] > 1e-6) & (d["cdf_margin"] > 1e-6) & (d["topp_margin"] > 1e-6)
        assert ok.mean() >= 0.75, name
        np.testing.assert_array_equal(n[ok], z[name + "__n_acc"][ok], err_msg=name)
        np.testing.assert_array_equal(y[ok], z[name + "__y"][ok], err_msg=name)
        np.testing.assert_allclose(d["px"], z[name + "__px"], rtol=REL, atol=1e-30, err_msg=name)
        np.testing.assert_allclose(d["qx"], z[name + "__qx"], rtol=REL, atol=1e-30, err_msg=name)
