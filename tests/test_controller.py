"""Controller maths and adaptation (CPU only).

Replays the reference controllers' recorded behaviour (fixtures generated from
reference specdec/controller.py by tests/golden/make_golden.py) and re-checks
the properties the reference's tests/test_controller.py asserts.
"""
import json
import random
import statistics

import pytest
import torch

from specdec.controller import (ConfidenceEarlyExit, EWMAAnalytic, FixedK, UCBBandit, best_k,
                                expected_speedup, make_controller)
from tests.golden import GOLDEN

G = json.loads((GOLDEN / "controller.json").read_text())


def test_best_k_grid_matches_reference():
    for a, c, ef, k, speeds in G["best_k_grid"]:
        assert best_k(a, c, 8, ef) == k, (a, c, ef)
        for kk, v in enumerate(speeds, start=1):
            assert expected_speedup(kk, a, c, ef) == pytest.approx(v, rel=1e-12)


def test_ewma_trajectory_matches_reference():
    ew = EWMAAnalytic(k_max=8, beta=0.95, warmup=3)
    for k, n_acc, dt, tdf, ttf, alpha, c in G["ewma_trace"]:
        assert ew.propose_k() == k
        ew.update(k, n_acc, dt, t_draft_fwd=tdf, t_target_fwd=ttf)
        assert ew.alpha == pytest.approx(alpha, rel=1e-12)
        assert ew.c == pytest.approx(c, rel=1e-12)


def test_ucb_trajectory_matches_reference():
    u = UCBBandit(k_max=5)
    for k, n_acc, dt, mu in G["ucb_trace"]:
        assert u.propose_k() == k
        u.update(k, n_acc, dt)
        for kk, v in mu.items():
            assert u.mu[int(kk)] == pytest.approx(v, rel=1e-12)


def test_early_exit_and_names_match_reference():
    ee = ConfidenceEarlyExit(FixedK(6), tau=0.4, min_k=2)
    for i, conf, want in G["early_exit"]:
        assert ee.should_stop_drafting(i, torch.tensor(conf)) == want
    for spec, name in G["make_controller_names"].items():
        assert make_controller(spec).state()["name"] == name


def test_speedup_shape():
    assert all(expected_speedup(4, a, 0.15) < expected_speedup(4, a + 0.1, 0.15)
               for a in (0.4, 0.5, 0.6, 0.7, 0.8))
    assert all(expected_speedup(4, 0.8, c) > expected_speedup(4, 0.8, c + 0.05)
               for c in (0.05, 0.1, 0.15, 0.2))
    assert all(best_k(a, 0.15) <= best_k(a + 0.05, 0.15) for a in (0.3, 0.5, 0.7, 0.9))
    assert best_k(0.05, 0.3) == 1 and best_k(0.98, 0.05, 8) == 8
    for a in (0.6, 0.78, 0.9):
        for c in (0.15, 0.5, 1.0, 1.6):
            assert best_k(a, c, 8, 1) >= best_k(a, c, 8, 0)


def test_alpha_counts_positions_reached():
    ctl = EWMAAnalytic(beta=0.5, warmup=0)
    for _ in range(40):
        ctl.update(4, [1], 1.0, t_draft_fwd=0.1, t_target_fwd=1.0)
    assert abs(ctl.alpha - 0.5) < 0.02


@pytest.mark.parametrize("alpha,c", [(0.45, 0.12), (0.7, 0.12), (0.9, 0.08)])
def test_converges_to_oracle_k(alpha, c):
    oracle = best_k(alpha, c)
    ctl = EWMAAnalytic(warmup=20)
    rng = random.Random(0)
    ks, ahat = [], []
    for r in range(3000):
        k = ctl.propose_k()
        a = 0
        while a < k and rng.random() < alpha:
            a += 1
        ctl.update(k, [a], 1.0, t_draft_fwd=c, t_target_fwd=1.0)
        if r > 1000:
            ks.append(k)
            ahat.append(ctl.alpha)
    assert statistics.mode(ks) == oracle
    assert abs(statistics.mean(ahat) - alpha) < 0.03


def _two_phase(ctl, rounds=4000, c=0.12):
    rng = random.Random(0)
    tok = cost = 0.0
    for r in range(rounds):
        alpha = 0.9 if (r // 250) % 2 == 0 else 0.35
        k = min(ctl.propose_k(), 8)
        a = 0
        while a < k and rng.random() < alpha:
            a += 1
        cst = (k + 1) * c + 1.0
        tok += a + 1
        cost += cst
        ctl.update(k, [a], cst, t_draft_fwd=c, t_target_fwd=1.0)
    return tok / cost


def test_adaptive_beats_best_fixed_on_shifting_workload():
    fixed_best = max(_two_phase(FixedK(k)) for k in range(1, 9))
    assert _two_phase(EWMAAnalytic(beta=0.9)) >= fixed_best


def test_ucb_explores_then_converges():
    b = UCBBandit(k_max=4)
    seen = []
    for _ in range(4):
        k = b.propose_k()
        seen.append(k)
        b.update(k, [1], 1.0)
    assert sorted(seen) == [1, 2, 3, 4]
    b = UCBBandit(k_max=4)
    for _ in range(600):
        k = b.propose_k()
        b.update(k, [1], 1.0 + abs(k - 3))
    assert max(b.mu, key=b.mu.get) == 3
