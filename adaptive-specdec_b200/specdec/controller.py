"""Draft-length controllers (host side; a few scalar operations per round).

Same interface and maths as the reference's specdec/controller.py:

* expected tokens per round  E(k) = (1 - a^(k+1)) / (1 - a)          (:57-60)
* cost per round             (k + extra_fwd) * c + 1                  (:61)
* best_k = argmax over k in [1, k_max] of E(k) / cost(k)              (:64-67)
* EWMAAnalytic: alpha = decayed accepted / decayed positions reached, the
  decay applied per position evaluated (beta ** reached), c <- 0.9 c + 0.1 c_obs
  (:101-159)
* ConfidenceEarlyExit: stop drafting when the mean running product of the
  drafted tokens' draft probabilities falls below tau (:162-195)
* UCBBandit: UCB1 over k with reward = emitted tokens per second (:198-231)
* make_controller(spec) for 'fixedN' | 'ewma' | 'ucb' with optional '+exit'
  (:234-251)

The controllers never touch the GPU except ConfidenceEarlyExit, which reads
one scalar (the batch-mean confidence) per drafted token.
"""
import math

__all__ = ["Controller", "FixedK", "EWMAAnalytic", "ConfidenceEarlyExit", "UCBBandit",
           "expected_speedup", "best_k", "make_controller"]


def expected_speedup(k, alpha, c, extra_fwd=1):
    """Expected committed tokens per round over the round's cost (target units)."""
    k = max(1, int(k))
    if alpha >= 1.0 - 1e-9:
        per_round = float(k + 1)
    else:
        per_round = (1.0 - alpha ** (k + 1)) / (1.0 - alpha)
    return per_round / ((k + extra_fwd) * c + 1.0)


def best_k(alpha, c, k_max=8, extra_fwd=1):
    """The k in [1, k_max] with the highest expected speedup (first on ties)."""
    best, best_v = 1, -math.inf
    for k in range(1, int(k_max) + 1):
        v = expected_speedup(k, alpha, c, extra_fwd)
        if v > best_v:
            best, best_v = k, v
    return best


class Controller:
    """Shared by the engine and the vLLM proposer."""

    name = "base"

    def propose_k(self) -> int:
        raise NotImplementedError

    def should_stop_drafting(self, i, conf) -> bool:
        """i = tokens drafted so far this round; conf = [B] running product of q(x)."""
        return False

    def update(self, k, n_accepted, dt, t_draft_fwd=None, t_target_fwd=None):
        """n_accepted: per-row accepted counts of the round that just finished."""

    def state(self):
        return {"name": self.name}


class FixedK(Controller):
    def __init__(self, k):
        self.k = int(k)
        self.name = f"fixed{self.k}"

    def propose_k(self):
        return self.k


class EWMAAnalytic(Controller):
    """Online alpha and cost ratio c; k = best_k(alpha, c)."""

    name = "ewma-analytic"

    def __init__(self, k_max=8, beta=0.99, k_init=4, c_init=0.15, warmup=3, extra_fwd=1):
        self.k_max = int(k_max)
        self.beta = float(beta)
        self.k_init = int(k_init)
        self.c = float(c_init)
        self.warmup = int(warmup)
        self.extra_fwd = int(extra_fwd)
        self._acc_w = 0.0        # decayed accepted tokens
        self._reach_w = 0.0      # decayed positions evaluated
        self._rounds = 0
        self._last_k = self.k_init

    @property
    def alpha(self):
        if self._reach_w <= 0:
            return 0.7
        return min(0.999, max(0.0, self._acc_w / self._reach_w))

    def propose_k(self):
        if self._rounds < self.warmup:
            self._last_k = self.k_init
        else:
            self._last_k = best_k(self.alpha, self.c, self.k_max, self.extra_fwd)
        return self._last_k

    def update(self, k, n_accepted, dt, t_draft_fwd=None, t_target_fwd=None):
        accepted = float(sum(n_accepted))
        # position i was evaluated iff every earlier one was accepted: a + 1 of
        # them per row, capped at k
        reached = float(sum(min(a + 1, k) for a in n_accepted))
        decay = self.beta ** reached
        self._acc_w = decay * self._acc_w + accepted
        self._reach_w = decay * self._reach_w + reached
        if t_draft_fwd and t_target_fwd and t_target_fwd > 0:
            self.c = 0.9 * self.c + 0.1 * (t_draft_fwd / t_target_fwd)
        self._rounds += 1

    def state(self):
        return {"name": self.name, "alpha": self.alpha, "c": self.c, "k": self._last_k,
                "rounds": self._rounds, "extra_fwd": self.extra_fwd}


class ConfidenceEarlyExit(Controller):
    """Any controller plus a mid-round stop on low draft confidence."""

    def __init__(self, base, tau=0.3, min_k=1):
        self.base = base
        self.tau = float(tau)
        self.min_k = int(min_k)
        self.name = f"{base.name}+exit{self.tau}"

    def propose_k(self):
        return self.base.propose_k()

    def should_stop_drafting(self, i, conf):
        if i < self.min_k:
            return False
        return float(conf.mean()) < self.tau

    def update(self, k, n_accepted, dt, t_draft_fwd=None, t_target_fwd=None):
        self.base.update(k, n_accepted, dt, t_draft_fwd, t_target_fwd)

    def state(self):
        st = dict(self.base.state())
        st.update({"name": self.name, "tau": self.tau})
        return st


class UCBBandit(Controller):
    """UCB1 over k in [1, k_max]; reward = emitted tokens / dt."""

    name = "ucb"

    def __init__(self, k_max=8, cexp=0.5):
        self.ks = list(range(1, int(k_max) + 1))
        self.n = {k: 0 for k in self.ks}
        self.mu = {k: 0.0 for k in self.ks}
        self.t = 0
        self.cexp = float(cexp)
        self._last_k = self.ks[0]

    def propose_k(self):
        self.t += 1
        for k in self.ks:
            if self.n[k] == 0:
                self._last_k = k
                return k
        logt = math.log(self.t)
        best, best_v = self.ks[0], -math.inf
        for k in self.ks:
            v = self.mu[k] + self.cexp * math.sqrt(logt / self.n[k])
            if v > best_v:
                best, best_v = k, v
        self._last_k = best
        return best

    def update(self, k, n_accepted, dt, t_draft_fwd=None, t_target_fwd=None):
        reward = sum(a + 1 for a in n_accepted) / dt if dt > 0 else 0.0
        self.n[k] += 1
        self.mu[k] += (reward - self.mu[k]) / self.n[k]

    def state(self):
        return {"name": self.name, "k": self._last_k,
                "mu": {str(k): round(v, 2) for k, v in self.mu.items()}}


def make_controller(spec, k_max=8, tau=0.3, extra_fwd=1):
    """'ar' is not a controller; 'fixedN' | 'ewma' | 'ucb', optionally '+exit'."""
    s = spec.strip().lower()
    with_exit = s.endswith("+exit")
    if with_exit:
        s = s[:-len("+exit")]
    if s.startswith("fixed"):
        base = FixedK(int(s[len("fixed"):]))
    elif s == "ewma":
        base = EWMAAnalytic(k_max=k_max, extra_fwd=extra_fwd)
    elif s == "ucb":
        base = UCBBandit(k_max=k_max)
    else:
        raise ValueError(f"unknown controller spec: {spec!r}")
    return ConfidenceEarlyExit(base, tau=tau) if with_exit else base
