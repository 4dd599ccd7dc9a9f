"""CPU restatement of the vocabulary-sharded verify round.  TEST INFRASTRUCTURE ONLY.

Only ``tests/`` may use this module, as the checker: it is a phase backend for
``specdec.sharded.run_round`` / ``verify_sharded`` that computes, with numpy on
the host, exactly what the CUDA phase kernels (``sd_shard_phase``) compute, on
the same byte-level messages.  With it the round's host orchestration and its
message arithmetic run over gloo on CPU, and the sharded result can be
compared with the unsharded oracle (``sampling_oracle.verify``), which
restates ``specdec/engine.py:282-303`` and ``specdec/sampling.py:34-95``.

Arithmetic per element (as the unsharded oracle): d = fl32(x / T),
t = fl32(d - m) with m the global maximum, e = fl32(exp(t)) (exp in float64),
p = fl32(e * fl32(1 / S)); depth bin = int(fl32(-t * fl32(8 log2 e))), 128 bins
(16 base-2 units), bin 128 below the window.  Top-p: bins whose cumulative
approximate mass stays below top_p - 1e-5 are kept whole, bins starting above
top_p + 1e-5 are dropped, the bins between (plus one on each side) are sorted
across shards by (p desc, index asc) and the reference's rule
fl32(fl32(cum) - p) < top_p is applied to them.
"""
import numpy as np
import torch

F32, F64 = np.float32, np.float64
NB = 128
CAP = 128
DELTA = 1e-5
STATUS_FALLBACK = 2
BIN_SCALE = F32(F32(8.0) * F32(1.4426950408889634))
MSG3 = np.dtype([("pre", F64), ("n", np.int32), ("flags", np.int32), ("e", np.uint64, CAP)])
MSG1 = np.dtype([("m", F32), ("dx", F32)])


def _fkey(p):
    b = np.asarray(p, dtype=F32).view(np.uint32).copy()
    b[b == 0x80000000] = 0
    neg = (b & 0x80000000) != 0
    return np.where(neg, ~b, b | np.uint32(0x80000000)).astype(np.uint32)


def _pkey(p, j):
    return (_fkey(p).astype(np.uint64) << np.uint64(32)) | (
        np.uint64(0xFFFFFFFF) - np.asarray(j, dtype=np.uint64))


def _pkey_val(k):
    u = (np.asarray(k, dtype=np.uint64) >> np.uint64(32)).astype(np.uint32)
    b = np.where((u & 0x80000000) != 0, u & np.uint32(0x7FFFFFFF), ~u).astype(np.uint32)
    return b.view(F32)


def _exp32(t):
    return np.exp(np.asarray(t, dtype=F32).astype(F64)).astype(F32)


def _bin(t):
    y = (-np.asarray(t, dtype=F32)).astype(F32) * BIN_SCALE
    y = y.astype(F32)
    return np.where(y < F32(NB), np.floor(np.minimum(y, F32(NB))), NB).astype(np.int64)


class NumpyShardBackend:
    """Phase backend with the interface of specdec.sharded.CudaShardBackend."""

    def bind(self, tgt, drf, xs, u_acc, u_res, alive, v_start, rank, V, temperature, top_p,
             top_k):
        to = lambda t: None if t is None else t.detach().cpu().float().numpy()
        self.tgt, self.drf = to(tgt), to(drf)
        self.xs = xs.detach().cpu().numpy().astype(np.int64)
        self.u_acc, self.u_res = to(u_acc), to(u_res)
        self.alive = None if alive is None else alive.detach().cpu().numpy().astype(bool)
        self.v_start, self.rank, self.V = list(v_start), rank, V
        self.nranks = len(v_start) - 1
        self.T, self.top_p = F32(temperature), F32(top_p)
        self.greedy = not temperature > 0
        self.truncate = 0.0 < top_p < 1.0
        self.B, k1, self.Vr = self.tgt.shape
        self.k = k1 - 1
        self.per = 2 * self.k + 1
        self.nvec = self.B * self.per
        self.v0 = v_start[rank]
        self._status = 0

    # vector v -> scaled logits of this shard, and its probe token
    def _vec(self, v):
        b, l = divmod(v, self.per)
        if l <= self.k:
            x, pos = self.tgt[b, l], l
        else:
            x, pos = self.drf[b, l - self.k - 1], l - self.k - 1
        probe = int(self.xs[b, pos]) if pos < self.k else -1
        return (x.astype(F32) / self.T).astype(F32), probe

    def _owner(self, x):
        r = 0
        while r + 1 < self.nranks and x >= self.v_start[r + 1]:
            r += 1
        return r

    def send_bytes(self, phase):
        if self.greedy:
            return self.B * (self.k + 1) * 8 if phase == 1 else 0
        return {1: self.nvec * 8, 2: self.nvec * (1 + NB) * 8, 3: self.nvec * MSG3.itemsize,
                4: self.B * 16, 5: self.B * 8}.get(phase, 0)

    def phase(self, phase, recv):
        rb = None if recv is None else recv.detach().cpu().numpy().view(np.uint8)
        out = getattr(self, f"_g{phase}" if self.greedy else f"_p{phase}")(rb)
        return None if out is None else torch.from_numpy(np.ascontiguousarray(out).view(np.uint8)
                                                         .reshape(-1).copy())

    def status(self):
        return self._status

    def outputs(self):
        return torch.from_numpy(self.n_acc.copy()), torch.from_numpy(self.y.copy())

    # ---- greedy ---------------------------------------------------------------
    def _g1(self, _):
        out = np.zeros(self.B * (self.k + 1), dtype=np.int64)
        for b in range(self.B):
            for i in range(self.k + 1):
                x = self.tgt[b, i].astype(F32)
                if x.size == 0:
                    continue
                # every NaN (either sign bit) counts as the maximum
                fk = np.where(np.isnan(x), np.uint32(0xFFFFFFFF), _fkey(x))
                keys = (fk.astype(np.uint64) << np.uint64(31)) | (
                    np.uint64(0x7FFFFFFF) - (self.v0 + np.arange(x.size)).astype(np.uint64))
                out[b * (self.k + 1) + i] = np.int64(keys.max())
        return out

    def _g6(self, rb):
        keys = rb.view(np.int64)
        k1 = self.k + 1
        amax = lambda b, i: 0x7FFFFFFF - int(keys[b * k1 + i] & 0x7FFFFFFF)
        self.n_acc = np.zeros(self.B, dtype=np.int64)
        self.y = np.zeros(self.B, dtype=np.int64)
        for b in range(self.B):
            alive = True if self.alive is None else bool(self.alive[b])
            n = 0
            for i in range(self.k):
                ok = alive and n == i and int(self.xs[b, i]) == amax(b, i)
                n += int(ok)
                alive = alive and ok
            self.n_acc[b], self.y[b] = n, amax(b, n)
        return None

    # ---- sampling -------------------------------------------------------------
    def _p1(self, _):
        out = np.zeros(self.nvec, dtype=MSG1)
        for v in range(self.nvec):
            d, probe = self._vec(v)
            out["m"][v] = d.max() if d.size else -np.inf
            out["dx"][v] = d[probe - self.v0] if self.v0 <= probe < self.v0 + self.Vr else np.nan
        return out

    def _p2(self, rb):
        msgs = rb.view(MSG1).reshape(self.nranks, self.nvec)
        self.m = msgs["m"].max(axis=0).astype(F32)
        self.dx = np.full(self.nvec, np.nan, dtype=F32)
        out = np.zeros((self.nvec, 1 + NB), dtype=F64)
        for v in range(self.nvec):
            d, probe = self._vec(v)
            if 0 <= probe < self.V:
                self.dx[v] = msgs["dx"][self._owner(probe), v]
            t = (d - self.m[v]).astype(F32)
            e = _exp32(t)
            out[v, 0] = e.astype(F64).sum()
            if self.truncate:
                bins = _bin(t)
                sel = bins < NB
                out[v, 1:] = np.bincount(bins[sel], weights=e[sel].astype(F64), minlength=NB)
        return out

    def _p3(self, rb):
        tot = rb.view(F64).reshape(self.nvec, 1 + NB)
        self.S = tot[:, 0].copy()
        self.inv_s = (1.0 / self.S).astype(F32)
        self.lo = np.full(self.nvec, NB + 1, dtype=np.int64)
        self.hi = np.full(self.nvec, NB, dtype=np.int64)
        self.flags = np.zeros(self.nvec, dtype=np.int32)
        out = np.zeros(self.nvec, dtype=MSG3)
        tp = F64(self.top_p)
        for v in range(self.nvec):
            if self.truncate:
                A, lo_b, hi_b = 0.0, -1, -1
                for i in range(NB):
                    mb = tot[v, 1 + i] * F64(self.inv_s[v])
                    if lo_b < 0 and A + mb > tp - DELTA:
                        lo_b = i
                    if A < tp + DELTA:
                        hi_b = i
                    A += mb
                if A < tp + DELTA or lo_b < 0 or hi_b >= NB - 1:
                    self.flags[v] = 1
                    self.lo[v], self.hi[v] = 0, -1
                else:
                    self.lo[v], self.hi[v] = max(lo_b - 1, 0), hi_b + 1
            d, _ = self._vec(v)
            t = (d - self.m[v]).astype(F32)
            p = (_exp32(t) * self.inv_s[v]).astype(F32)
            bins = _bin(t)
            pre = bins < self.lo[v]
            bnd = (bins >= self.lo[v]) & (bins <= self.hi[v])
            out["pre"][v] = p[pre].astype(F64).sum()
            idx = np.nonzero(bnd)[0]
            out["n"][v] = idx.size
            out["flags"][v] = self.flags[v] | (1 if idx.size > CAP else 0)
            keys = _pkey(p[idx[:CAP]], self.v0 + idx[:CAP])
            out["e"][v, :keys.size] = keys
        return out

    def _pprime(self, v, d, j):
        t = (np.asarray(d, dtype=F32) - self.m[v]).astype(F32)
        p = (_exp32(t) * self.inv_s[v]).astype(F32)
        bins = _bin(t)
        kept = (bins < self.lo[v]) | ((bins <= self.hi[v]) & (_pkey(p, j) >= self.cut[v]))
        return np.where(kept, (p / self.zf[v]).astype(F32), F32(0.0)).astype(F32)

    def _p4(self, rb):
        msgs = rb.view(MSG3).reshape(self.nranks, self.nvec)
        self.cut = np.full(self.nvec, np.uint64(0xFFFFFFFFFFFFFFFF), dtype=np.uint64)
        self.zf = np.zeros(self.nvec, dtype=F32)
        for v in range(self.nvec):
            fl = int(self.flags[v])
            pre = 0.0
            ents = []
            for r in range(self.nranks):
                pre += float(msgs["pre"][r, v])
                fl |= int(msgs["flags"][r, v])
                n = min(int(msgs["n"][r, v]), CAP)
                ents.append(msgs["e"][r, v, :n])
            Z = pre
            if self.truncate and not fl & 1:
                keys = np.sort(np.concatenate(ents))[::-1]
                cum = F64(pre)
                for i, kk in enumerate(keys):
                    p = _pkey_val(kk)
                    cum += F64(p)
                    c = F32(F32(cum) - p)
                    if c < self.top_p or (i == 0 and self.lo[v] == 0):
                        self.cut[v] = kk
                        Z += float(p)
                    else:
                        break
            zf = F32(Z)
            self.zf[v] = max(zf, F32(1e-12))
            self.flags[v] = fl
            if fl & 1:
                self._status |= STATUS_FALLBACK
        # per row: accept test, residual mass of this shard
        self.n_acc = np.zeros(self.B, dtype=np.int64)
        self.pick = np.zeros(self.B, dtype=np.int64)
        self.all_acc = np.zeros(self.B, dtype=bool)
        out = np.zeros((self.B, 2), dtype=F64)
        for b in range(self.B):
            alive = True if self.alive is None else bool(self.alive[b])
            n = 0
            for i in range(self.k):
                vt, vd = b * self.per + i, b * self.per + self.k + 1 + i
                x = int(self.xs[b, i])
                inr = 0 <= x < self.V
                px = self._pprime(vt, self.dx[vt], x) if inr else F32(0)
                qx = self._pprime(vd, self.dx[vd], x) if inr else F32(0)
                thr = min(F32(F32(px) / max(F32(qx), F32(1e-10))), F32(1.0))
                ok = alive and n == i and F32(self.u_acc[b, i]) < thr
                n += int(ok)
                alive = alive and ok
            self.n_acc[b], self.pick[b], self.all_acc[b] = n, min(n, self.k - 1), n == self.k
            r, pm = self._row_masses(b, degen=False)
            out[b] = (r.astype(F64).sum(), pm.astype(F64).sum())
        return out

    def _row_masses(self, b, degen):
        vp = b * self.per + (self.k if self.all_acc[b] else int(self.pick[b]))
        vq = b * self.per + self.k + 1 + int(self.pick[b])
        j = self.v0 + np.arange(self.Vr)
        dp, _ = self._vec(vp)
        pj = self._pprime(vp, dp, j)
        if self.all_acc[b] or degen:
            return pj, pj
        dq, _ = self._vec(vq)
        qj = self._pprime(vq, dq, j)
        return np.maximum((pj - qj).astype(F32), F32(0.0)).astype(F32), pj

    def _p5(self, rb):
        m4 = rb.view(F64).reshape(self.nranks, self.B, 2)
        out = np.full(self.B, -1, dtype=np.int64)
        for b in range(self.B):
            Rt = float(m4[:, b, 0].sum())
            degen = (not self.all_acc[b]) and F32(Rt) <= F32(1e-9)
            use = 1 if (self.all_acc[b] or degen) else 0
            w = m4[:, b, use]
            total = float(w.sum())
            before = float(w[:self.rank].sum())
            mine = float(w[self.rank])
            t = F64(F32(self.u_res[b])) * total
            mode = 2 if t >= total else (1 if (mine > 0 and before <= t < before + mine) else 0)
            if mode == 0:
                continue
            r, _ = self._row_masses(b, degen)
            best = -1
            if mode == 1:
                c = before + np.cumsum(r.astype(F64))
                hit = np.nonzero((r > 0) & (c > t))[0]
                best = int(hit[0]) if hit.size else -1
            if best < 0:
                nz = np.nonzero(r > 0)[0]
                best = int(nz[-1]) if nz.size else -1
            out[b] = self.v0 + best if best >= 0 else -1
        return out

    def _p6(self, rb):
        self.y = rb.view(np.int64).copy()
        return None
