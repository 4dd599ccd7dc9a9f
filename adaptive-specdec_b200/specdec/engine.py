"""Batched speculative decoding over two HuggingFace causal LMs, on B200 kernels.

Drop-in for the reference's specdec/engine.py (SpecDecodeEngine, SamplingConfig,
RunStats; engine.py:40-388): same constructor, same ``generate`` /
``generate_autoregressive`` signatures and return values, same round
structure (engine.py:1-30):

  1. feed `pending` to the draft            -> q_1, sample x_1
  2. feed x_i to the draft, i = 1..k-1      -> q_{i+1}, sample x_{i+1}
  3. feed x_k to the draft                  (commit-only)
  4. feed [pending, x_1..x_k] to the target -> p_1..p_{k+1}, ONE forward
  5. accept a tokens, roll both caches back by k-a
  6. y = residual draw (a<k) or bonus draw from p_{k+1} (a==k); pending <- y

What runs where:
* each draft step's to_probs + draw + q(x) is one ``draft_sample`` call;
* steps 5-6 are one ``verify_sample`` call (fused to_probs on the k+1 target
  and k draft vectors, accept test, residual/bonus draw);
* the rollback is ``RaggedCache.commit`` on the device (no host copy);
* attention reads the ragged cache through the verify-attention kernel
  (models are switched to attn_implementation "specdec_b200");
* the one designed host sync per round reads n_acc, y and the drafted ids
  together (the reference reads them at engine.py:309, :322-323);
* with ``cuda_graphs=True`` (the default) every fixed-shape step after the
  first round -- each draft step (forward, cache advance, draw), the
  commit-only draft forward and the target verify forward -- replays a CUDA
  graph captured once per generate call: nothing in them reads the device
  lengths back, so the eager per-layer launch overhead of the HF forwards
  (most of a round's time at small batch) is paid once.

Draws use uniforms from the round's torch.Generator, so runs are reproducible
for a seed; the random stream differs from the reference's multinomial calls,
so agreement with the reference is distributional (gate G1) and exact for
greedy decoding (gate G2).
"""
import time
from dataclasses import dataclass, field

import torch

from specdec import attention as A
from specdec.kvcache import PAGE, PagedRaggedCache, RaggedCache
from specdec.sampling import draft_sample, to_probs, verify_sample

__all__ = ["SamplingConfig", "RunStats", "SpecDecodeEngine"]


@dataclass
class SamplingConfig:
    temperature: float = 0.0     # 0 => greedy, and the generic path still applies
    top_p: float = 1.0
    top_k: int = 0

    def probs(self, logits):
        return to_probs(logits, self.temperature, self.top_p, self.top_k)


@dataclass
class RunStats:
    """Counters with the reference's definitions (engine.py:50-129)."""
    rounds: int = 0
    batch: int = 1
    proposed: int = 0
    accepted: int = 0
    emitted: int = 0
    draft_forwards: int = 0
    target_forwards: int = 0
    t_draft: float = 0.0
    t_target: float = 0.0
    t_total: float = 0.0
    offered_at: list = field(default_factory=list)
    accepted_at: list = field(default_factory=list)
    k_history: list = field(default_factory=list)
    accept_history: list = field(default_factory=list)

    def _grow(self, n):
        while len(self.offered_at) < n:
            self.offered_at.append(0)
            self.accepted_at.append(0)

    def observe(self, k, n_accepted_per_row):
        """Position i counts as offered iff the round reached it (a >= i)."""
        self._grow(k)
        for a in n_accepted_per_row:
            for i in range(min(k, a + 1)):
                self.offered_at[i] += 1
            for i in range(min(k, a)):
                self.accepted_at[i] += 1

    @property
    def acceptance_rate(self):
        return self.accepted / max(1, self.proposed)

    @property
    def alpha_conditional(self):
        return self.accepted / max(1, sum(self.offered_at))

    @property
    def mean_accepted_len(self):
        return self.emitted / max(1, self.rounds * self.batch)

    def alpha_by_position(self):
        return [a / o if o else 0.0 for a, o in zip(self.accepted_at, self.offered_at)]

    def to_dict(self):
        return {
            "rounds": self.rounds, "batch": self.batch, "proposed": self.proposed,
            "accepted": self.accepted, "emitted": self.emitted,
            "acceptance_rate": self.acceptance_rate, "alpha_conditional": self.alpha_conditional,
            "mean_accepted_len": self.mean_accepted_len, "draft_forwards": self.draft_forwards,
            "target_forwards": self.target_forwards, "t_draft": self.t_draft,
            "t_target": self.t_target, "t_total": self.t_total,
            "tokens_per_s": self.emitted / self.t_total if self.t_total else 0.0,
            "alpha_by_position": self.alpha_by_position(), "offered_at": list(self.offered_at),
            "accepted_at": list(self.accepted_at), "reached": sum(self.offered_at),
            "k_history": self.k_history, "accept_history": self.accept_history,
        }


class _RoundGraphs:
    """CUDA graphs of one generate call's fixed-shape round steps.

    Static buffers carry the inputs and outputs across replays: ``feed`` (the
    token each draft step consumes), ``u`` (draft uniforms), ``xs`` / ``qx``
    (drafted ids and q(x)), ``vin[k]`` (the target's [B, k+1] verify input)
    and ``vlog[k]`` (its logits).  A graph is captured on first use, after the
    eager first round has created every workspace, and is then replayed; a
    capture records the kernels without running them.  The caches' host
    mirrors are invalidated so that no step touches host state.
    """

    def __init__(self, eng, B, k_max, dcache, tcache, drf_buf, T, tp, tk):
        dev = eng.device
        self.eng, self.B = eng, B
        self.dcache, self.tcache, self.drf_buf = dcache, tcache, drf_buf
        self.T, self.tp, self.tk = T, tp, tk
        self.pool = torch.cuda.graph_pool_handle()
        self.feed = torch.zeros(B, 1, dtype=torch.long, device=dev)
        self.u = torch.zeros(k_max, B, dtype=torch.float32, device=dev)
        self.xs = torch.zeros(B, k_max, dtype=torch.long, device=dev)
        self.qx = torch.ones(k_max, B, dtype=torch.float32, device=dev)
        self.rows0 = torch.zeros(B, dtype=torch.long, device=dev)
        self.vin, self.vlog, self.graphs = {}, {}, {}
        self.stream = torch.cuda.Stream(device=dev)

    def _run(self, key, body):
        self.dcache.invalidate_host()
        self.tcache.invalidate_host()
        g = self.graphs.get(key)
        if g is None:
            g = torch.cuda.CUDAGraph()
            self.stream.wait_stream(torch.cuda.current_stream(self.eng.device))
            with torch.cuda.graph(g, pool=self.pool, stream=self.stream):
                body()
            torch.cuda.current_stream(self.eng.device).wait_stream(self.stream)
            self.graphs[key] = g
        g.replay()

    def draft_step(self, i):
        e, B = self.eng, self.B

        def body():
            logits = e._forward(e.draft, self.dcache, self.feed)[:, -1]
            self.dcache.advance(1)
            self.drf_buf[:, i].copy_(logits)
            x, q = draft_sample(self.drf_buf[:, i], self.u[i], self.T, self.tp, self.tk)
            self.xs[:, i].copy_(x)
            self.qx[i].copy_(q)
            self.feed.copy_(x.view(B, 1))
        self._run(("draft", i), body)

    def draft_commit(self):
        e = self.eng

        def body():
            e._forward(e.draft, self.dcache, self.feed, rows_last=self.rows0)
            self.dcache.advance(1)
        self._run(("commit",), body)

    def target(self, k):
        e = self.eng
        if k not in self.vin:
            self.vin[k] = torch.zeros(self.B, k + 1, dtype=torch.long, device=e.device)

        def body():
            self.vlog[k] = e._forward(e.target, self.tcache, self.vin[k])
            self.tcache.advance(k + 1)
        self._run(("target", k), body)
        return self.vlog[k]


class _NullCtx:
    def __enter__(self):
        return None

    def __exit__(self, *a):
        return False


class SpecDecodeEngine:
    """Speculative decoding for a (target, draft) pair sharing a tokenizer."""

    def __init__(self, target, draft, tokenizer, device=None, capacity=4096, nvtx=False,
                 time_phases=False, cuda_graphs=True, fused_qkv=True, fused_norm_mlp=True,
                 paged_kv=False, kv_pages=None):
        self.target = target.eval()
        self.draft = draft.eval()
        self.tok = tokenizer
        self.device = torch.device(device) if device is not None else \
            next(target.parameters()).device
        if self.device.type != "cuda":
            raise RuntimeError("SpecDecodeEngine runs on the B200 kernels (no CPU fallback)")
        self.capacity = capacity
        self.nvtx = nvtx
        self.time_phases = time_phases
        self.cuda_graphs = bool(cuda_graphs)
        tcfg, dcfg = target.config, draft.config
        if tcfg.vocab_size != dcfg.vocab_size:
            raise ValueError(
                f"target vocab {tcfg.vocab_size} != draft vocab {dcfg.vocab_size}; "
                "speculative decoding requires a shared tokenizer")
        self.vocab_size = tcfg.vocab_size
        self.eos_ids = self._eos_ids(tokenizer, tcfg)
        A.register()
        for m in (self.target, self.draft):
            m.set_attn_implementation(A.IMPL)
        # fused_qkv (default): one QKV GEMM and one norm + RoPE + KV-append
        # kernel per attention layer of a bf16 model (specdec.fused_attention;
        # layers of other dtypes keep their own forward)
        self.fused_qkv = bool(fused_qkv)
        # fused_norm_mlp (default): every RMSNorm one launch, every SiLU-gated
        # MLP one gate / up GEMM + one activation launch (specdec.fused_layers)
        self.fused_norm_mlp = bool(fused_norm_mlp)
        if self.fused_norm_mlp:
            from specdec import fused_layers as FL
            for m in (self.target, self.draft):
                FL.install(m)
        # paged_kv: both caches are PagedRaggedCache pools sized from the
        # prompts' own lengths (kv_pages: pages per pool instead)
        self.paged_kv = bool(paged_kv)
        self.kv_pages = kv_pages
        if self.fused_qkv:
            from specdec import fused_attention as FA
            for m in (self.target, self.draft):
                FA.install(m)

    @staticmethod
    def _eos_ids(tok, cfg):
        ids = set()
        for src in (getattr(tok, "eos_token_id", None), getattr(cfg, "eos_token_id", None)):
            if isinstance(src, (list, tuple)):
                ids.update(int(i) for i in src)
            elif src is not None:
                ids.add(int(src))
        return ids

    # ---- plumbing ----------------------------------------------------------
    def _mk_cache(self, model, batch, plen=None, max_new=0, k_max=16):
        n_layers = model.config.num_hidden_layers
        if not self.paged_kv:
            return RaggedCache(n_layers, batch, self.capacity, self.device, attn_impl=A.IMPL)
        n_pages = self.kv_pages
        if n_pages is None:
            # a row ends within plen + max_new + k_max + 1 tokens of its own
            # and grows by one per round after that (at most max_new rounds);
            # a round holds up to k_max + 1 more before its commit
            pl = plen.to("cpu", torch.long)
            per = (pl + 2 * int(max_new) + 2 * (int(k_max) + 1)).clamp(max=self.capacity)
            n_pages = int(((per + PAGE - 1) // PAGE).sum()) + 1
        return PagedRaggedCache(n_layers, batch, self.capacity, self.device, attn_impl=A.IMPL,
                                n_pages=n_pages)

    def _forward(self, model, cache, tokens, valid=None, rows_last=None):
        """Forward `tokens` [B, q] against `cache`.

        Returns logits [B, q, V], or [B, V] at per-row positions `rows_last`
        (the LM head then runs on B hidden states only).  A model carrying a
        ``specdec_head(hidden, ids)`` callable gets its logits from it instead
        of ``lm_head``; ``ids`` are the input tokens at the same positions.
        """
        q = tokens.shape[1]
        mask = cache.attn_mask(q, model.dtype, valid=valid)
        # cache_position given explicitly: derived from the cache it would read
        # the device lengths back on the host (and could not be graph-captured)
        hidden = model.model(input_ids=tokens, position_ids=cache.positions(q),
                             attention_mask=mask, past_key_values=cache,
                             cache_position=cache.cache_position(q),
                             use_cache=True).last_hidden_state
        if rows_last is not None:
            rows = torch.arange(hidden.shape[0], device=hidden.device)
            hidden = hidden[rows, rows_last]
            tokens = tokens[rows, rows_last]
        head = getattr(model, "specdec_head", None)
        if head is not None:
            # a replacement LM head that also sees the token each hidden state
            # was computed at (the config-5 benchmark's shared-prior drafts)
            return head(hidden, tokens)
        return model.lm_head(hidden)

    def _range(self, name):
        return torch.profiler.record_function(name) if self.nvtx else _NullCtx()

    def _prefill(self, model, cache, input_ids, plen):
        """Right-padded prefill; logits [B, V] at each row's last real token."""
        if isinstance(cache, PagedRaggedCache):
            cache.reserve_prefill(input_ids.shape[1], plen)
        logits = self._forward(model, cache, input_ids, valid=plen, rows_last=plen - 1)
        cache.set_lengths(plen)
        return logits

    def _sync_phase(self):
        if self.time_phases:
            torch.cuda.synchronize(self.device)

    # ---- main loop ---------------------------------------------------------
    @torch.inference_mode()
    def generate(self, input_ids, plen, max_new_tokens, sampling=None, controller=None,
                 seed=None, k_fixed=None):
        """input_ids [B, P] right-padded, plen [B] real prompt lengths.

        Returns (list of generated id lists, RunStats).
        """
        sp = sampling or SamplingConfig()
        T, tp, tk = sp.temperature, sp.top_p, sp.top_k
        dev = self.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(int(seed) if seed is not None else int(torch.seed() % (2 ** 63)))
        B = input_ids.shape[0]
        input_ids = input_ids.to(dev)
        plen = plen.to(dev)
        k_cap = int(k_fixed) if k_fixed is not None else int(getattr(controller, "k_max", 16))
        tcache = self._mk_cache(self.target, B, plen, max_new_tokens, k_cap)
        dcache = self._mk_cache(self.draft, B, plen, max_new_tokens, k_cap)
        paged = self.paged_kv
        st = RunStats(batch=B)
        t0 = time.perf_counter()

        with self._range("prefill"):
            tlog = self._prefill(self.target, tcache, input_ids, plen)
            self._prefill(self.draft, dcache, input_ids, plen)
            st.target_forwards += 1
            st.draft_forwards += 1

        pending, _ = draft_sample(tlog, torch.rand(B, generator=gen, device=dev), T, tp, tk)
        pend_l = pending.tolist()
        out = [[int(pend_l[b])] for b in range(B)]
        done_l = [int(pend_l[b]) in self.eos_ids for b in range(B)]
        st.emitted += B
        drf_buf = None
        graphs = None
        K_BUF = 8

        while not all(done_l):
            k = int(k_fixed) if k_fixed is not None else controller.propose_k()
            k = max(1, k)
            r0 = time.perf_counter()
            if drf_buf is None or drf_buf.shape[1] < k:
                drf_buf = torch.empty(B, max(k, K_BUF), self.vocab_size, dtype=self.draft.dtype,
                                      device=dev)
                graphs = None                      # graphs write into drf_buf
            # the first round (and any round after drf_buf grew) runs eagerly and
            # warms every workspace; later rounds replay graphs
            use_g = self.cuda_graphs and st.rounds > 0 and graphs is not None
            if self.cuda_graphs and graphs is None and st.rounds > 0:
                graphs = _RoundGraphs(self, B, drf_buf.shape[1], dcache, tcache, drf_buf,
                                      T, tp, tk)
                use_g = True
            if paged:
                # pages for this round's k + 1 tokens per cache, from the
                # lengths read back at the end of the last round (no sync)
                dcache.reserve(k + 1)
                tcache.reserve(k + 1)
            conf = torch.ones(B, device=dev)
            u_draft = torch.rand(k, B, generator=gen, device=dev)
            d0 = time.perf_counter()
            k_eff = k
            with self._range("draft_loop"):
                if use_g:
                    graphs.feed.copy_(pending.view(B, 1))
                    graphs.u[:k].copy_(u_draft)
                    for i in range(k):
                        graphs.draft_step(i)
                        st.draft_forwards += 1
                        if controller is not None:
                            conf = conf * graphs.qx[i]
                            if controller.should_stop_drafting(i + 1, conf):
                                k_eff = i + 1
                                break
                    graphs.draft_commit()
                    st.draft_forwards += 1
                    xs = graphs.xs[:, :k_eff]
                else:
                    xs = torch.empty(B, k, dtype=torch.long, device=dev)
                    feed = pending.view(B, 1)
                    for i in range(k):
                        logits = self._forward(self.draft, dcache, feed)[:, -1]
                        dcache.advance(1)
                        st.draft_forwards += 1
                        drf_buf[:, i].copy_(logits)
                        x, qx = draft_sample(drf_buf[:, i], u_draft[i], T, tp, tk)
                        xs[:, i] = x
                        feed = x.view(B, 1)
                        if controller is not None:
                            conf = conf * qx
                            if controller.should_stop_drafting(i + 1, conf):
                                k_eff = i + 1
                                break
                    # commit-only forward: puts the last drafted token in the draft cache
                    self._forward(self.draft, dcache, feed,
                                  rows_last=torch.zeros(B, dtype=torch.long, device=dev))
                    dcache.advance(1)
                    st.draft_forwards += 1
                    xs = xs[:, :k_eff]
            self._sync_phase()
            st.t_draft += time.perf_counter() - d0

            v0 = time.perf_counter()
            with self._range("verify"):
                if use_g:
                    if k_eff not in graphs.vin:
                        graphs.vin[k_eff] = torch.zeros(B, k_eff + 1, dtype=torch.long,
                                                        device=dev)
                    vin = graphs.vin[k_eff]
                    vin[:, :1].copy_(pending.view(B, 1))
                    vin[:, 1:].copy_(xs)
                    vlog = graphs.target(k_eff)
                else:
                    verify_in = torch.cat([pending.view(B, 1), xs], dim=1)
                    vlog = self._forward(self.target, tcache, verify_in)
                    tcache.advance(k_eff + 1)
                st.target_forwards += 1
            self._sync_phase()
            st.t_target += time.perf_counter() - v0

            with self._range("accept"):
                u_acc = torch.rand(B, k_eff, generator=gen, device=dev)
                u_res = torch.rand(B, generator=gen, device=dev)
                alive = torch.tensor([not d for d in done_l], device=dev)
                n_acc, y = verify_sample(vlog, drf_buf[:, :k_eff], xs, u_acc, u_res, T, tp, tk,
                                         alive=alive)
                tcache.commit(n_acc, k_eff)
                dcache.commit(n_acc, k_eff)
                # the one designed host sync of the round (with the paged
                # caches' lengths, for the next round's page reservation)
                cols = [n_acc.view(B, 1), y.view(B, 1), xs]
                if paged:
                    cols += [tcache.lengths.view(B, 1), dcache.lengths.view(B, 1)]
                host = torch.cat(cols, dim=1).tolist()
                if paged:
                    tcache.set_host_lengths([r[-2] for r in host])
                    dcache.set_host_lengths([r[-1] for r in host])
            n_acc_l = [r[0] for r in host]

            st.rounds += 1
            st.proposed += k_eff * B
            st.accepted += sum(n_acc_l)
            st.observe(k_eff, n_acc_l)
            st.k_history.append(k_eff)
            st.accept_history.append(n_acc_l)
            for b in range(B):
                if done_l[b]:
                    continue
                row = host[b]
                for j in range(n_acc_l[b]):
                    tok = row[2 + j]
                    out[b].append(tok)
                    st.emitted += 1
                    if tok in self.eos_ids or len(out[b]) >= max_new_tokens:
                        done_l[b] = True
                        break
                if done_l[b]:
                    continue
                out[b].append(row[1])
                st.emitted += 1
                if row[1] in self.eos_ids or len(out[b]) >= max_new_tokens:
                    done_l[b] = True
            pending = y

            if controller is not None:
                controller.update(k_eff, n_acc_l, time.perf_counter() - r0,
                                  t_draft_fwd=st.t_draft / max(1, st.draft_forwards),
                                  t_target_fwd=st.t_target / max(1, st.target_forwards))

        st.t_total = time.perf_counter() - t0
        return out, st

    # ---- baseline ----------------------------------------------------------
    @torch.inference_mode()
    def generate_autoregressive(self, input_ids, plen, max_new_tokens, sampling=None, seed=None):
        """Target-only decoding through the same cache, attention and sampling kernels."""
        sp = sampling or SamplingConfig()
        T, tp, tk = sp.temperature, sp.top_p, sp.top_k
        dev = self.device
        gen = torch.Generator(device=dev)
        gen.manual_seed(int(seed) if seed is not None else int(torch.seed() % (2 ** 63)))
        B = input_ids.shape[0]
        input_ids, plen = input_ids.to(dev), plen.to(dev)
        cache = self._mk_cache(self.target, B, plen, max_new_tokens, 1)
        st = RunStats(batch=B)
        t0 = time.perf_counter()
        logits = self._prefill(self.target, cache, input_ids, plen)
        st.target_forwards += 1
        nxt, _ = draft_sample(logits, torch.rand(B, generator=gen, device=dev), T, tp, tk)
        nl = nxt.tolist()
        out = [[int(nl[b])] for b in range(B)]
        done_l = [int(nl[b]) in self.eos_ids for b in range(B)]
        st.emitted += B
        while not all(done_l):
            if isinstance(cache, PagedRaggedCache):
                cache.reserve(1)
            logits = self._forward(self.target, cache, nxt.view(B, 1),
                                   rows_last=torch.zeros(B, dtype=torch.long, device=dev))
            cache.advance(1)
            st.target_forwards += 1
            nxt, _ = draft_sample(logits, torch.rand(B, generator=gen, device=dev), T, tp, tk)
            nl = nxt.tolist()
            for b in range(B):
                if done_l[b]:
                    continue
                out[b].append(nl[b])
                st.emitted += 1
                if nl[b] in self.eos_ids or len(out[b]) >= max_new_tokens:
                    done_l[b] = True
        st.t_total = time.perf_counter() - t0
        st.t_target = st.t_total
        return out, st
