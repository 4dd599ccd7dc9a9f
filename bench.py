"""Benchmark of the fused verify round (config 2) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--mode sample|greedy]

A step is one verify call over one batch: B=64 rows, k=4 draft tokens,
V=151936, bf16 target [64,5,V] and draft [64,4,V] logits, T=0.7, top-p 0.9
(mode greedy: T=0, target only).  Rows are sharded across ranks with no
collective (weak scaling: every rank verifies its own 64-row batch); `value`
is rows/s summed over ranks, timed on the device with CUDA events as the max
over ranks.  Two input sets (350 MB, > the 126 MB L2) alternate so no step
reads logits left in L2 by the previous one.  Steps are replayed from CUDA
graphs of up to 100 calls.

`e2e` is the same metric through the public API from pinned host buffers:
every step copies that step's logits host->device, runs verify_sample and
reads n_acc / y back.  `cpu_baseline` times the CPU oracle (a restatement of
the reference path, single thread) on 64 rows of the same workload.
`--impl reference` times that CPU path on the host cores alone.
"""
import argparse
import json
import os
import pathlib
import statistics
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
for _p in (str(ROOT / "adaptive-specdec_b200"), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

B, K_DRAFT, VOCAB = 64, 4, 151936
T_SAMPLE, TOP_P = 0.7, 0.9
NBUF = 2
GRAPH_CALLS = 100


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--mode", default="sample",
                    choices=["sample", "greedy", "attn", "vshard", "vshard-greedy", "engine",
                             "adaptive", "rejection"])
    ap.add_argument("--new-tokens", type=int, default=None,
                    help="--mode engine / adaptive: tokens per row (256 / 512)")
    ap.add_argument("--rows", type=int, default=8, help="--mode adaptive: rows per GPU")
    ap.add_argument("--temperature", type=float, default=T_SAMPLE,
                    help="--mode sample: temperature (config 2: 0.7)")
    ap.add_argument("--top-p", type=float, default=TOP_P, help="--mode sample: top-p (config 2: 0.9)")
    ap.add_argument("--flat", action="store_true",
                    help="--mode sample: N(0, 1) logits (random-model-like flat rows) instead of "
                         "config 2's peaked ones")
    ap.add_argument("--beta-hi", type=float, default=48.0,
                    help="--mode adaptive: shared-prior strength of the high-agreement phase")
    ap.add_argument("--beta-lo", type=float, default=5.0,
                    help="--mode adaptive: shared-prior strength of the low-agreement phase")
    ap.add_argument("--no-fused-qkv", dest="fused_qkv", action="store_false",
                    help="--mode engine / adaptive: the layers' own forwards instead of one QKV "
                         "GEMM + the fused norm / RoPE / KV-append kernel per attention layer")
    ap.add_argument("--no-fused-norm-mlp", dest="fused_norm_mlp", action="store_false",
                    help="--mode engine / adaptive: the RMSNorm and MLP modules' own forwards "
                         "instead of one launch per norm and a fused gate / up GEMM + activation")
    ap.add_argument("--profile-range", action="store_true",
                    help="--mode engine: cudaProfilerStart / Stop around the timed generate "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--paged", action="store_true",
                    help="--mode attn: time the paged-cache kernel (the same K/V scattered over "
                         "128-token pages in a random order); --mode engine / adaptive: paged "
                         "caches")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="default run: skip the greedy / attention / rejection-sampler lines "
                         "reported under 'also'")
    ap.add_argument("--attn-rows", type=int, default=64, help="--mode attn: rows (config 3: 64)")
    ap.add_argument("--attn-ctx", default="512:8192",
                    help="--mode attn: context lengths uniform in LO:HI (config 3: 512:8192; "
                         "the engine's config-4 rounds: about 512:640)")
    ap.add_argument("--attn-queries", type=int, default=5,
                    help="--mode attn: queries per row (verify: k + 1 = 5; a draft step: 1)")
    ap.add_argument("--attn-heads", default="32:8",
                    help="--mode attn: query:kv heads (Qwen3-8B 32:8, Qwen3-0.6B 16:8)")
    return ap.parse_args()


def metric_name(mode, T=T_SAMPLE, tp=TOP_P, flat=False):
    if mode == "greedy":
        return "verify rows/s (B=64,k=4,V=151936 bf16, greedy)"
    return (f"verify rows/s (B=64,k=4,V=151936 bf16, T={T:g} top-p {tp:g}"
            + (", flat N(0,1) logits)" if flat else ")"))


def workload_config(mode, n, T=T_SAMPLE, tp=TOP_P, flat=False):
    knobs = "greedy" if mode == "greedy" else f"T={T:g} top-p {tp:g}"
    return {"workload": f"config 2 fused verify round, {knobs}"
                        + (", flat N(0,1) logits" if flat else ""),
            "rows_per_gpu": B, "k": K_DRAFT, "vocab": VOCAB, "logits": "bf16",
            "parallelism": f"row-sharded x{n}, no collective",
            "l2": "2 input sets of 175 MB alternate (> 126 MB L2)"}


# ---------------------------------------------------------------------------
# CPU path (oracle restatement of the reference), used by both arms
# ---------------------------------------------------------------------------
def _cpu_inputs(rows, seed):
    import numpy as np
    import torch
    from specdec import workloads as W
    g = torch.Generator().manual_seed(seed)
    tgt = W.zipf_logits(rows * (K_DRAFT + 1), VOCAB, g).reshape(rows, K_DRAFT + 1, VOCAB)
    drf = tgt[:, :K_DRAFT] + torch.randn(rows, K_DRAFT, VOCAB, generator=g) * W.DRAFT_SIGMA
    tgt = tgt.bfloat16().float().numpy()
    drf = drf.bfloat16().float().numpy()
    rng = np.random.default_rng(seed)
    xs = tgt[:, :K_DRAFT].argmax(-1)
    xs = np.where(rng.random((rows, K_DRAFT)) < 0.5, xs, rng.integers(0, VOCAB, (rows, K_DRAFT)))
    ua = rng.random((rows, K_DRAFT), dtype=np.float32)
    ur = rng.random(rows, dtype=np.float32)
    return tgt, drf, xs, ua, ur


def _load_ref_sampling():
    """The reference's own specdec/sampling.py, from the offline install in
    baseline/_ref (loaded under its own module name: the package name
    `specdec` is also this repository's).  None when it is not installed."""
    import importlib.util
    path = ROOT / "baseline" / "_ref" / "specdec" / "sampling.py"
    if not path.exists():
        return None
    spec = importlib.util.spec_from_file_location("_ref_specdec_sampling", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ref_inverse_cdf(probs, u):
    """Smallest j with float64 cumsum(probs)[j] > u * sum (the uniforms-as-
    tensors stand-in for torch.multinomial, BASELINE's CPU plan)."""
    import torch
    c = probs.double().cumsum(-1)
    tgt = u.double()[:, None] * c[:, -1:]
    j = (c <= tgt).sum(-1)
    return j.clamp(max=probs.shape[-1] - 1)


def ref_verify(ref, tgt, drf, xs, ua, ur, T, tp):
    """One verify round through the reference's to_probs / gather_prob /
    residual_probs and its accept loop (reference specdec/engine.py:282-303),
    uniforms passed in as tensors."""
    import torch
    B, k1, _ = tgt.shape
    k = k1 - 1
    ps = [ref.to_probs(tgt[:, i, :], T, tp) for i in range(k1)]
    qs = ps[:k] if drf is None else [ref.to_probs(drf[:, i, :], T, tp) for i in range(k)]
    n_acc = torch.zeros(B, dtype=torch.long)
    alive = torch.ones(B, dtype=torch.bool)
    for i in range(k):
        ratio = ref.gather_prob(ps[i], xs[:, i]) / ref.gather_prob(qs[i], xs[:, i]).clamp_min(1e-10)
        ok = (ua[:, i] < ratio.clamp(max=1.0)) & alive & (n_acc == i)
        n_acc = n_acc + ok.long()
        alive = alive & ok
    all_acc = n_acc == k
    pick = n_acc.clamp(max=k - 1)
    p_stop = torch.stack(ps[:k], 1)[torch.arange(B), pick]
    q_stop = torch.stack(qs, 1)[torch.arange(B), pick]
    y_res = _ref_inverse_cdf(ref.residual_probs(p_stop, q_stop), ur)
    y_bonus = _ref_inverse_cdf(ps[k], ur)
    return n_acc, torch.where(all_acc, y_bonus, y_res)


def _ref_inputs(rows, seed, greedy):
    import torch
    tgt, drf, xs, ua, ur = _cpu_inputs(rows, seed)
    bf = lambda a: torch.from_numpy(a).bfloat16()
    return (bf(tgt), None if greedy else bf(drf), torch.from_numpy(xs).long(),
            torch.from_numpy(ua), torch.from_numpy(ur))


def ref_rate(mode, rows, budget_s, max_steps, warmup=1):
    """rows/s of the reference CPU path on `rows`-row batches, all host threads.
    Returns (rows/s, timed steps, kind, threads)."""
    import torch
    greedy = mode == "greedy"
    T, tp = (0.0, 1.0) if greedy else (T_SAMPLE, TOP_P)
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    ref = _load_ref_sampling()
    inp = _ref_inputs(rows, 11, greedy)
    if ref is None:                    # the port, when the reference is not installed
        from oracle import sampling_oracle as O
        args = tuple(None if t is None else t.float().numpy() for t in inp)
        fn = lambda: O.verify(args[0], args[0][:, :K_DRAFT] if greedy else args[1], args[2],
                              args[3], args[4], T, tp, 0)
        kind = "port"
    else:
        fn = lambda: ref_verify(ref, *inp, T, tp)
        kind = "reference"
    t0 = time.perf_counter()
    for _ in range(max(1, warmup)):
        fn()
    t_step = (time.perf_counter() - t0) / max(1, warmup)
    steps = max(1, min(max_steps, int(budget_s / max(t_step, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(steps):
        fn()
    dt = time.perf_counter() - t0
    return rows * steps / dt, steps, kind, cores


def cpu_baseline(mode, rows=16):
    """The reference CPU path on a bounded 16-row sample, all host threads."""
    rate, steps, kind, cores = ref_rate(mode, rows, budget_s=15.0, max_steps=8)
    return rate, steps, kind, cores, rows


def reference_arm(a):
    """--impl reference: the reference's own CPU implementation of the path
    (its specdec/sampling.py to_probs / gather_prob / residual_probs and the
    accept loop of engine.py:282-303, installed offline into baseline/_ref) on
    all host threads, one full config-2 batch (B=64) per step.  The number of
    timed steps is bounded (at most --steps, about a minute of work) so any
    --steps finishes within minutes; rank 0 only.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wu = min(max(a.warmup, 3), 5)           # >= 3 warm-up rounds, bounded (~2 s each on CPU)
    rate, steps, kind, cores = ref_rate(a.mode, B, budget_s=60.0, max_steps=a.steps, warmup=wu)
    src = ("specdec/sampling.py of the reference (baseline/_ref), torch CPU"
           if kind == "reference" else "oracle/sampling_oracle.py (reference not installed)")
    print(json.dumps({
        "impl": "reference", "metric": metric_name(a.mode), "value": rate, "unit": "rows/s",
        "n_gpus": a.gpus, "steps": steps, "warmup": wu,
        "ms_per_step": 1e3 * B / rate, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded config-2 logits, bf16 inputs)",
        "config": workload_config(a.mode, 1),
        "cpu_baseline": {"value": rate, "unit": "rows/s", "cores": cores, "kind": kind,
                         "sample": f"{steps} full B=64 verify rounds through {src}, "
                                   f"{cores} threads"},
        "e2e": {"value": rate, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}))


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML polling thread)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x20: "sync_boost", 0x40: "sw_thermal_slowdown",
               0x80: "hw_thermal_slowdown", 0x100: "hw_power_brake_slowdown",
               0x200: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons = [], 0
        self._stop = threading.Event()
        self.max_mhz = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            try:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(
                    "GPU-" + str(torch.cuda.get_device_properties(index).uuid))
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                fn = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    self.nv.nvmlDeviceGetCurrentClocksThrottleReasons
                self.reasons |= fn(self.h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self.nv is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def attn_bench(a):
    """--mode attn: verify attention at config 3 (one layer of the Qwen3-8B
    shape: B=64 rows, 32 query / 8 kv heads x 128, 5 queries per row, context
    lengths uniform in [512, 8192]), one GPU.  Algorithmic bytes: every live
    K and V row read once, plus Q and the output."""
    import torch
    from specdec import attention as A
    from specdec import workloads as W
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    B, D, ql = a.attn_rows, 128, a.attn_queries
    Hq, Hkv = (int(x) for x in a.attn_heads.split(":"))
    lo, hi = (int(x) for x in a.attn_ctx.split(":"))
    lens = W.attn_lengths(B, lo, hi, seed=0)
    cfg3 = (lo, hi, ql, Hq, Hkv) == (512, 8192, 5, 32, 8)
    C = int(lens.max()) + ql + 3
    if a.paged:
        from specdec.kvcache import PAGE
        C = -(-C // PAGE) * PAGE
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(B, Hq, ql, D, generator=g, device=dev).to(torch.bfloat16)
    kc = torch.randn(B, Hkv, C, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(B, Hkv, C, D, generator=g, device=dev).to(torch.bfloat16)
    lens_d = lens.to(dev)
    out = torch.empty(B, ql, Hq, D, dtype=torch.bfloat16, device=dev)
    live = int((lens + ql).sum())
    bytes_call = live * Hkv * D * 2 * 2 + 2 * q.numel() * 2
    flops_call = sum(4 * Hq * ql * (int(n) + (ql + 1) // 2) * D for n in lens)
    # correctness before timing: eight rows spread over the length range
    # against the fp32 rule (key s visible to query j of row b iff
    # s <= len[b] + j); a mismatch aborts the bench
    A.verify_attention(q, kc, vc, lens_d, out=out)
    torch.cuda.synchronize(dev)
    rows = sorted(range(B), key=lambda b: int(lens[b]))[::max(1, B // 8)][:8]
    worst = 0.0
    for b in rows:
        n = int(lens[b]) + ql
        kf = kc[b, :, :n].float().repeat_interleave(Hq // Hkv, dim=0)
        vf = vc[b, :, :n].float().repeat_interleave(Hq // Hkv, dim=0)
        sc = torch.einsum("hqd,hkd->hqk", q[b].float(), kf) * D ** -0.5
        lim = int(lens[b]) + torch.arange(ql, device=dev).view(1, ql, 1)
        sc = sc.masked_fill(torch.arange(n, device=dev).view(1, 1, n) > lim, float("-inf"))
        ref = torch.einsum("hqk,hkd->qhd", torch.softmax(sc, -1), vf)
        worst = max(worst, float((out[b].float() - ref).abs().max()))
    if not worst < 3e-2:
        raise SystemExit(f"verify attention differs from the fp32 rule: max abs error {worst}")
    bt = None
    if a.paged:
        # the same K / V over pages of one pool in a random page order; the
        # paged call must reproduce the contiguous output bit for bit
        Wp = C // PAGE
        perm = torch.randperm(B * Wp, generator=torch.Generator().manual_seed(0)).to(dev)

        def to_pool(c):
            pages = c.view(B, Hkv, Wp, PAGE, D).permute(0, 2, 1, 3, 4).reshape(B * Wp, Hkv,
                                                                                 PAGE, D)
            pool = torch.empty_like(pages)
            pool[perm] = pages
            return pool
        kc, vc = to_pool(kc), to_pool(vc)
        bt = perm.view(B, Wp).to(torch.int32).contiguous()
        out_c = out.clone()
        A.verify_attention(q, kc, vc, lens_d, out=out, block_table=bt)
        torch.cuda.synchronize(dev)
        if not torch.equal(out, out_c):
            raise SystemExit("paged verify attention differs from the contiguous cache")
    # caches smaller than L2 (short contexts): rotate over copies holding
    # more than 2x L2 between them, as a forward's layers would
    kv_bytes = 2 * kc.numel() * kc.element_size()
    nrep = max(1, -(-(2 * 126 * 2 ** 20) // kv_bytes)) if kv_bytes < 2 * 126 * 2 ** 20 else 1
    sets = [(kc, vc)] + [(kc.clone(), vc.clone()) for _ in range(nrep - 1)]
    s = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(s):
        for i in range(max(3, a.warmup)):
            A.verify_attention(q, *sets[i % nrep], lens_d, out=out, block_table=bt)
        torch.cuda.synchronize(dev)
        steps = max(5, min(a.steps, 200))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(dev.index or 0) as clk:
            e0.record(s)
            for i in range(steps):
                A.verify_attention(q, *sets[i % nrep], lens_d, out=out, block_table=bt)
            e1.record(s)
            torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / steps
    gbs = bytes_call / (ms * 1e-3) / 1e9
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = peaks.get("hbm_gbs") or 6650.0
    print(json.dumps({
        "metric": ("verify attention GB/s (config 3, one layer: B=64, 32q/8kv x 128, 5 queries, "
                   "len U[512,8192])" if cfg3 and B == 64 else
                   f"verify attention GB/s (one layer: B={B}, {Hq}q/{Hkv}kv x {D}, {ql} queries, "
                   f"len U[{lo},{hi}])"), "value": gbs, "unit": "GB/s", "n_gpus": 1, "steps": steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) q / k / v)",
        "config": {"workload": ("config 3 verify attention, one layer" if cfg3 else
                                f"verify attention, one layer, len U[{lo},{hi}]") +
                   ("" if B == 64 else f" ({B} rows)") +
                   (", paged cache (128-token pages, random order)" if a.paged else "") +
                   (", mma.sync kernel" if os.environ.get("SD_ATTN_KERNEL", "")[:1] == "m"
                    else ""), "rows": B, "Hq": Hq,
                   "Hkv": Hkv, "head_dim": D, "queries": ql, "live_keys": live,
                   "checked": f"8 rows vs the fp32 mask rule before timing, max abs error "
                              f"{worst:.2e}",
                   "l2": ("one layer reads >1 GB of K/V (> 126 MB L2)" if nrep == 1 else
                          f"{nrep} cache copies rotated ({nrep * kv_bytes / 1e6:.0f} MB of K/V "
                          f"> 126 MB L2)")},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "tflops": flops_call / (ms * 1e-3) / 1e12,
                     "scope": f"{bytes_call} algorithmic bytes per call / event-timed call"},
        "gpu_launches": 2 * steps, "clocks": clk.summary()}))


def vshard_bench(a):
    """--mode vshard / vshard-greedy: the vocabulary-sharded verify round.

    Every rank holds V/N columns of the same config-2 batch (B=64, k=4) and
    runs specdec.sharded.verify_sharded: the local phase kernels plus the
    round's NCCL collectives (5 for sampling, 1 for greedy) and the host read
    of the status word.  Total work is fixed as N grows (strong scaling);
    value = rows verified per second by the whole job, device-timed with CUDA
    events on the current stream, max over ranks.
    """
    import torch
    import torch.distributed as dist
    from specdec import sampling as S
    from specdec import sharded as SH
    from specdec import workloads as W
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    greedy = a.mode == "vshard-greedy"
    T, tp = (0.0, 1.0) if greedy else (T_SAMPLE, TOP_P)
    vs = SH.even_split(VOCAB, world)
    sl = slice(vs[rank], vs[rank + 1])
    inputs = []
    for i in range(NBUF):
        tgt, drf = W.cfg2_logits(B, K_DRAFT, VOCAB, seed=i, device=dev)
        xs, _ = S.draft_sample(drf.reshape(-1, VOCAB), torch.rand(
            B * K_DRAFT, generator=torch.Generator(device=dev).manual_seed(i), device=dev), T, tp)
        ua, ur = W.uniforms(B, K_DRAFT, seed=i, device=dev)
        inputs.append((tgt[..., sl].contiguous(), drf[..., sl].contiguous(),
                       xs.view(B, K_DRAFT), ua, ur))
        del tgt, drf
    comm = SH.ProcessGroupCollectives() if world > 1 else _SelfComm()
    backend = SH.CudaShardBackend(dev)

    def step(i):
        t, d, xs, ua, ur = inputs[i % NBUF]
        return SH.verify_sharded(t, None if greedy else d, xs, ua, ur, vs, comm, temperature=T,
                                 top_p=tp, backend=backend)

    for i in range(max(3, a.warmup)):
        step(i)
    torch.cuda.synchronize(dev)
    steps = max(5, min(a.steps, 2000))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clk:
        e0.record()
        for i in range(steps):
            step(i)
        e1.record()
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    per_rank = W.bytes_per_verify(B, K_DRAFT, vs[rank + 1] - vs[rank], greedy=greedy)
    line = {
        "metric": "vocab-sharded verify rows/s (B=64,k=4,V=151936 bf16, " +
                  ("greedy)" if greedy else "T=0.7 top-p 0.9)"),
        "value": B * steps / (ms / 1e3), "unit": "rows/s", "n_gpus": world, "steps": steps,
        "warmup": a.warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded config-2 logits, see specdec/workloads.py)",
        "config": {"workload": "config 2 verify round, vocabulary sharded " +
                               ("(greedy)" if greedy else "(T=0.7 top-p 0.9)"),
                   "rows": B, "k": K_DRAFT, "vocab": VOCAB, "columns_per_gpu": vs[1] - vs[0],
                   "parallelism": f"vocab-sharded x{world}, "
                                  f"{1 if greedy else 5} collectives per round",
                   "logits_bytes_per_gpu": per_rank},
        "gpu_launches": (2 if greedy else 7) * steps, "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


class _NoTok:
    """Tokenizer stand-in: random-init models have no end-of-sequence token."""
    eos_token_id = None


def _qwen_pair(dev):
    """Random-init bf16 models (N(0, 0.02), no checkpoints offline): the
    Qwen3-8B target shape (36 layers, 4096 hidden, 32/8 heads x 128, FFN 12288,
    V 151936, RMSNorm, rope theta 1e6) and the Qwen3-0.6B draft shape (28
    layers, 1024 hidden, 16/8 heads x 128, FFN 3072, tied embeddings)."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    common = dict(vocab_size=VOCAB, head_dim=128, num_key_value_heads=8, rope_theta=1e6,
                  max_position_embeddings=16384, rms_norm_eps=1e-6, initializer_range=0.02)
    tcfg = Qwen3Config(hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
                       num_attention_heads=32, tie_word_embeddings=False, **common)
    dcfg = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                       num_attention_heads=16, tie_word_embeddings=True, **common)
    torch.manual_seed(0)
    with torch.device(dev):
        target = Qwen3ForCausalLM(tcfg).to(torch.bfloat16).eval()
        draft = Qwen3ForCausalLM(dcfg).to(torch.bfloat16).eval()
    return target, draft


class _SharedPrior:
    """The config-5 agreement knob.  Target logits for the draft positions do
    not exist when the draft runs, so "mixing the draft toward the target" is
    realised by a component both models share: each model's logits at a
    position get beta * z(x) added, where x is the token at that position and
    z(x) = U[x] @ W is a fixed pseudo-bigram prior (rank 16, N(0, 1) entries).
    beta = 0 leaves two unrelated random models (acceptance ~0.05); a larger
    beta makes both distributions follow z, so the draft agrees with the
    target more often.  beta is a device scalar, read inside the engine's CUDA
    graphs, and switched between rounds."""

    def __init__(self, dev, r=16, seed=7):
        import torch
        g = torch.Generator(device=dev).manual_seed(seed)
        self.U = (torch.randn(VOCAB, r, generator=g, device=dev) / r ** 0.5).to(torch.bfloat16)
        self.W = torch.randn(r, VOCAB, generator=g, device=dev).to(torch.bfloat16)
        self.beta = torch.zeros(1, dtype=torch.bfloat16, device=dev)

    def head(self, lm_head):
        def f(hidden, ids):
            return lm_head(hidden) + self.beta * (self.U[ids] @ self.W)
        return f


class _AlphaSchedule:
    """Controller proxy for config 5: delegates k to the wrapped controller and
    switches the shared-prior strength every `period` emitted tokens per row
    (high agreement first), keeping per-phase acceptance counts."""

    def __init__(self, ctrl, prior, betas, period=64):
        self.ctrl, self.prior, self.betas, self.period = ctrl, prior, betas, period
        self.tokens = 0.0
        self.phase = 0
        self.acc = [0, 0]
        self.prop = [0, 0]
        self.offered = [0, 0]
        self.k_hist = {}
        prior.beta.fill_(betas[0])

    def propose_k(self):
        k = self.ctrl.propose_k()
        self.k_hist[k] = self.k_hist.get(k, 0) + 1
        return k

    def should_stop_drafting(self, i, conf):
        return self.ctrl.should_stop_drafting(i, conf)

    def update(self, k, n_accepted, dt, **kw):
        self.ctrl.update(k, n_accepted, dt, **kw)
        self.acc[self.phase] += sum(n_accepted)
        self.prop[self.phase] += k * len(n_accepted)
        self.offered[self.phase] += sum(min(k, a + 1) for a in n_accepted)
        self.tokens += (sum(n_accepted) + len(n_accepted)) / len(n_accepted)
        phase = int(self.tokens // self.period) % 2
        if phase != self.phase:
            self.phase = phase
            self.prior.beta.fill_(self.betas[phase])


def adaptive_bench(a):
    """--mode adaptive: config 5, the adaptive-k serving sweep, rows sharded by
    GPU (weak scaling: every rank runs its own --rows rows; no collective on
    the data path, one all-reduce of the results after the timed region).

    Per rank: the config-4 model shapes (random init), --rows rows with prompt
    lengths uniform in [128, 4096] (random ids, rank-seeded), --new-tokens new
    tokens per row (default 512 here), T = 0.7 / top-p 0.9, the "ewma"
    controller choosing k in [1, 8] from its online alpha and cost ratio.  The
    draft-target agreement alternates every 64 tokens between a high and a
    low setting of the shared prior (_SharedPrior; --beta-hi / --beta-lo,
    calibrated for alpha near 0.9 and 0.45).  value = tokens emitted by all
    ranks / the slowest rank's generate time (CUDA events around generate,
    max over ranks).  256 rows per GPU do not fit the capacity-padded cache
    with 4096-token prompts (about 330 GB of K/V); the mode runs any --rows
    that fits.
    """
    import torch
    import torch.distributed as dist
    from specdec.controller import make_controller
    from specdec.engine import SamplingConfig, SpecDecodeEngine
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)
    target, draft = _qwen_pair(dev)
    prior = _SharedPrior(dev)
    target.specdec_head = prior.head(target.lm_head)
    draft.specdec_head = prior.head(draft.lm_head)
    rows, new, kmax, pmin, pmax = a.rows, a.new_tokens, 8, 128, 4096
    eng = SpecDecodeEngine(target, draft, _NoTok(), device=dev,
                           capacity=pmax + 2 * new + 2 * kmax + 8, fused_qkv=a.fused_qkv,
                           fused_norm_mlp=a.fused_norm_mlp, paged_kv=a.paged)
    g = torch.Generator().manual_seed(1000 + rank)
    plen = torch.randint(pmin, pmax + 1, (rows,), generator=g)
    ids = torch.randint(0, VOCAB, (rows, int(plen.max())), generator=g)
    sp = SamplingConfig(temperature=T_SAMPLE, top_p=TOP_P)
    betas = (a.beta_hi, a.beta_lo)
    warm = _AlphaSchedule(make_controller("ewma", k_max=kmax), prior, betas)
    eng.generate(ids[:, :256], plen.clamp(max=256), 24, sampling=sp, seed=0, controller=warm)
    ctrl = _AlphaSchedule(make_controller("ewma", k_max=kmax), prior, betas)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clk:
        e0.record()
        _, st = eng.generate(ids, plen, new, sampling=sp, seed=1 + rank, controller=ctrl)
        e1.record()
        torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    res = torch.tensor([ms, float(st.emitted), float(ctrl.acc[0]), float(ctrl.prop[0]),
                        float(ctrl.acc[1]), float(ctrl.prop[1]), float(ctrl.offered[0]),
                        float(ctrl.offered[1])], dtype=torch.float64, device=dev)
    if world > 1:
        mx = res[:1].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(res, op=dist.ReduceOp.SUM)
        res[0] = mx[0]
    ms, emitted = float(res[0]), float(res[1])
    # alpha as the reference's RunStats.alpha_conditional (accepted / offered
    # positions) and the acceptance rate (accepted / proposed), per phase
    alpha_hi = float(res[2] / max(res[6], 1.0))
    alpha_lo = float(res[4] / max(res[7], 1.0))
    rate_hi = float(res[2] / max(res[3], 1.0))
    rate_lo = float(res[4] / max(res[5], 1.0))
    d = st.to_dict()
    line = {
        "metric": "accepted tok/s (config 5: adaptive k, Qwen3-8B / Qwen3-0.6B shapes, "
                  "rows sharded by GPU)",
        "value": emitted / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": 1,
        "warmup": 1, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02), random prompt ids)",
        "config": {"workload": "config 5 adaptive-k serving sweep", "rows_per_gpu": rows,
                   "prompt": f"U[{pmin},{pmax}]", "new_tokens": new, "k_range": [1, kmax],
                   "controller": "ewma", "temperature": T_SAMPLE, "top_p": TOP_P,
                   "alpha_switch_tokens": 64, "beta_hi_lo": list(betas),
                   "fused_qkv": a.fused_qkv, "fused_norm_mlp": a.fused_norm_mlp,
                   "paged_kv": a.paged,
                   "parallelism": f"row-sharded x{world}, no collective on the data path"},
        "alpha_conditional": {"high_phase": alpha_hi, "low_phase": alpha_lo},
        "acceptance_rate": {"high_phase": rate_hi, "low_phase": rate_lo},
        "engine_rank0": {key: d[key] for key in ("rounds", "emitted", "acceptance_rate",
                                                 "mean_accepted_len", "draft_forwards",
                                                 "target_forwards")},
        "k_histogram_rank0": {str(kk): v for kk, v in sorted(ctrl.k_hist.items())},
        "clocks": clk.summary()}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def engine_bench(a):
    """--mode engine: config 4, the whole speculative round through the engine.

    Random-init bf16 models (N(0, 0.02), no checkpoints offline) with the
    Qwen3-8B target shape (36 layers, 4096 hidden, 32/8 heads x 128, FFN
    12288, V 151936, RMSNorm, rope theta 1e6) and the Qwen3-0.6B draft shape
    (28 layers, 1024 hidden, 16/8 heads x 128, FFN 3072); B=32 rows of 512
    random prompt ids, k=4, --new-tokens per row, T=0.7 top-p 0.9.  Every
    attention, KV append / rollback and sampling step runs on this package's
    kernels; the projections and MLPs are torch / cuBLAS.  value = accepted
    (emitted) tokens per second over the whole generate call, timed with CUDA
    events around it (one step = one generate call).
    """
    import torch
    from specdec.engine import SamplingConfig, SpecDecodeEngine
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    target, draft = _qwen_pair(dev)

    Bq, P, k = 32, 512, 4
    new = max(8, a.new_tokens)
    # rows that finish early keep one cache slot per round until the slowest row
    # ends (the reference's rollback leaves k - n_acc with n_acc = 0 for them),
    # so a row can reach P + 2 * new
    eng = SpecDecodeEngine(target, draft, _NoTok(), device=dev,
                           capacity=P + 2 * new + 2 * k + 8, time_phases=True,
                           fused_qkv=a.fused_qkv, fused_norm_mlp=a.fused_norm_mlp,
                           paged_kv=a.paged)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, VOCAB, (Bq, P), generator=g)
    plen = torch.full((Bq,), P, dtype=torch.long)
    sp = SamplingConfig(temperature=T_SAMPLE, top_p=TOP_P)
    eng.generate(ids, plen, 16, sampling=sp, seed=0, k_fixed=k)          # warm-up
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index or 0) as clk:
        if a.profile_range:
            torch.cuda.profiler.start()
        e0.record()
        _, st = eng.generate(ids, plen, new, sampling=sp, seed=1, k_fixed=k)
        e1.record()
        torch.cuda.synchronize(dev)
        if a.profile_range:
            torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1)
    d = st.to_dict()
    print(json.dumps({
        "metric": "accepted tok/s (config 4: Qwen3-8B / Qwen3-0.6B shapes, B=32, k=4)",
        "value": st.emitted / (ms / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": 1,
        "warmup": 1, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights N(0,0.02), random prompt ids)",
        "config": {"workload": "config 4 full speculative round", "rows": Bq, "prompt": P,
                   "new_tokens": new, "k": k, "temperature": T_SAMPLE, "top_p": TOP_P,
                   "target": "Qwen3-8B shape (random init)",
                   "draft": "Qwen3-0.6B shape (random init)", "fused_qkv": a.fused_qkv,
                   "fused_norm_mlp": a.fused_norm_mlp, "paged_kv": a.paged},
        "engine": {key: d[key] for key in ("rounds", "emitted", "acceptance_rate",
                                           "mean_accepted_len", "draft_forwards",
                                           "target_forwards", "t_draft", "t_target",
                                           "t_total")},
        "clocks": clk.summary()}))


class _SelfComm:
    """Collectives of a one-rank job (identity)."""
    nranks, rank = 1, 0

    def all_gather(self, t):
        return t

    def all_reduce_sum(self, t):
        return t

    def all_reduce_max(self, t):
        return t


def rejection_bench(a):
    """--mode rejection: vLLM's rejection-sampler step at config 2 (64 requests,
    4 draft tokens each, V=151936, bf16 target logits, fp32 draft probabilities,
    T=0.7, top-p 0.9), through ``vllm_draft_spec.rejection.B200RejectionSampler``
    (the fused kernel) and through vLLM 0.22's own ``RejectionSampler``, on the
    same inputs.  A step is one ``forward`` call, host work included (both
    make small host copies); time per step = wall clock over the timed steps
    with the device synchronised at both ends."""
    import time
    import torch
    from vllm.v1.sample.logits_processor import LogitsProcessors
    from vllm.v1.sample.metadata import SamplingMetadata
    from vllm.v1.sample.rejection_sampler import RejectionSampler
    from vllm.v1.sample.sampler import Sampler
    from vllm.v1.spec_decode.metadata import SpecDecodeMetadata
    from specdec import sampling as S
    from specdec import workloads as W
    from vllm_draft_spec.rejection import B200RejectionSampler
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    B, k, V, T, tp = 64, K_DRAFT, VOCAB, 0.7, 0.9
    tgt, drf = W.cfg2_logits(B, k, V, seed=0, device=dev)
    q = S.to_probs(drf, T, tp).reshape(B * k, V)
    xs, _ = S.draft_sample(drf.reshape(-1, V), torch.rand(B * k, device=dev), T, tp)
    logits = tgt.reshape(B * (k + 1), V)
    md = SpecDecodeMetadata.make_dummy(xs.view(B, k).tolist(), dev)
    blk = torch.arange(B, device=dev, dtype=torch.int32) * (k + 1)
    md.target_logits_indices = (blk[:, None] + torch.arange(k, device=dev, dtype=torch.int32)).reshape(-1)
    md.bonus_logits_indices = blk + k
    zeros = torch.zeros(B, device=dev)
    smd = SamplingMetadata(
        temperature=torch.full((B,), T, device=dev), all_greedy=False, all_random=True,
        top_p=torch.full((B,), tp, device=dev), top_k=None, generators={}, max_num_logprobs=None,
        no_penalties=True, prompt_token_ids=None, frequency_penalties=zeros,
        presence_penalties=zeros, repetition_penalties=torch.ones(B, device=dev),
        output_token_ids=[[] for _ in range(B)], allowed_token_ids_mask=None,
        bad_words_token_ids={}, logitsprocs=LogitsProcessors())
    ours = B200RejectionSampler(Sampler(), None, dev)
    stock = RejectionSampler(Sampler(), None, dev)
    steps = max(5, min(a.steps, 200))
    res = {}
    for name, rs in (("b200", ours), ("vllm", stock)):
        for _ in range(max(3, a.warmup)):
            out = rs.forward(md, q, logits, smd)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        for _ in range(steps):
            out = rs.forward(md, q, logits, smd)
        torch.cuda.synchronize(dev)
        res[name] = (time.perf_counter() - t0) / steps * 1e3
        res[name + "_tokens"] = float((out.sampled_token_ids >= 0).sum()) / B
        if name == "b200":
            assert ours.calls["vllm"] == 0, "the batch must take the fused path"
    print(json.dumps({
        "metric": "vLLM rejection-sampler steps/s (config 2: 64 requests x 4 drafts, V=151936, "
                  "T=0.7 top-p 0.9)", "value": 1e3 / res["b200"], "unit": "steps/s",
        "n_gpus": 1, "steps": steps, "warmup": a.warmup, "ms_per_step": res["b200"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded config-2 logits, see specdec/workloads.py)",
        "config": {"workload": "vLLM RejectionSampler.forward, fused kernel vs vLLM 0.22's own",
                   "vllm_stock_ms_per_step": res["vllm"],
                   "speedup_vs_vllm": res["vllm"] / res["b200"],
                   "tokens_per_request_last_step": {"b200": res["b200_tokens"],
                                                     "vllm": res["vllm_tokens"]},
                   "timing": "wall clock per forward() call, host work included"},
        "gpu_launches": 2 * steps}))


def extra_measurements():
    """The other verify-round rows, each from its own bench mode in a child
    process on this GPU (its own clock samples, timing and checks), so that the
    default run's record carries them: the greedy round (config 2), the verify
    attention (config 3, checked against fp32 before timing) and the vLLM
    rejection-sampler step against vLLM's own.  A mode that fails is recorded
    with its error; the main line is unaffected."""
    import subprocess
    runs = {"greedy": ["--mode", "greedy", "--steps", "1000", "--warmup", "10", "--no-cpu-baseline"],
            "attn": ["--mode", "attn", "--steps", "100", "--warmup", "5"],
            "rejection": ["--mode", "rejection", "--steps", "50", "--warmup", "5"]}
    keep = ("metric", "value", "unit", "ms_per_step", "roofline", "clocks", "config", "e2e")
    out = {}
    for name, argv in runs.items():
        try:
            r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *argv], capture_output=True,
                               text=True, timeout=600, cwd=str(ROOT))
            last = [x for x in r.stdout.splitlines() if x.startswith("{")]
            if r.returncode != 0 or not last:
                out[name] = {"error": f"exit {r.returncode}: {r.stderr.strip()[-300:]}"}
                continue
            d = json.loads(last[-1])
            out[name] = {k: d[k] for k in keep if k in d}
        except Exception as e:                          # noqa: BLE001 - recorded, not raised
            out[name] = {"error": repr(e)[-300:]}
    return out


def main():
    a = parse()
    if a.impl == "reference":
        return reference_arm(a)
    if a.mode == "attn":
        return attn_bench(a)
    if a.mode.startswith("vshard"):
        return vshard_bench(a)
    if a.mode == "engine":
        if a.new_tokens is None:
            a.new_tokens = 256
        return engine_bench(a)
    if a.mode == "adaptive":
        if a.new_tokens is None:
            a.new_tokens = 512
        return adaptive_bench(a)
    if a.mode == "rejection":
        return rejection_bench(a)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cpu_rate = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu_rate = cpu_baseline(a.mode)       # before any CUDA work
    import torch
    import torch.distributed as dist
    from specdec import sampling as S
    from specdec import workloads as W
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    greedy = a.mode == "greedy"
    T, tp = (0.0, 1.0) if greedy else (a.temperature, a.top_p)

    bufs = []
    for i in range(NBUF):
        tgt, drf = W.cfg2_logits(B, K_DRAFT, VOCAB, seed=100 * rank + i, device=dev)
        if a.flat:
            g = torch.Generator(device=dev).manual_seed(100 * rank + i)
            tgt = torch.randn(tgt.shape, generator=g, device=dev).to(torch.bfloat16)
            drf = (tgt[:, :K_DRAFT].float() + 0.3 * torch.randn(drf.shape, generator=g,
                                                                 device=dev)).to(torch.bfloat16)
        xs, _ = S.draft_sample(drf.reshape(-1, VOCAB), torch.rand(B * K_DRAFT, device=dev), T, tp)
        ua, ur = W.uniforms(B, K_DRAFT, seed=100 * rank + i, device=dev)
        bufs.append((tgt, drf, xs.view(B, K_DRAFT), ua, ur))

    def call(i):
        tgt, drf, xs, ua, ur = bufs[i % NBUF]
        return S.verify_sample(tgt, drf, xs, ua, ur, T, tp)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for i in range(max(3, a.warmup)):
            call(i)
    torch.cuda.synchronize(dev)
    graphs = {}

    def graph_of(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for i in range(n):
                    call(i)
            graphs[n] = g
        return graphs[n]

    plan = [GRAPH_CALLS] * (a.steps // GRAPH_CALLS)
    if a.steps % GRAPH_CALLS:
        plan.append(a.steps % GRAPH_CALLS)
    with torch.cuda.stream(s):
        for n in set(plan):
            graph_of(n).replay()      # warm the graphs too
    torch.cuda.synchronize(dev)

    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    # graphs replay on the current stream: keep replays and events on `s`
    with ClockSampler(dev.index if dev.index is not None else 0) as clk, torch.cuda.stream(s):
        ev0.record(s)
        for n in plan:
            graph_of(n).replay()
        ev1.record(s)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        dist.barrier()
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / a.steps
    value = world * B * a.steps / (ms / 1e3)
    bytes_call = W.bytes_per_verify(B, K_DRAFT, VOCAB, greedy=greedy)

    # roofline time: one verify call's share of the timed region (graph replays
    # of back-to-back calls, events on the launching stream).  A call is the
    # stats kernel and its row pass, or for greedy the argmax streaming kernel
    # and its small per-row pass; the
    # whole call is charged to the dominant kernel, so `achieved` is a lower
    # bound for it.  The same call timed alone between its own event pair
    # (launch gaps included) is reported beside it.
    n_k = max(20, min(a.steps, 200))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(n_k)]
    with torch.cuda.stream(s):
        # keep the GPU busy while the host enqueues the calls, so that each
        # event pair times GPU work only (a call can be shorter than its launch
        # path on the host); ~100 us of spin per call covers the enqueue
        torch.cuda._sleep(int(2e5 * n_k))
        for i, (k0, k1) in enumerate(evs):
            k0.record(s)
            call(i)
            k1.record(s)
        torch.cuda.synchronize(dev)
    call_ms_isolated = statistics.mean(k0.elapsed_time(k1) for k0, k1 in evs)
    k_ms = ms_step
    gbs = bytes_call / (k_ms * 1e-3) / 1e9
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = peaks.get("hbm_gbs")
    peak_src = "measured" if peak else "fallback"
    peak = peak or 6650.0

    # end to end through the public API from pinned host buffers
    host = []
    for i in range(NBUF):
        tgt, drf, xs, ua, ur = bufs[i]
        host.append(tuple(t.cpu().pin_memory() for t in (tgt, drf, xs, ua, ur)))
    dev_in = [tuple(torch.empty_like(t, device=dev) for t in host[0]) for _ in range(NBUF)]
    res = [(torch.empty(B, dtype=torch.long).pin_memory(),
            torch.empty(B, dtype=torch.long).pin_memory()) for _ in range(NBUF)]
    n_e2e = max(3, min(a.steps, 100))

    def e2e_step(i):
        d = dev_in[i % NBUF]
        for dst, src in zip(d, host[i % NBUF]):
            dst.copy_(src, non_blocking=True)
        n, y = S.verify_sample(d[0], None if greedy else d[1], d[2], d[3], d[4], T, tp)
        res[i % NBUF][0].copy_(n, non_blocking=True)
        res[i % NBUF][1].copy_(y, non_blocking=True)

    with torch.cuda.stream(s):
        for i in range(3):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for i in range(n_e2e):
            e2e_step(i)
        e1.record(s)
        torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    h2d = sum(t.numel() * t.element_size() for t in host[0][:1] + host[0][2:])
    if not greedy:
        h2d += host[0][1].numel() * host[0][1].element_size()
    traffic = None
    prof = ROOT / "profiles" / ("verify_greedy_traffic.json" if greedy else "verify_sample_traffic.json")
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("bytes_per_call")
    # our kernels per verify call: the stats kernel and the row pass, or for
    # greedy the argmax streaming kernel and its per-row pass
    launches_per_step = 2
    line = {
        "metric": metric_name(a.mode, T, tp, a.flat), "value": value, "unit": "rows/s",
        "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded config-2 logits, see specdec/workloads.py)",
        "config": workload_config(a.mode, world, T, tp, a.flat),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                     "frac": gbs / peak, "traffic": traffic,
                     "peak_source": peak_src,
                     "kernel": "argmax16_kernel" if greedy else "hist_stats_kernel",
                     "kernel_ms": k_ms, "call_ms_isolated": call_ms_isolated,
                     "scope": f"algorithmic bytes {bytes_call} per call (every logits element "
                              "read once) / one call's share of the event-timed region "
                              "(graph replays of back-to-back calls, all of the call's "
                              "kernels and gaps charged to the dominant kernel)"},
        "e2e": {"value": world * B * n_e2e / (e2e_ms / 1e3), "unit": "rows/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 2 * B * 8, "steps": n_e2e},
        "gpu_launches": launches_per_step * a.steps,
        "clocks": clk.summary(),
    }
    if cpu_rate is not None:
        rate, steps, kind, cores, rows = cpu_rate
        line["cpu_baseline"] = {"value": rate, "unit": "rows/s", "cores": cores, "kind": kind,
                                "sample": f"{steps} batches of {rows} config-2 rows through the "
                                          "reference's specdec/sampling.py (baseline/_ref, "
                                          f"torch CPU, {cores} threads)" if kind == "reference"
                                          else f"{steps} batches of {rows} rows through "
                                          "oracle/sampling_oracle.py"}
    if (rank == 0 and world == 1 and a.mode == "sample" and not a.flat and not a.no_extras
            and T == T_SAMPLE and tp == TOP_P):
        line["also"] = extra_measurements()
    if rank == 0:
        print(json.dumps(line))
    for g in graphs.values():
        del g
    graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
