"""Vocabulary-sharded verify round (the SPMD form of ``verify_sample``).

With a vocab-parallel LM head every rank holds the columns
``[v_start[r], v_start[r+1])`` of every target / draft logits vector.  This
module runs the verify round of ``specdec/engine.py:282-303`` on such slices
and leaves every rank with the same ``(n_acc, y)`` that ``verify_sample``
returns on the full vectors.  The local work is the C-ABI phase kernels
(``sd_shard_phase``); between phases one collective crosses the ranks:

    temperature > 0:  P1, all_gather, P2, all_reduce(sum), P3, all_gather,
                      P4, all_gather, P5, all_reduce(max), P6
    temperature <= 0: P1, all_reduce(max), P6

What travels is small (per vector: two floats, a 129-entry float64
histogram, the top-p boundary elements; per row: two float64 and a token
id), never the logits.  When the top-p boundary cannot be decided from those
messages (a very flat distribution), every rank sees the same status bit and
the round is re-run on all-gathered full vectors with the single-device
kernel.
"""
import torch

from . import _lib as L
from . import sampling as S

__all__ = ["ProcessGroupCollectives", "CudaShardBackend", "run_round", "run_round_local",
           "verify_sharded", "verify_sharded_local", "even_split"]


def even_split(V, nranks, align=8):
    """v_start for nranks near-equal contiguous slices of a vocabulary of V.

    Every boundary but the last is a multiple of `align` columns (8 bf16 /
    fp16 columns = 16 bytes), so every slice except possibly the last has a
    width that keeps its rows 16-byte aligned and the phase kernels on their
    16-byte loads for any rank count; a vocabulary narrower than `align`
    columns per rank is split column by column."""
    units, tail = divmod(V, align)
    if units < nranks:
        base, extra = divmod(V, nranks)
        out = [0]
        for r in range(nranks):
            out.append(out[-1] + base + (1 if r < extra else 0))
        return out
    base, extra = divmod(units, nranks)
    out = [0]
    for r in range(nranks):
        out.append(out[-1] + (base + (1 if r < extra else 0)) * align)
    out[-1] += tail
    return out


class ProcessGroupCollectives:
    """The three collectives of a round over a torch.distributed group
    (NCCL for CUDA tensors; gloo works for CPU tensors)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.nranks = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t):
        """Concatenate every rank's byte buffer in rank order."""
        out = torch.empty(self.nranks * t.numel(), dtype=t.dtype, device=t.device)
        if t.is_cuda:
            self.dist.all_gather_into_tensor(out, t, group=self.group)
        else:
            self.dist.all_gather(list(out.chunk(self.nranks)), t, group=self.group)
        return out

    def all_reduce_sum(self, t):
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM, group=self.group)
        return t

    def all_reduce_max(self, t):
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)
        return t


class CudaShardBackend:
    """The local phases on this rank's GPU (``sd_shard_phase``).  Send buffers
    and the workspace are kept and reused across rounds."""

    def __init__(self, device):
        self.device = torch.device(device)
        self._bufs = {}
        self._ws = None
        self.args = None

    def _buf(self, key, nbytes):
        b = self._bufs.get(key)
        if b is None or b.numel() < nbytes:
            b = torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=self.device)
            self._bufs[key] = b
        return b[:nbytes]

    def bind(self, tgt, drf, xs, u_acc, u_res, alive, v_start, rank, V, temperature, top_p,
             top_k):
        """Set the round's inputs (all on this backend's device)."""
        L.require_cuda(tgt, drf, xs, u_acc, u_res, alive)
        lib = L.lib()
        B, k1, _ = tgt.shape
        k = k1 - 1
        nranks = len(v_start) - 1
        a = L.ShardArgs()
        self._keep = (tgt, drf, xs, u_acc, u_res, alive)
        a.tgt, a.tgt_bs, a.tgt_ps = tgt.data_ptr(), tgt.stride(0), tgt.stride(1)
        if drf is not None:
            a.drf, a.drf_bs, a.drf_ps = drf.data_ptr(), drf.stride(0), drf.stride(1)
        a.dtype = L.dtype_code(tgt.dtype)
        a.xs, a.xs_bs = xs.data_ptr(), xs.stride(0)
        if u_acc is not None:
            a.u_acc, a.u_bs = u_acc.data_ptr(), u_acc.stride(0)
        if u_res is not None:
            a.u_res = u_res.data_ptr()
        if alive is not None:
            a.alive = alive.data_ptr()
        a.B, a.k, a.V, a.rank, a.nranks = B, k, V, rank, nranks
        for i, v in enumerate(v_start):
            a.v_start[i] = v
        a.temperature, a.top_p, a.top_k = float(temperature), float(top_p), int(top_k)
        self.n_acc = torch.empty(B, dtype=torch.long, device=self.device)
        self.y = torch.empty(B, dtype=torch.long, device=self.device)
        a.n_acc, a.y = self.n_acc.data_ptr(), self.y.data_ptr()
        nws = lib.sd_shard_workspace_bytes(B, k, nranks)
        if self._ws is None or self._ws.numel() < nws:
            self._ws = torch.empty(nws, dtype=torch.uint8, device=self.device)
        a.workspace, a.workspace_bytes = self._ws.data_ptr(), self._ws.numel()
        self.args = a
        self.greedy = not temperature > 0
        self.B, self.k, self.nranks = B, k, nranks

    def send_bytes(self, phase):
        return L.lib().sd_shard_send_bytes(self.B, self.k, self.nranks, int(self.greedy), phase)

    def phase(self, phase, recv):
        """Run local phase `phase` on `recv`; returns the send buffer (uint8)."""
        nb = self.send_bytes(phase) if phase < 6 else 0
        send = self._buf(phase, nb) if nb else None
        with torch.cuda.device(self.device):
            L.check(L.lib().sd_shard_phase(
                ctypes_byref(self.args), phase, L.ptr(recv), L.ptr(send),
                L.stream_ptr(self.device)), f"sd_shard_phase({phase})")
        return send

    def status(self):
        """The round's status word (synchronises with the stream)."""
        return int(self._ws[:4].view(torch.int32).item())

    def outputs(self):
        return self.n_acc, self.y


def ctypes_byref(x):
    import ctypes
    return ctypes.byref(x)


def run_round(backend, comm, greedy):
    """The fixed phase / collective sequence of one round on this rank."""
    if greedy:
        s1 = backend.phase(1, None)
        comm.all_reduce_max(s1.view(torch.int64))
        backend.phase(6, s1)
        return
    s1 = backend.phase(1, None)
    r1 = comm.all_gather(s1)
    s2 = backend.phase(2, r1)
    comm.all_reduce_sum(s2.view(torch.float64))
    s3 = backend.phase(3, s2)
    r3 = comm.all_gather(s3)
    s4 = backend.phase(4, r3)
    r4 = comm.all_gather(s4)
    s5 = backend.phase(5, r4)
    comm.all_reduce_max(s5.view(torch.int64))
    backend.phase(6, s5)


def run_round_local(backends, greedy):
    """The same round with every shard's backend in this process (collectives
    emulated in rank order): all shards on one device, or CPU checking."""
    def gather(bufs):
        return torch.cat(list(bufs))

    def reduce(bufs, dtype, op):
        views = [b.view(dtype) for b in bufs]
        acc = views[0].clone()
        for v in views[1:]:
            acc = op(acc, v.to(acc.device))
        for v in views:
            v.copy_(acc.to(v.device))
        return bufs

    if greedy:
        s1 = reduce([b.phase(1, None) for b in backends], torch.int64, torch.maximum)
        for b, s in zip(backends, s1):
            b.phase(6, s)
        return
    r1 = gather([b.phase(1, None) for b in backends])
    s2 = reduce([b.phase(2, r1) for b in backends], torch.float64, torch.add)
    r3 = gather([b.phase(3, s) for b, s in zip(backends, s2)])
    r4 = gather([b.phase(4, r3) for b in backends])
    s5 = reduce([b.phase(5, r4) for b in backends], torch.int64, torch.maximum)
    for b, s in zip(backends, s5):
        b.phase(6, s)


def verify_sharded_local(tgt, drf, xs, u_acc, u_res, v_start, temperature=1.0, top_p=1.0,
                         top_k=0, alive=None, backend_factory=None):
    """Split full [B, k+1, V] / [B, k, V] logits at v_start and run the sharded
    round with all shards in this process.  Returns every shard's (n_acc, y)
    and the status words (for tests and single-device checks)."""
    nranks = len(v_start) - 1
    if temperature > 0 and top_k:
        raise L.SpecdecError("the vocabulary-sharded round supports top_k = 0 only")
    greedy = not temperature > 0
    backends = []
    for r in range(nranks):
        be = backend_factory() if backend_factory else CudaShardBackend(tgt.device)
        sl = slice(v_start[r], v_start[r + 1])
        t = tgt[..., sl].contiguous()
        d = None if (drf is None or greedy) else drf[..., sl].contiguous()
        al = None if alive is None else alive.to(torch.uint8).contiguous()
        be.bind(t, d, xs.long().contiguous(),
                None if u_acc is None else u_acc.float().contiguous(),
                None if u_res is None else u_res.float().contiguous(), al, v_start, r,
                v_start[-1], temperature, top_p, top_k)
        backends.append(be)
    run_round_local(backends, greedy)
    return [b.outputs() for b in backends], [0 if greedy else b.status() for b in backends]


def _gather_full(t, v_start, comm):
    """[..., Vr] slices of every rank -> [..., V] (fallback path)."""
    vmax = max(b - a for a, b in zip(v_start[:-1], v_start[1:]))
    pad = torch.zeros(*t.shape[:-1], vmax, dtype=t.dtype, device=t.device)
    pad[..., :t.shape[-1]] = t
    flat = comm.all_gather(pad.contiguous().view(-1).view(torch.uint8))
    parts = flat.view(t.dtype).view(len(v_start) - 1, *t.shape[:-1], vmax)
    return torch.cat([parts[r, ..., :v_start[r + 1] - v_start[r]]
                      for r in range(len(v_start) - 1)], dim=-1)


def verify_sharded(tgt, drf, xs, u_acc, u_res, v_start, comm, temperature=1.0, top_p=1.0,
                   top_k=0, alive=None, backend=None):
    """One verify round on vocabulary slices.

    tgt [B, k+1, Vr] and drf [B, k, Vr] are this rank's slices (columns
    v_start[rank]:v_start[rank+1] of the full logits); xs [B, k] holds global
    token ids.  Returns (n_acc, y) int64 [B], identical on every rank and equal
    to ``verify_sample`` on the full vectors.
    """
    rank, nranks = comm.rank, comm.nranks
    if len(v_start) != nranks + 1 or v_start[0] != 0:
        raise L.SpecdecError("v_start must hold nranks + 1 offsets starting at 0")
    if nranks > L.SHARD_MAX_RANKS:
        raise L.SpecdecError(f"at most {L.SHARD_MAX_RANKS} vocabulary shards")
    if temperature > 0 and top_k:
        raise L.SpecdecError("the vocabulary-sharded round supports top_k = 0 only")
    V = v_start[-1]
    if tgt.shape[-1] != v_start[rank + 1] - v_start[rank]:
        raise L.SpecdecError("slice width does not match v_start")
    if backend is None:
        backend = CudaShardBackend(tgt.device)
    if tgt.stride(-1) != 1:
        tgt = tgt.contiguous()
    if drf is not None and drf.stride(-1) != 1:
        drf = drf.contiguous()
    xs = xs.long().contiguous()
    u_acc = None if u_acc is None else u_acc.float().contiguous()
    u_res = None if u_res is None else u_res.float().contiguous()
    al = None if alive is None else alive.to(torch.uint8).contiguous()
    backend.bind(tgt, drf, xs, u_acc, u_res, al, v_start, rank, V, temperature, top_p, top_k)
    greedy = not temperature > 0
    run_round(backend, comm, greedy)
    if not greedy and backend.status() & L.SHARD_STATUS_FALLBACK:
        full_t = _gather_full(tgt, v_start, comm)
        full_d = _gather_full(drf, v_start, comm)
        return S.verify_sample(full_t, full_d, xs, u_acc, u_res, temperature=temperature,
                               top_p=top_p, top_k=top_k, alive=alive)
    return backend.outputs()
