"""Vocabulary-sharded verify round on the CPU (no GPU needed).

* The round's phase arithmetic, restated in numpy (``oracle/shard_oracle.py``)
  and driven by the product's own orchestration (``specdec.sharded``), gives
  the unsharded oracle's n_acc / y for 1-4 shards (rows inside the contract's
  1e-6 exemption margins excepted).
* Two real gloo ranks run ``verify_sharded`` (the NCCL path's host logic)
  and agree with the oracle.
* The C ABI rejects bad arguments on the host.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch

from oracle import sampling_oracle as O
from oracle.shard_oracle import NumpyShardBackend
from specdec import sharded as SH

EPS = 1e-6


def _inputs(B, k, V, T, tp, seed, sig=3.0, draft_sigma=1.0):
    g = torch.Generator().manual_seed(seed)
    tgt = (torch.randn(B, k + 1, V, generator=g) * sig).to(torch.bfloat16)
    drf = (tgt[:, :k].float() + torch.randn(B, k, V, generator=g) * draft_sigma).to(torch.bfloat16)
    # draft tokens drawn from the draft's own distribution (inverse CDF)
    Q = O.to_probs(drf.float().numpy(), T, tp) if T > 0 else O.to_probs(drf.float().numpy(), 0.0)
    u = torch.rand(B, k, generator=g).numpy()
    xs = torch.tensor([[O._icdf(Q[b, i], Q[b, i].astype(np.float64).sum(), u[b, i])[0]
                        for i in range(k)] for b in range(B)], dtype=torch.long)
    ua = torch.rand(B, k, generator=g)
    ur = torch.rand(B, generator=g)
    return tgt, drf, xs, ua, ur


def _oracle(tgt, drf, xs, ua, ur, T, tp):
    n, y, d = O.verify(tgt.float().numpy(), drf.float().numpy(), xs.numpy(), ua.numpy(),
                       ur.numpy(), T, tp, 0, return_details=True)
    ok = (d["acc_margin"] > EPS) & (d["cdf_margin"] > EPS) & (d["topp_margin"] > EPS)
    return n, y, ok


@pytest.mark.parametrize("T,tp", [(0.7, 0.9), (1.0, 1.0), (0.7, 0.5), (0.0, 1.0)])
@pytest.mark.parametrize("nranks", [1, 2, 3, 4])
def test_protocol_matches_unsharded_oracle(T, tp, nranks):
    B, k, V = 6, 4, 2999                              # uneven slices when nranks = 2, 4
    for seed in range(2):
        tgt, drf, xs, ua, ur = _inputs(B, k, V, T, tp, seed)
        n_o, y_o, ok = _oracle(tgt, drf, xs, ua, ur, T, tp)
        outs, status = SH.verify_sharded_local(tgt, drf, xs, ua, ur, SH.even_split(V, nranks),
                                               T, tp, backend_factory=NumpyShardBackend)
        assert status == [0] * nranks
        for n, y in outs:
            bad = np.nonzero(ok & ((n.numpy() != n_o) | (y.numpy() != y_o)))[0]
            assert bad.size == 0, (T, tp, nranks, seed, bad)


def test_alive_mask_and_all_accepted_rows():
    B, k, V = 5, 3, 1500
    tgt, drf, xs, ua, ur = _inputs(B, k, V, 0.8, 0.95, seed=7)
    xs[0] = tgt[0, :k].float().argmax(-1)              # likely accepted
    ua[1] = 0.0                                        # every test passes: bonus draw
    alive = torch.tensor([1, 1, 0, 1, 1], dtype=torch.bool)
    n_o, y_o, d = O.verify(tgt.float().numpy(), drf.float().numpy(), xs.numpy(), ua.numpy(),
                           ur.numpy(), 0.8, 0.95, 0, alive=alive.numpy(), return_details=True)
    assert n_o[1] == k and n_o[2] == 0
    outs, status = SH.verify_sharded_local(tgt, drf, xs, ua, ur, SH.even_split(V, 3), 0.8, 0.95,
                                           alive=alive, backend_factory=NumpyShardBackend)
    for n, y in outs:
        assert np.array_equal(n.numpy(), n_o) and np.array_equal(y.numpy(), y_o)


def test_flat_distribution_raises_the_fallback_status_on_every_rank():
    # T = 2 on N(0, 3^2) logits: the top-p boundary bins hold more elements than
    # a shard may send; every rank must see the same status
    B, k, V = 4, 2, 3000
    tgt, drf, xs, ua, ur = _inputs(B, k, V, 2.0, 0.95, seed=0)
    _, status = SH.verify_sharded_local(tgt, drf, xs, ua, ur, SH.even_split(V, 1), 2.0, 0.95,
                                        backend_factory=NumpyShardBackend)
    assert status == [2]
    _, status = SH.verify_sharded_local(tgt, drf, xs, ua, ur, [0, 1500, 3000], 4.0, 0.999,
                                        backend_factory=NumpyShardBackend)
    assert len(set(status)) == 1


def test_top_k_is_rejected():
    tgt, drf, xs, ua, ur = _inputs(2, 2, 64, 0.7, 0.9, seed=0)
    with pytest.raises(RuntimeError):
        SH.verify_sharded_local(tgt, drf, xs, ua, ur, [0, 32, 64], 0.7, 0.9, top_k=5,
                                backend_factory=NumpyShardBackend)


# ---------------------------------------------------------------------------
# two gloo ranks through the product orchestration
# ---------------------------------------------------------------------------
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, T, tp, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, k, V = 6, 4, 2001
        tgt, drf, xs, ua, ur = _inputs(B, k, V, T, tp, seed=3)
        vs = SH.even_split(V, world)
        sl = slice(vs[rank], vs[rank + 1])
        n, y = SH.verify_sharded(tgt[..., sl], drf[..., sl], xs, ua, ur, vs,
                                 SH.ProcessGroupCollectives(), temperature=T, top_p=tp,
                                 backend=NumpyShardBackend())
        torch.save((n, y), os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("T,tp", [(0.7, 0.9), (0.0, 1.0)])
def test_gloo_two_ranks(tmp_path, T, tp):
    import torch.multiprocessing as mp
    port = _free_port()
    mp.start_processes(_rank_main, args=(2, port, T, tp, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    B, k, V = 6, 4, 2001
    tgt, drf, xs, ua, ur = _inputs(B, k, V, T, tp, seed=3)
    n_o, y_o, ok = _oracle(tgt, drf, xs, ua, ur, T, tp)
    res = [torch.load(tmp_path / f"r{r}.pt") for r in range(2)]
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])
    n, y = res[0]
    bad = np.nonzero(ok & ((n.numpy() != n_o) | (y.numpy() != y_o)))[0]
    assert bad.size == 0, bad


# ---------------------------------------------------------------------------
# the C ABI validates on the host
# ---------------------------------------------------------------------------
def test_shard_abi_rejects_bad_arguments():
    import importlib.util
    import pathlib
    root = pathlib.Path(__file__).resolve().parent.parent
    spec = importlib.util.spec_from_file_location("sd_build", root / "adaptive-specdec_b200" /
                                                  "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build()
    from specdec import _lib as L
    lib = L.lib()
    assert lib.sd_shard_workspace_bytes(64, 4, 8) > 0
    assert lib.sd_shard_send_bytes(64, 4, 8, 0, 3) == 64 * 9 * (16 + 8 * L.SHARD_BOUNDARY_CAP)
    assert lib.sd_shard_send_bytes(64, 4, 8, 1, 1) == 64 * 5 * 8
    a = L.ShardArgs()
    assert lib.sd_shard_phase(ctypes.byref(a), 1, None, None, None) == -22     # B = 0
    a.B, a.k, a.V, a.rank, a.nranks, a.dtype = 4, 2, 100, 0, 2, 2
    a.v_start[0], a.v_start[1], a.v_start[2] = 0, 50, 100
    a.temperature, a.top_p, a.top_k = 0.7, 0.9, 3
    assert lib.sd_shard_phase(ctypes.byref(a), 1, None, None, None) == -95     # top_k
    a.top_k = 0
    assert lib.sd_shard_phase(ctypes.byref(a), 1, None, None, None) == -22     # NULL inputs
    a.nranks = 17
    assert lib.sd_shard_phase(ctypes.byref(a), 1, None, None, None) == -22     # too many ranks
