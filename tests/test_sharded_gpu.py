"""Vocabulary-sharded verify round on the GPU.

All shards on one device (``verify_sharded_local`` with the CUDA phase
kernels) against the fused single-device kernel and the oracle, at config-2
shapes; and, when the box has two GPUs, two NCCL ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import sampling_oracle as O
from oracle.shard_oracle import NumpyShardBackend
from specdec import sampling as S
from specdec import sharded as SH
from specdec import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
EPS = 1e-6


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(scope="module")
def cfg2_16():
    B, k = 16, 4
    tgt, drf = W.cfg2_logits(B=B, k=k, seed=1)
    ua, ur = W.uniforms(B, k, seed=1)
    xs, _ = S.draft_sample(drf.reshape(-1, drf.shape[-1]), torch.rand(
        B * k, generator=torch.Generator(device=DEV).manual_seed(5), device=DEV), 0.7, 0.9)
    return tgt, drf, xs.reshape(B, k), ua, ur


def _oracle_ok(tgt, drf, xs, ua, ur, T, tp):
    n, y, d = O.verify(_np(tgt), _np(drf), xs.cpu().numpy(), _np(ua), _np(ur), T, tp, 0,
                       return_details=True)
    ok = (d["acc_margin"] > EPS) & (d["cdf_margin"] > EPS) & (d["topp_margin"] > EPS)
    return n, y, ok


@pytest.mark.parametrize("nranks", [1, 2, 4, 8])
def test_cfg2_shapes_match_fused_kernel_and_oracle(cfg2_16, nranks):
    tgt, drf, xs, ua, ur = cfg2_16
    V = tgt.shape[-1]
    n_f, y_f = S.verify_sample(tgt, drf, xs, ua, ur, 0.7, 0.9, 0)
    n_o, y_o, ok = _oracle_ok(tgt, drf, xs, ua, ur, 0.7, 0.9)
    assert ok.mean() >= 0.9
    outs, status = SH.verify_sharded_local(tgt, drf, xs, ua, ur, SH.even_split(V, nranks),
                                           0.7, 0.9)
    assert status == [0] * nranks
    for n, y in outs:
        n, y = n.cpu().numpy(), y.cpu().numpy()
        bad = np.nonzero(ok & ((n != n_o) | (y != y_o)))[0]
        assert bad.size == 0, (nranks, bad)
        bad = np.nonzero(ok & ((n != n_f.cpu().numpy()) | (y != y_f.cpu().numpy())))[0]
        assert bad.size == 0, (nranks, bad)


@pytest.mark.parametrize("T,tp", [(1.0, 1.0), (0.7, 0.5), (0.0, 1.0)])
def test_other_knobs(cfg2_16, T, tp):
    tgt, drf, xs, ua, ur = cfg2_16
    if T == 0.0:
        xs = torch.where(torch.rand(xs.shape, device=DEV) < 0.7, tgt[:, :-1].float().argmax(-1), xs)
    n_o, y_o, ok = _oracle_ok(tgt, drf, xs, ua, ur, T, tp)
    outs, status = SH.verify_sharded_local(tgt, drf, xs, ua, ur, SH.even_split(tgt.shape[-1], 4),
                                           T, tp)
    assert status == [0] * 4
    for n, y in outs:
        bad = np.nonzero(ok & ((n.cpu().numpy() != n_o) | (y.cpu().numpy() != y_o)))[0]
        assert bad.size == 0, (T, tp, bad)


def test_cuda_phases_agree_with_numpy_restatement():
    g = torch.Generator(device=DEV).manual_seed(11)
    B, k, V = 6, 3, 5003
    tgt = (torch.randn(B, k + 1, V, generator=g, device=DEV) * 3).to(torch.bfloat16)
    drf = (tgt[:, :k].float() + torch.randn(B, k, V, generator=g, device=DEV)).to(torch.bfloat16)
    xs = torch.randint(0, V, (B, k), generator=g, device=DEV)
    xs[:, 0] = tgt[:, 0].float().argmax(-1)
    ua = torch.rand(B, k, generator=g, device=DEV)
    ur = torch.rand(B, generator=g, device=DEV)
    vs = [0, 1000, 1001, 4000, V]                      # one single-column shard
    outs_c, st_c = SH.verify_sharded_local(tgt, drf, xs, ua, ur, vs, 0.9, 0.8)
    outs_n, st_n = SH.verify_sharded_local(tgt.cpu(), drf.cpu(), xs.cpu(), ua.cpu(), ur.cpu(), vs,
                                           0.9, 0.8, backend_factory=NumpyShardBackend)
    n_o, y_o, ok = _oracle_ok(tgt, drf, xs, ua, ur, 0.9, 0.8)
    assert st_c == st_n == [0] * 4
    for (n, y), (nn, yn) in zip(outs_c, outs_n):
        sel = ok
        assert np.array_equal(n.cpu().numpy()[sel], nn.numpy()[sel])
        assert np.array_equal(y.cpu().numpy()[sel], yn.numpy()[sel])
        assert np.array_equal(n.cpu().numpy()[sel], n_o[sel])


def test_draw_crossing_on_a_part_boundary():
    """P5 walks the slice in PSPLIT = 8 parts.  Here the residual (p - q)+ of
    the first three parts (columns 0-23 of a 64-column vector) is zero and
    u_res = 0, so the inverse-CDF crossing falls exactly on the boundary of
    part 3: the draw must be column 24 (the first with residual mass), on 1
    and 2 shards alike, as in the numpy restatement and the oracle."""
    V = 64
    tgt = torch.zeros(2, 2, V)
    drf = torch.zeros(2, 1, V)
    tgt[:, 0, 24:32] = 3.0                    # p puts its mass on columns 24-31
    drf[:, 0, :24] = 3.0                      # q on columns 0-23
    tgt[1, 1] = torch.linspace(-1, 1, V)
    tgt, drf = tgt.to(DEV, torch.bfloat16), drf.to(DEV, torch.bfloat16)
    xs = torch.zeros(2, 1, dtype=torch.long, device=DEV)       # q(0) >> p(0): rejected
    ua = torch.full((2, 1), 0.5, device=DEV)
    ur = torch.tensor([0.0, 0.37], device=DEV)
    n_o, y_o, _ = O.verify(_np(tgt), _np(drf), xs.cpu().numpy(), _np(ua), _np(ur), 1.0, 1.0, 0,
                           return_details=True)
    assert list(n_o) == [0, 0] and y_o[0] == 24
    for vs in ([0, V], [0, 32, V]):
        outs_c, st_c = SH.verify_sharded_local(tgt, drf, xs, ua, ur, vs, 1.0, 1.0)
        outs_n, st_n = SH.verify_sharded_local(tgt.cpu(), drf.cpu(), xs.cpu(), ua.cpu(), ur.cpu(),
                                               vs, 1.0, 1.0, backend_factory=NumpyShardBackend)
        assert st_c == st_n == [0] * (len(vs) - 1)
        for (n, y), (nn, yn) in zip(outs_c, outs_n):
            assert n.cpu().tolist() == nn.tolist() == [0, 0], vs
            assert y.cpu().tolist() == yn.tolist() == [int(y_o[0]), int(y_o[1])], vs


def test_fallback_status_matches_restatement():
    g = torch.Generator(device=DEV).manual_seed(0)
    B, k, V = 4, 2, 3000
    tgt = (torch.randn(B, k + 1, V, generator=g, device=DEV) * 3).to(torch.bfloat16)
    drf = (tgt[:, :k].float() + torch.randn(B, k, V, generator=g, device=DEV)).to(torch.bfloat16)
    xs = torch.randint(0, V, (B, k), generator=g, device=DEV)
    ua, ur = torch.rand(B, k, generator=g, device=DEV), torch.rand(B, generator=g, device=DEV)
    _, st_c = SH.verify_sharded_local(tgt, drf, xs, ua, ur, [0, V], 2.0, 0.95)
    _, st_n = SH.verify_sharded_local(tgt.cpu(), drf.cpu(), xs.cpu(), ua.cpu(), ur.cpu(), [0, V],
                                      2.0, 0.95, backend_factory=NumpyShardBackend)
    assert st_c == st_n == [2]


# ---------------------------------------------------------------------------
# two NCCL ranks (needs two GPUs)
# ---------------------------------------------------------------------------
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_rank(rank, world, port, out_dir):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        B, k = 8, 4
        tgt, drf = W.cfg2_logits(B=B, k=k, seed=2, device=dev)
        ua, ur = W.uniforms(B, k, seed=2, device=dev)
        xs = tgt[:, :k].float().argmax(-1)
        V = tgt.shape[-1]
        vs = SH.even_split(V, world)
        sl = slice(vs[rank], vs[rank + 1])
        comm = SH.ProcessGroupCollectives()
        res = {}
        for T, tp in [(0.7, 0.9), (0.0, 1.0)]:
            n, y = SH.verify_sharded(tgt[..., sl], drf[..., sl], xs, ua, ur, vs, comm,
                                     temperature=T, top_p=tp)
            n_f, y_f = S.verify_sample(tgt, drf, xs, ua, ur, T, tp, 0)
            res[(T, tp)] = (n.cpu(), y.cpu(), n_f.cpu(), y_f.cpu())
        torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_two_ranks(tmp_path):
    import torch.multiprocessing as mp
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.start_processes(_nccl_rank, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                           join=True, start_method="spawn")
    finally:
        os.environ.clear()
        os.environ.update(env)
    r0 = torch.load(tmp_path / "r0.pt")
    r1 = torch.load(tmp_path / "r1.pt")
    for key in r0:
        n0, y0, nf, yf = r0[key]
        n1, y1, _, _ = r1[key]
        assert torch.equal(n0, n1) and torch.equal(y0, y1), key
        # the fused kernel on the full vectors decides the same except at margins
        assert (n0 == nf).float().mean() >= 0.875 and (y0 == yf).float().mean() >= 0.875, key
