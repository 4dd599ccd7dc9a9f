"""sd_verify_greedy_static: the greedy verify round on the library's fixed
device scratch (no workspace, no allocation) against sd_verify_sample.  It
exists for callers that may not allocate device memory, such as a serving
framework that owns the whole GPU memory pool.

Kept in its own file, collected last, so it runs both after the rest of the
suite and alone (`pytest tests/test_zz_no_alloc.py -m gpu`).
"""
import pytest
import torch

from specdec import _lib as L
from specdec import sampling as S
from specdec import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(seed, B=24, k=4, V=32003):
    g = torch.Generator(device=DEV).manual_seed(seed)
    tgt = (torch.randn(B, k + 1, V, generator=g, device=DEV) * 3).to(torch.bfloat16)
    am = tgt.float().argmax(-1)
    # draft ids: the target argmax for most positions, so prefixes of every length occur
    xs = torch.where(torch.rand(B, k, generator=g, device=DEV) < 0.8, am[:, :k],
                     torch.randint(0, V, (B, k), generator=g, device=DEV))
    ua = torch.rand(B, k, generator=g, device=DEV)
    ur = torch.rand(B, generator=g, device=DEV)
    alive = torch.rand(B, generator=g, device=DEV) < 0.9
    return tgt, xs.contiguous(), ua, ur, alive


def _static(tgt, xs, ua, alive):
    B, k1, V = tgt.shape
    k = k1 - 1
    n = torch.full((B,), -7, dtype=torch.long, device=DEV)
    y = torch.full((B,), -7, dtype=torch.long, device=DEV)
    px = torch.empty(B, k, dtype=torch.float32, device=DEV)
    al = alive.to(torch.uint8).contiguous()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    rc = L.lib().sd_verify_greedy_static(
        L.ptr(tgt), tgt.stride(0), tgt.stride(1), L.dtype_code(tgt.dtype), L.ptr(xs),
        xs.stride(0), L.ptr(ua), ua.stride(0), L.ptr(al), B, k, V, L.ptr(n), L.ptr(y),
        L.ptr(px), None, L.stream_ptr(tgt.device))
    torch.cuda.synchronize()
    assert rc == 0
    assert torch.cuda.mem_get_info()[0] == free0          # nothing allocated on the device
    return n, y, px


def test_static_scratch_matches_workspace_entry_point():
    for call in range(2):                                  # two calls in a row
        tgt, xs, ua, ur, alive = _inputs(call)
        n_w, y_w, px_w, _ = S.verify_sample(tgt, None, xs, ua, ur, 0.0, 1.0, alive=alive,
                                             return_probs=True)
        n_s, y_s, px_s = _static(tgt, xs, ua, alive)
        assert torch.equal(n_s, n_w), call
        assert torch.equal(y_s, y_w), call
        assert torch.equal(px_s, px_w), call


def test_static_scratch_config2_shape():
    tgt, _ = W.cfg2_logits(B=64, seed=3)
    xs = tgt[:, :4].float().argmax(-1).contiguous()
    ua, ur = W.uniforms(64, 4, seed=3)
    alive = torch.ones(64, dtype=torch.bool, device=DEV)
    n_w, y_w = S.verify_sample(tgt, None, xs, ua, ur, 0.0, 1.0)
    n_s, y_s, _ = _static(tgt, xs, ua, alive)
    assert torch.equal(n_s, n_w) and torch.equal(y_s, y_w)


def test_static_scratch_rejects_oversize():
    B, k, V = 4096, 4, 151936                              # needs more than the fixed scratch
    tgt = torch.zeros(1, dtype=torch.bfloat16, device=DEV)
    xs = torch.zeros(1, dtype=torch.long, device=DEV)
    ua = torch.zeros(1, device=DEV)
    out = torch.zeros(1, dtype=torch.long, device=DEV)
    rc = L.lib().sd_verify_greedy_static(
        L.ptr(tgt), V * (k + 1), V, L.dtype_code(tgt.dtype), L.ptr(xs), k, L.ptr(ua), k, None,
        B, k, V, L.ptr(out), L.ptr(out), None, None, L.stream_ptr(tgt.device))
    assert rc == -28                                        # SD_ENOSPC, before any launch
