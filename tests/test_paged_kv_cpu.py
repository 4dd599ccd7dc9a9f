"""Host-side page bookkeeping of the paged KV cache (no GPU).

PageTable hands pages of PAGE slots to rows before the forwards that write
them; the kernels then read and write through its block table.  These tests
replay engine-like traces (growth by k + 1, commits that roll back, a
right-padded prefill, finished rows released) and check after every step that
no page is owned twice, none is lost, and every slot a forward can touch has
a page.
"""
import numpy as np
import pytest

from specdec import _lib as L
from specdec.kvcache import PAGE, PageTable


def _covered(pt, lengths, q):
    for b, n in enumerate(lengths):
        need = -(-(int(n) + q) // PAGE)
        assert (pt.bt[b, :need] >= 0).all() and (pt.bt[b, :need] != pt.sink).all()


def test_reserve_hands_out_pages_in_slot_order():
    pt = PageTable(3, 8, 20)
    assert pt.reserve([0, 0, 0], 1)
    assert pt.bt[:, 0].tolist() == [0, 1, 2] and (pt.bt[:, 1:] == -1).all()
    assert not pt.reserve([1, 1, 1], 5)                 # still inside the first page
    assert pt.reserve([120, 0, 300], 10)
    assert pt.owned.tolist() == [2, 1, 3]
    pt.check()
    assert len(pt.free) == 19 - 6


def test_prefill_points_padding_at_the_sink():
    pt = PageTable(3, 8, 30)
    P = 3 * PAGE + 5
    pt.reserve_prefill([0, 0, 0], P, [P, 10, 2 * PAGE])
    assert pt.owned.tolist() == [4, 1, 2]
    assert (pt.bt[1, 1:4] == pt.sink).all() and (pt.bt[2, 2:4] == pt.sink).all()
    assert (pt.bt[0, :4] != pt.sink).all()
    pt.check()
    assert pt.unsink()
    assert not (pt.bt == pt.sink).any()
    assert (pt.bt[1, 1:] == -1).all()
    pt.check()


def test_pool_exhaustion_raises():
    pt = PageTable(2, 4, 4)                              # 3 pages to hand out
    with pytest.raises(L.SpecdecError):
        pt.reserve([0, 0], PAGE + 1)                     # 2 + 2 wanted
    pt2 = PageTable(2, 4, 40)
    with pytest.raises(RuntimeError):
        pt2.reserve([4 * PAGE - 2, 0], 3)                # past the row capacity


def test_release_and_reuse():
    pt = PageTable(3, 4, 10)
    pt.reserve([0, 0, 0], 2 * PAGE)
    got = set(pt.bt[1, :2].tolist())
    pt.release([1])
    assert (pt.bt[1] == -1).all() and pt.owned[1] == 0
    pt.reserve([0, 0, 0], 3 * PAGE)                      # freed pages are handed out first
    assert got <= set(pt.bt[:, :3].ravel().tolist())
    pt.check()
    pt.reset()
    assert len(pt.free) == 9 and (pt.bt == -1).all()


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_engine_trace_keeps_every_touched_slot_paged(seed):
    """Prefill, then rounds of k + 1 appends and a commit that keeps n_acc + 1
    of them; rows that finish keep growing by one per round; half the rows
    are released and refilled mid-way."""
    rng = np.random.default_rng(seed)
    B, W = 16, 12
    pt = PageTable(B, W, B * W + 1)
    plen = rng.integers(1, 3 * PAGE, B)
    P = int(plen.max())
    lens = np.zeros(B, dtype=np.int64)
    pt.reserve_prefill(lens, P, plen)
    pt.check()
    lens = plen.copy()
    pt.unsink()
    for rnd in range(200):
        k = int(rng.integers(1, 8))
        if int((lens + k + 1).max()) > W * PAGE:
            break
        pt.reserve(lens, k + 1)
        _covered(pt, lens, k + 1)
        lens = lens + 1 + rng.integers(0, k + 1, B)      # commit: n_acc + 1 kept
        if rnd == 60:
            rows = np.arange(0, B, 2)
            pt.release(rows)
            lens[rows] = 0
            pt.reserve(lens, 50)                         # refill the released rows
            _covered(pt, lens, 50)
            lens[rows] = 50
        pt.check()
    assert rnd > 20
