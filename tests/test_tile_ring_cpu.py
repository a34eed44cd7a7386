"""CPU restatement of the weight-tile producers' group schedule (the
persistent kernel's mega_producer, s2k_mega.cu, and tgemv_kernel's producer,
s2k_gemv.cu): tiles go out in groups of up to four, one bulk copy per lane,
and lane 0 waits once per group for the consumers to release one earlier
tile.  The properties checked here are what keep the ring safe: a tile is
copied into a slot only after the slot's previous tile was consumed, a wait
never targets a tile that is not yet issued (it would never end), and the
standalone kernel issues exactly its first ring-full of tiles without a check
(an aborting launch drains exactly those).  No GPU."""
from __future__ import annotations

import pytest

K_MSTAGES = 10  # kMStages
K_MAX_PL = 4  # kMaxPL / kGemvPL


def mega_groups(ntiles: int, depth: int, lanes: int):
    """(first tile, tiles in the group, tile whose release is awaited or -1),
    as mega_producer forms them."""
    gmax = max(1, min(min(lanes, K_MAX_PL), depth))
    ps = 0
    while ps < ntiles:
        n = min(gmax, ntiles - ps)
        q = ps + n - 1 - depth
        yield ps, n, q if q >= 0 else -1
        ps += n


def gemv_groups(ntiles: int, ns: int):
    """The same for tgemv_kernel's producer (ring of ns slots, depth ns):
    groups never straddle tile ns, and tiles below ns are issued unchecked."""
    t = 0
    while t < ntiles:
        n = min(min(K_MAX_PL, ntiles - t), ns - t if t < ns else K_MAX_PL)
        q = t + n - 1 - ns
        yield t, n, q if t + n - 1 >= ns else -1
        t += n


def _check_schedule(groups, ntiles: int, ns: int, depth: int):
    issued = 0
    for first, n, q in groups:
        assert first == issued and 1 <= n <= K_MAX_PL
        assert q < first, "a wait on a tile of its own group or later never ends"
        released = q  # consumers release in order: every tile <= q is free
        for t in range(first, first + n):
            # the slot's previous tile (t - ns) and the in-flight bound (t - depth) are released
            assert t - ns <= released and t - depth <= released
            assert len({(tt % ns) for tt in range(first, first + n)}) == n  # distinct slots in a group
        issued += n
    assert issued == ntiles


@pytest.mark.parametrize("lanes", [1, 2, 3, 4, 7])
@pytest.mark.parametrize("depth", [1, 2, 4, 9, 10])
def test_persistent_producer_groups_are_safe(lanes, depth):
    for ntiles in (0, 1, 3, 9, 10, 11, 25, 57, 1000):
        _check_schedule(mega_groups(ntiles, depth, lanes), ntiles, K_MSTAGES, depth)


@pytest.mark.parametrize("ns", [5, 7, 9])
def test_gemv_producer_groups_are_safe_and_drainable(ns):
    for ntiles in (0, 1, 4, ns - 1, ns, ns + 1, 2 * ns + 3, 200):
        groups = list(gemv_groups(ntiles, ns))
        _check_schedule(iter(groups), ntiles, ns, ns)
        # exactly the first min(ntiles, ns) tiles go out before the first check
        unchecked = 0
        for first, n, q in groups:
            if q >= 0:
                break
            unchecked += n
        assert unchecked == min(ntiles, ns)
        # and the first check awaits a tile inside that drained ring-full
        checked = [q for _, _, q in groups if q >= 0]
        if checked:
            assert checked[0] < min(ntiles, ns)
