"""CPU tests of the attention kernels' launch order (``grouped_order`` and
``locality_group`` in ``csrc/attn_common.cuh``), called through host wrappers in the
test-only self-test library.

The order decides which (head, batch) pair and which tile each CTA (or each persistent
work item) takes, so it must be a bijection onto every (tile, pair) of the grid, keep
each group's tiles heaviest first, and fall back to the plain heaviest-first order when
the shared tiles fit in L2. The GPU side (every output written, heads of the first and
last group against the oracle) is ``tests/test_locality_order.py``.
"""

import ctypes
import os

import pytest

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc", "libfh_selftest.so")
MB = 1 << 20


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        from tests.csrc.build_selftest import build

        build()
    so = ctypes.CDLL(LIB)
    so.fh_selftest_grouped_order.argtypes = [ctypes.c_int] * 4 + [ctypes.POINTER(ctypes.c_int)] * 2
    so.fh_selftest_grouped_order.restype = None
    so.fh_selftest_locality_group.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_longlong]
    so.fh_selftest_locality_group.restype = ctypes.c_int
    return so


def _order(lib, tiles, pairs, g):
    ti, pair = ctypes.c_int(), ctypes.c_int()
    out = []
    for w in range(tiles * pairs):
        lib.fh_selftest_grouped_order(w, tiles, pairs, g, ctypes.byref(ti), ctypes.byref(pair))
        out.append((ti.value, pair.value))
    return out


@pytest.mark.parametrize("tiles,pairs,g", [
    (16, 64, 64), (16, 64, 32), (64, 64, 4), (64, 13, 5), (7, 104, 21), (3, 10, 1), (5, 9, 9), (5, 9, 20),
    (32, 128, 16), (1, 7, 3),
])
def test_grouped_order_is_a_bijection_heaviest_first_per_group(lib, tiles, pairs, g):
    order = _order(lib, tiles, pairs, g)
    assert sorted(order) == [(t, p) for t in range(tiles) for p in range(pairs)]
    gs = min(g, pairs)
    for w, (t, p) in enumerate(order):
        grp = p // gs
        # Every item of group `grp` comes after all items of the earlier groups.
        assert w >= grp * gs * tiles
        assert w < grp * gs * tiles + min(gs, pairs - grp * gs) * tiles
    # Within a group the tile index never decreases (heaviest first), pairs fastest.
    for a, b in zip(order, order[1:]):
        if a[1] // gs == b[1] // gs:
            assert b[0] >= a[0]


def test_one_group_is_the_plain_order(lib):
    tiles, pairs = 16, 64
    assert _order(lib, tiles, pairs, pairs) == [(w // pairs, w % pairs) for w in range(tiles * pairs)]


def test_locality_group_sizes(lib):
    lg = lib.fh_selftest_locality_group
    # Headline (B4 H16 S2048 D64): 1 MB (query pass) / 0.75 MB (key pass) per head, all
    # 64 pairs fit in L2 -> one group, the plain order.
    assert lg(64, 1, 4 * 2048 * 64 * 2) == 64
    assert lg(64, 1, 3 * 2048 * 64 * 2) == 64
    # Configuration 3 (B2 H32 S8192 D128): 8 MB / 6 MB per head -> groups of 4 / 5.
    assert lg(64, 1, 4 * 8192 * 128 * 2) == 4
    assert lg(64, 1, 3 * 8192 * 128 * 2) == 5
    # Configuration 4 (B8 H16, Sk 2048, Sq 4096, D128): 2 MB / 3 MB -> 16 / 10.
    assert lg(128, 1, 4 * 2048 * 128 * 2) == 16
    assert lg(128, 1, 3 * 4096 * 128 * 2) == 10
    # GQA: whole query-head groups (a multiple of `shared`), counted by key heads.
    assert lg(208, 2, 2 * 2048 * 128 * 2) == 64
    assert lg(48, 2, 2 * MB) == 48  # 24 key heads x 2 MB = 48 MB fits
    # Heads larger than a group's budget: one key head (its query heads) per group.
    assert lg(64, 1, 100 * MB) == 1
    assert lg(64, 4, 100 * MB) == 4
    # Exactly at the L2 bound stays plain; just above it groups.
    assert lg(96, 1, MB) == 96
    assert lg(97, 1, MB) == 32
