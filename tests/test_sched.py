"""Host-side checks of the persistent DP + stream-K schedule (no GPU).

The kernel walks exactly these work lists, so proving coverage here proves the
device does every k-iteration of every tile exactly once."""

from __future__ import annotations

from collections import defaultdict

import pytest

from gfx950_gluon_tutorials_b200 import _lib, ops

ROLE_FULL, ROLE_OWNER, ROLE_CONTRIB, ROLE_PAIR = 0, 1, 2, 3

SHAPES = [
    (_lib.KIND_F16, 4096, 4096, 8192),     # 256 pair tiles over 74 pairs
    (_lib.KIND_F16, 3840, 3840, 8192),     # 225 tiles
    (_lib.KIND_BF16, 512, 512, 1024),      # fewer tiles than units: all stream-K
    (_lib.KIND_F16, 300, 700, 200),        # ragged everything
    (_lib.KIND_E5M2, 4096, 4096, 8192),
    (_lib.KIND_MXE5M2, 4096, 4096, 8192),
    (_lib.KIND_MXFP4, 4096, 4096, 8192),
    (_lib.KIND_MXFP4, 16384, 6656, 16384),  # one 8-GPU shard of the large config
    (_lib.KIND_MXFP4, 128, 256, 64),       # a single tile, single k-iteration
]


@pytest.fixture(params=[(0, 1), (1, 1), (2, 1), (3, 1), (4, 1), (1, 0), (2, 0), (3, 0), (4, 0)],
                ids=lambda p: f"sk{p[0]}-pair{p[1]}")
def options(request):
    sk, pair = request.param
    old = {k: _lib.get_option(k) for k in (_lib.OPT_SK_MODE, _lib.OPT_PAIR,
                                           _lib.OPT_MIN_SK_ITERS)}
    _lib.set_option(_lib.OPT_SK_MODE, sk)
    _lib.set_option(_lib.OPT_PAIR, pair)
    _lib.set_option(_lib.OPT_MIN_SK_ITERS, 1)
    yield
    for k, v in old.items():
        _lib.set_option(k, v)


@pytest.mark.parametrize("num_sms", [148, 132, 20])
@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_schedule_covers_every_iteration_once(options, shape, num_sms):
    kind, M, N, K = shape
    p = ops.plan(kind, M, N, K, num_sms)
    tiles = p["tiles_m"] * p["tiles_n"]
    cover = defaultdict(int)
    owners = {}
    contrib_of = defaultdict(list)
    pairs = defaultdict(list)
    coords = {}
    for u in range(p["launched"]):
        items = ops.plan_items(kind, M, N, K, u, num_sms)
        seen_sk = False
        for idx, (t, tm, tn, kb, ke, role, first, n_c, stride, nh, ph) in enumerate(items):
            assert 0 <= t < tiles and 0 <= tm < p["tiles_m"] and 0 <= tn < p["tiles_n"]
            assert coords.setdefault(t, (tm, tn)) == (tm, tn)
            assert 0 <= kb < ke <= p["k_iters"]
            assert nh in (-1, 0, 1)
            if nh >= 0:
                # half-width tiles: whole K, no partial-tile reduction
                assert p["half"] == 1 and role == ROLE_FULL and (kb, ke) == (0, p["k_iters"])
            # a whole tile covers both 128-column halves
            for h in ((0, 1) if nh < 0 else (nh,)):
                for k in range(kb, ke):
                    cover[(t, h, k)] += 1
            if role == ROLE_CONTRIB:
                # a unit contributes at most once, in its first stream-K segment
                assert not seen_sk
                assert u < p["sk_units"]
                contrib_of[t].append(u)
            if role == ROLE_OWNER:
                assert kb == 0 and ke < p["k_iters"]
                assert t not in owners
                owners[t] = (u, [first + i * stride for i in range(n_c)])
                assert idx == len(items) - 1  # the owner's wait is its last item
            if role == ROLE_PAIR:
                # one of two pieces: the unit's last item, naming its peer
                assert p["splits"] == 2 and ph in (0, 1) and idx == len(items) - 1
                pairs[t].append((u, ph, first, kb, ke))
            else:
                assert ph == -1
            if t >= p["dp_tiles"]:
                seen_sk = True
    assert len(cover) == 2 * tiles * p["k_iters"]
    assert all(v == 1 for v in cover.values())
    assert len(set(coords.values())) == tiles
    for t, units in contrib_of.items():
        u, listed = owners[t]
        assert sorted(units) == listed
        assert u < min(listed)
    assert set(owners) == set(contrib_of)
    for t, pieces in pairs.items():
        # the two pieces keep complementary column halves and name each other
        assert len(pieces) == 2
        (u0, h0, peer0, kb0, ke0), (u1, h1, peer1, kb1, ke1) = sorted(pieces, key=lambda x: x[1])
        assert (h0, h1) == (0, 1) and peer0 == u1 and peer1 == u0
        assert kb0 == 0 and ke0 == kb1 and ke1 == p["k_iters"]


def test_default_plan_for_the_headline_config():
    p = ops.plan(_lib.KIND_F16, 4096, 4096, 8192, 148)
    assert p["cta_group"] == 2 and p["units"] == 74
    assert p["tiles_m"] * p["tiles_n"] == 256
    # 3 full waves of 74 pair tiles, then 34 tiles split in 2 k-halves on 68 pairs
    assert p["dp_tiles"] == 222 and p["splits"] == 2 and p["sk_units"] == 68
    p = ops.plan(_lib.KIND_MXFP4, 4096, 4096, 8192, 148)
    # 4096 bytes of packed K per row, in stages of two 128-byte chunks
    assert p["cta_group"] == 2 and p["units"] == 74 and p["k_iters"] == 16
    # 16-stage tiles are too short to split (a piece must span 16 stages):
    # the 34 leftover tiles run as 68 half-width tiles instead
    assert p["splits"] == 0 and p["half"] == 1 and p["sk_units"] == 68


@pytest.fixture
def half_mode():
    old = _lib.get_option(_lib.OPT_SK_MODE)
    _lib.set_option(_lib.OPT_SK_MODE, 4)
    yield
    _lib.set_option(_lib.OPT_SK_MODE, old)


def test_half_mode_plans(half_mode):
    # 4096^2: the 34 leftover tiles as 68 half-width tiles on 68 pairs
    p = ops.plan(_lib.KIND_F16, 4096, 4096, 8192, 148)
    assert p["dp_tiles"] == 222 and p["half"] == 1 and p["sk_units"] == 68
    # 3840^2: 225 tiles = 3 waves + 3 leftovers -> 6 half tiles fit
    p = ops.plan(_lib.KIND_F16, 3840, 3840, 8192, 148)
    assert p["half"] == 1 and p["sk_units"] == 6
    # 50 leftover tiles (2 x 50 > 74 units): k-splits instead
    p = ops.plan(_lib.KIND_F16, 256 * 11, 256 * 11, 8192, 148)   # 121 tiles = 74 + 47
    assert p["dp_tiles"] == 74 and p["half"] == 0 and p["splits"] >= 1


@pytest.mark.parametrize("kind,M,N,K,expect", [
    (_lib.KIND_F16, 4096, 4096, 8192, 16),      # A (64 MiB) stays in L2: column strips
    (_lib.KIND_F16, 3840, 3840, 8192, 15),
    (_lib.KIND_MXE5M2, 4096, 4096, 8192, 1),    # A and B fit in L2 together: row-major
    (_lib.KIND_MXFP4, 4096, 4096, 8192, 1),
    (_lib.KIND_MXFP4, 16384, 53248, 16384, 16),  # neither fits: bands of 16 x 2 MiB of A
    (_lib.KIND_MXFP4, 16384, 13312, 16384, 16),
    (_lib.KIND_MXFP4, 16384, 6656, 16384, 1),    # B (52 MiB) stays in L2: row-major
])
def test_automatic_raster_group(kind, M, N, K, expect):
    assert _lib.get_option(_lib.OPT_GROUP_M) == 0
    assert ops.plan(kind, M, N, K, 148)["group_m"] == expect
