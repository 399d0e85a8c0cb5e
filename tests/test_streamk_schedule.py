"""The stream-K work split of the tcgen05 GEMM, restated and checked on the CPU.

The GEMM (roofline.c_b200/csrc/cuda/gemm_tc.cu) runs R = tiles // P whole
waves of tiles; the L = tiles % P tiles of a partial last wave are cut into
L * C chunk units (C = K / chunk) dealt out in equal contiguous ranges, range
q = [L*C*q // P, L*C*(q+1) // P) (struct Sched). A tile cut by a range
boundary is finished by its owner, the group holding its chunk 0; later
groups (contributors) hand their partial sums over and raise a flag that the
owner waits on (the epilogue's `skm && sg.c0 > 0` / `sg.c1 < n_chunks`
branches). The host enables it (gemm_plan) for a partial last wave that
leaves at least half the groups idle or has >= 6 chunks per tile, and then
launches g = min(groups, units) groups when there is less than one wave.

Checked for every shape: the segments cover each (tile, chunk) exactly once;
a contributor segment is only ever the first stream-K segment of its group
and an owner segment only the last, so contributors never wait and no wait
is circular; the groups an owner's loop visits are exactly the tile's
contributors, each flag is raised once and cleared once per launch.
"""
import itertools

import pytest


def plan(tiles, chunks, groups, mode=1):
    """(grid groups, stream-K?) as gemm_plan chooses them."""
    last = tiles % groups
    pays = mode == 2 or last <= groups // 2 or chunks >= 6
    if mode and last != 0 and chunks > 1 and pays:
        units = tiles * chunks
        g = groups if tiles >= groups else min(units, groups)
        return g, True
    return min(tiles, groups), False


def segments(num_tiles, C, sk, P, p):
    """Struct Sched's sequence of (tile, c0, c1) for group p of P."""
    out = []
    if sk:
        R = num_tiles // P
        LC = (num_tiles % P) * C
        first = lambda q: LC * q // P  # noqa: E731
        u, ue = first(p), first(p + 1)
    else:
        R = -(-num_tiles // P)
        u = ue = 0
    for i in range(R):
        t = i * P + p
        if t < num_tiles:
            out.append((t, 0, C))
    while u < ue:
        tile = R * P + u // C
        c0 = u % C
        c1 = min(C, c0 + (ue - u))
        out.append((tile, c0, c1))
        u += c1 - c0
    return out


def owner_visits(num_tiles, C, P, p, tile):
    """The groups the owner's loop waits on for `tile` (gemm_tc.cu epilogue)."""
    R = num_tiles // P
    LC = (num_tiles % P) * C
    first = lambda q: LC * q // P  # noqa: E731
    end = (tile - R * P + 1) * C
    qs = []
    qq = p + 1
    while qq < P and first(qq) < end:
        if first(qq + 1) != first(qq):
            qs.append(qq)
        qq += 1
    return qs


SHAPES = list(itertools.product(
    [1, 2, 3, 7, 13, 26, 50, 73, 74, 75, 100, 147, 148, 149, 160, 200, 222, 296, 300, 312, 444, 600],
    [1, 2, 3, 4, 5, 6, 8, 12, 16, 24],
    [148, 74],
    [1, 2],
))


@pytest.mark.parametrize("tiles,C,groups,mode", SHAPES)
def test_streamk_split(tiles, C, groups, mode):
    P, sk = plan(tiles, C, groups, mode)
    cover = {}
    contributors = {}
    owners = {}
    for p in range(P):
        segs = segments(tiles, C, sk, P, p)
        R = tiles // P if sk else None
        sk_segs = [s for s in segs if sk and s[0] >= R * P]
        for k, (t, c0, c1) in enumerate(segs):
            assert 0 <= c0 < c1 <= C
            for c in range(c0, c1):
                assert (t, c) not in cover, (t, c)
                cover[(t, c)] = p
        for k, (t, c0, c1) in enumerate(sk_segs):
            if c0 > 0:                                  # contributor
                assert k == 0, "a contributor segment is the first of its range"
                contributors.setdefault(t, []).append(p)
            if c0 == 0 and c1 < C:                      # owner of a cut tile
                assert k == len(sk_segs) - 1, "an owner segment is the last of its range"
                assert t not in owners
                owners[t] = p
    assert len(cover) == tiles * C
    assert all(0 <= t < tiles for t, _ in cover)
    # every cut tile has one owner, earlier than all of its contributors,
    # and the owner's wait loop visits exactly those contributors
    assert set(contributors) == set(owners)
    flags = {}
    for t, q in contributors.items():
        p = owners[t]
        assert all(c > p for c in q)
        assert owner_visits(tiles, C, P, p, t) == sorted(q)
        for c in q:
            flags[c] = flags.get(c, 0) + 1
    assert all(v == 1 for v in flags.values()), "one flag raise per contributing group"
