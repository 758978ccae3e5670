"""Host-side check of the split-KV work schedule used by gqa_decode_kernel.

The kernel flattens all (segment, 64-token tile) pairs, splits them over
min(grid, total) CTAs (CTA c owns tiles [c*T/n, (c+1)*T/n)), files one piece
per (CTA, segment) pair it touches into workspace slot c + segment, and the
CTA that files a group's last piece merges np(group) pieces.  This restates
that arithmetic (scope_b200/csrc/gqa_decode.cu: split_start / split_owner /
SegTable::pieces and the slot list of the merge) and checks its invariants
on CPU for dense and ragged multi-share batches, including grids larger than
the tile count.
"""
import itertools
import random

import pytest

TILE = 64


def split_start(c, total, n):
    return (c * total) // n


def split_owner(t, total, n):
    return ((t + 1) * n + total - 1) // total - 1


def segments(lens_by_share, Hkv):
    """Segments in flattened order: (b, h, s) -> (group, first tile, tiles)."""
    B = len(lens_by_share[0])
    segs = []
    t = 0
    for b in range(B):
        for h in range(Hkv):
            for s, lens in enumerate(lens_by_share):
                nt = (lens[b] + TILE - 1) // TILE
                segs.append(((b * Hkv + h), t, nt))
                t += nt
    return segs, t


def check(lens_by_share, Hkv, grid):
    segs, total = segments(lens_by_share, Hkv)
    nseg = len(segs)
    n = max(1, min(grid, total))
    # every tile has exactly one owner, the one whose range holds it
    owner_of = {}
    for c in range(n):
        for t in range(split_start(c, total, n), split_start(c + 1, total, n)):
            assert t not in owner_of
            owner_of[t] = c
    assert len(owner_of) == total
    for t in range(total):
        assert split_owner(t, total, n) == owner_of[t]
    # every working CTA owns at least one tile
    assert all(split_start(c + 1, total, n) > split_start(c, total, n) for c in range(n)) or total == 0
    # pieces actually filed: distinct (cta, segment) pairs
    filed = {}
    for j, (g, t0, nt) in enumerate(segs):
        for t in range(t0, t0 + nt):
            filed.setdefault(g, set()).add((owner_of[t], j))
    slots = set()
    for g in range(len(lens_by_share[0]) * Hkv):
        pieces = filed.get(g, set())
        # np(group) as the kernel computes it
        np_ = 0
        listed = []
        for j, (gg, t0, nt) in enumerate(segs):
            if gg != g or nt == 0:
                continue
            c0, c1 = split_owner(t0, total, n), split_owner(t0 + nt - 1, total, n)
            np_ += c1 - c0 + 1
            listed += [c + j for c in range(c0, c1 + 1)]
        assert np_ == len(pieces), (g, np_, len(pieces))
        assert sorted(listed) == sorted(c + j for c, j in pieces)
        for c, j in pieces:
            s = c + j
            assert s not in slots          # slots never collide
            assert 0 <= s < n + nseg       # and fit the workspace
            slots.add(s)


@pytest.mark.parametrize("grid", [1, 7, 148])
def test_dense_rows(grid):
    for rows, L in [(4, 4096), (128, 131072), (300, 40), (3, 1), (16, 65536), (2, 0)]:
        check([[L] * rows], 1, grid)


@pytest.mark.parametrize("grid", [1, 10, 148, 1000])
def test_ragged_shares_random(grid):
    rng = random.Random(grid)
    for _ in range(40):
        B = rng.randint(1, 9)
        Hkv = rng.choice([1, 2, 8])
        nshare = rng.randint(1, 4)
        lens = [[rng.choice([0, 1, 63, 64, 65, rng.randint(0, 5000)]) for _ in range(B)] for _ in range(nshare)]
        check(lens, Hkv, grid)


def test_fewer_tiles_than_ctas():
    # the case that needs the min(grid, total) split: 10 tiles, 148 CTAs
    check([[300, 0], [0, 0]], 2, 148)
    check([[300, 5], [7, 0]], 2, 148)
