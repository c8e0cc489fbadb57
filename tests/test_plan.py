"""CPU: invariants of the device-side work split (mirrored in kernel_optim_b200/plan.py)."""

import random
from collections import defaultdict

import pytest

from kernel_optim_b200.plan import PAGE, all_units, max_units, plan, schedule


def check_plan(lengths, nkv, grid, fused, max_len=None, static_pct=100, skew=False):
    us = all_units(lengths, nkv, grid, fused, static_pct, skew)
    B = len(lengths)
    pl = plan(lengths, nkv, grid, fused, static_pct, skew)
    limit = max_units(B, nkv, max_len or max(lengths), grid)
    slots = [u.slot for u in us]
    assert len(slots) == len(set(slots)), "two units share a workspace slot"
    assert all(0 <= x < limit for x in slots)
    # every chunk is non-empty, except that all pieces are empty when P = 0, and the pieces past
    # pairs * parts in the pair-aligned layout
    for k in range(pl.total_chunks):
        x0, x1 = pl.chunk_range(k)
        assert (x1 > x0 or (k < grid and pl.static_pages == 0) or (pl.parts and k >= B * nkv * pl.parts)
                or (pl.group and k * pl.group >= B * nkv))
    if pl.parts:   # one unit per CTA, each pair cut into exactly `parts` pieces of its own
        assert all(sum(1 for u in us if u.chunk == k) <= 1 for k in range(grid))
        assert all(u.n == pl.parts for u in us)
    if pl.group:   # whole pairs, `group` of them per CTA: nothing split, nothing merged
        assert all(u.n == 1 for u in us)
        assert all(sum(1 for u in us if u.chunk == k) <= pl.group for k in range(grid))
    by_pair = defaultdict(list)
    for u in us:
        by_pair[u.q].append(u)
    assert set(by_pair) == set(range(B * nkv)), "a (sequence, kv head) pair has no unit"
    for q, lst in by_pair.items():
        b = q // nkv
        ls = lengths[b] - 1 if fused else lengths[b]
        pos = 0
        for u in lst:   # keys [0, Ls) covered exactly once, in order, on page boundaries
            assert u.t0 == pos and u.t0 % PAGE == 0
            pos = u.t1
        assert pos == ls
        # the units of a pair sit in consecutive chunks and agree on the split count
        assert [u.chunk for u in lst] == list(range(lst[0].c0, lst[0].c0 + lst[0].n))
        assert all(u.n == len(lst) for u in lst)
        assert [u.last for u in lst] == [False] * (len(lst) - 1) + [True]
    return pl, us


@pytest.mark.parametrize("fused", [False, True])
def test_baseline_configs(fused):
    pl, us = check_plan([4097] * 16, 8, 148, fused)
    assert pl.static_pages == pl.total_pages and pl.total_chunks == 148   # one piece per CTA
    assert pl.parts == 1                        # c2: 128 pairs of equal length, one per CTA
    assert len(us) == 128 and all(u.n == 1 and u.t0 == 0 for u in us)
    pl, _ = check_plan([4097] * 16, 8, 148, fused, static_pct=90)
    assert 0 < pl.static_pages < pl.total_pages and pl.total_chunks > 148
    check_plan([131072] * 4, 8, 148, fused)
    check_plan([1] * 3, 8, 148, fused)              # fewer pages than CTAs: no static pieces
    check_plan([5, 130, 77], 8, 148, fused, 136)


def test_random_lengths_grids_and_heads():
    rng = random.Random(0)
    for _ in range(300):
        B = rng.randint(1, 40)
        nkv = rng.choice([1, 2, 4, 8])
        grid = rng.choice([1, 2, 7, 37, 148, 296, 1000])
        lengths = [rng.choice([1, 2, 15, 16, 17, 512, 513, rng.randint(1, 20000)]) for _ in range(B)]
        check_plan(lengths, nkv, grid, rng.random() < 0.5, static_pct=rng.choice([0, 60, 90, 100]),
                   skew=rng.random() < 0.5)


def test_dynamic_claims_take_every_chunk_once():
    rng = random.Random(1)
    for _ in range(50):
        grid = rng.choice([1, 7, 148, 296])
        n = grid + rng.randint(0, 3000)
        speeds = [rng.uniform(0.7, 1.3) for _ in range(grid)]
        taken = schedule(n, grid, speeds)
        assert sorted(g for t in taken for g in t) == list(range(n))


def test_late_start_allowance():
    """Overlapped launches on c2: the last 4 pieces are 24, 12, 6 and 6 pages shorter (last CTA
    shortest), the others share the difference, and the split still covers every key once."""
    from kernel_optim_b200.plan import LATE_PAGES
    lens = [4097] * 15 + [3001]      # not all equal: the line is cut into pieces
    pl0, _ = check_plan(lens, 8, 148, True)
    pl, _ = check_plan(lens, 8, 148, True, skew=True)
    assert pl.late and not pl0.late
    q = pl.static_pages // 148
    lens = [pl.chunk_range(k)[1] - pl.chunk_range(k)[0] for k in range(148)]
    assert lens[-4:] == [q - d for d in reversed(LATE_PAGES)]
    assert min(lens[:-4]) >= q
    check_plan([5, 130, 77], 8, 148, True, skew=True)      # too short: no allowance


def test_whole_pair_groups():
    """Equal lengths, more pairs than CTAs: pieces of m whole pairs each (c5's decode step:
    32 x 8 = 256 pairs on 148 CTAs -> 128 pieces of 2 pairs), only when m divides the pair count
    and >= 80% of the grid is used."""
    pl, us = check_plan([1153] * 32, 8, 148, True)
    assert pl.group == 2 and pl.parts == 0 and not pl.late and len(us) == 256
    assert check_plan([1153] * 37, 8, 148, True)[0].group == 2     # 296 pairs: 148 pieces
    assert check_plan([1153] * 19, 8, 148, True)[0].group == 0     # 152 pairs: m = 2 leaves 76
    assert check_plan([1153] * 40, 8, 148, True)[0].group == 0     # 320 pairs: 3 does not divide
    assert check_plan([1153, 1000] * 16, 8, 148, True)[0].group == 0   # unequal lengths


def test_pair_aligned_pieces():
    """Equal lengths, no more pairs than CTAs: each pair cut into the same number of parts of its
    own (c4: 32 pairs x 4 parts = 128 CTAs, one unit each); only when >= 80% of the grid is used,
    every part has a page, and nothing is dynamic; skew (the late-start allowance) is off then."""
    pl, us = check_plan([131072] * 4, 8, 148, True, skew=True)
    assert pl.parts == 4 and not pl.late and len(us) == 128
    assert [pl.chunk_range(k)[1] - pl.chunk_range(k)[0] for k in range(4)] == [2048] * 4
    pl, _ = check_plan([4097] * 16, 8, 148, True, skew=True)
    assert pl.parts == 1 and not pl.late
    assert check_plan([4097] * 12, 8, 148, True)[0].parts == 0      # 96 pairs: 65% of the grid
    assert check_plan([4097] * 15, 8, 148, True)[0].parts == 1      # 120 pairs: 81%
    assert check_plan([17] * 4, 8, 148, True)[0].parts == 0         # 32 pairs of 1 page: k = 1, 22%
    assert check_plan([33] * 4, 4, 148, False)[0].parts == 0        # 16 pairs of 3 pages: 3 parts max
    assert check_plan([4097, 4096] * 8, 8, 148, True)[0].parts == 1  # 4096 / 4095 keys: 256 pages
    assert check_plan([4097, 4000] * 8, 8, 148, True)[0].parts == 0  # 256 / 250 pages
    assert check_plan([4097] * 16, 8, 148, True, static_pct=90)[0].parts == 0
    rng = random.Random(7)
    for _ in range(200):
        B, nkv = rng.randint(1, 20), rng.choice([1, 2, 4, 8])
        L = rng.choice([1, 16, 17, 100, 4097, rng.randint(1, 50000)])
        check_plan([L] * B, nkv, rng.choice([37, 100, 148, 296]), rng.random() < 0.5,
                   skew=rng.random() < 0.5)
