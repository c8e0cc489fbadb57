"""CPU: invariants of the skinny-GEMM work split (mirrored in kernel_optim_b200/gemv_plan.py)."""

import random
from collections import defaultdict

import pytest

from kernel_optim_b200.gemv_plan import gemv_split


def check(sp):
    seen = defaultdict(list)           # (tile, chunk) -> CTA
    written = {}                        # slot -> (cta, tile)
    per_tile = defaultdict(list)        # tile -> [(cta, whole)]
    for c in range(sp.grid):
        u0, u1 = sp.run(c)
        assert u1 > u0, "a CTA without work"
        segs = sp.segments(c)
        assert 1 <= len(segs)
        for tile, a, b, first, whole in segs:
            for ch in range(a, b):
                seen[(tile, ch)].append(c)
            per_tile[tile].append((c, whole))
            if not whole:
                slot = sp.write_slot(c, first)
                assert slot not in written, "two segments share a partial slot"
                written[slot] = (c, tile)
        # only a CTA's first and last segments can be partial
        for tile, a, b, first, whole in segs[1:-1]:
            assert whole
    assert len(seen) == sp.units and all(len(v) == 1 for v in seen.values()), "unit not covered once"
    for tile in range(sp.tiles):
        holders = list(sp.holders(tile))
        assert [c for c, _ in per_tile[tile]] == holders, "merge order differs from the CTAs' order"
        if len(holders) == 1:
            assert per_tile[tile][0][1], "a tile held by one CTA must be whole"
            continue
        assert not any(w for _, w in per_tile[tile])
        for k in holders:   # the merger reads exactly the slots the holders wrote for this tile
            slot = sp.read_slot(k, tile)
            assert written.get(slot) == (k, tile)
    assert not written or max(written) < 2 * sp.grid, "partial slot past the two per CTA"


@pytest.mark.parametrize("N,K,swiglu", [(6144, 2560, False), (2560, 4096, False), (9728, 2560, True),
                                        (2560, 9728, False), (151936, 2560, False), (3072, 2560, False)])
def test_qwen3_4b_projections(N, K, swiglu):
    sp = gemv_split(N, K, swiglu)
    check(sp)
    assert sp.grid <= 148


def test_random_shapes_and_grids():
    rng = random.Random(0)
    for _ in range(400):
        swiglu = rng.random() < 0.3
        N = 64 * rng.randint(1, 200) if swiglu else 16 * rng.randint(1, 800)
        K = 8 * rng.randint(1, 1500)
        check(gemv_split(N, K, swiglu, ctas=rng.choice([1, 2, 3, 7, 37, 148, 296, 1216])))
