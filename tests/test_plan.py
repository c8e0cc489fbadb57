"""CPU: invariants of the device-side work split (mirrored in kernel_optim_b200/plan.py)."""

import random
from collections import defaultdict

import pytest

from kernel_optim_b200.plan import CHUNK_TOKENS, PAGE, chunks, max_units, schedule


def check_plan(lengths, nkv, fused, max_len=None):
    cs = chunks(lengths, nkv, fused)
    B = len(lengths)
    assert [c.g for c in cs] == list(range(len(cs)))
    assert len(cs) <= max_units(B, nkv, max_len or max(lengths))
    by_pair = defaultdict(list)
    for c in cs:
        by_pair[c.q].append(c)
    assert set(by_pair) == set(range(B * nkv)), "a (sequence, kv head) pair has no chunk"
    for q, lst in by_pair.items():
        b = q // nkv
        ls = lengths[b] - 1 if fused else lengths[b]
        pos = 0
        for c in lst:   # keys [0, Ls) covered exactly once, in order, on page boundaries
            assert c.t0 == pos and c.t0 % PAGE == 0 and c.t1 - c.t0 <= CHUNK_TOKENS
            pos = c.t1
        assert pos == ls
        assert [c.g for c in lst] == list(range(lst[0].c0, lst[0].c0 + lst[0].n))
        assert [c.last for c in lst] == [False] * (len(lst) - 1) + [True]
    return cs


@pytest.mark.parametrize("fused", [False, True])
def test_baseline_configs(fused):
    c2 = check_plan([4097] * 16, 8, fused)
    assert len(c2) == 16 * 8 * (8 if fused else 9)   # 4096 or 4097 streamed keys per pair
    check_plan([131072] * 4, 8, fused)
    check_plan([1] * 3, 8, fused)              # only the appended key
    check_plan([5, 130, 77], 8, fused, 136)


def test_random_lengths_and_heads():
    rng = random.Random(0)
    for _ in range(300):
        B = rng.randint(1, 40)
        nkv = rng.choice([1, 2, 4, 8])
        lengths = [rng.choice([1, 2, 15, 16, 17, 512, 513, rng.randint(1, 20000)]) for _ in range(B)]
        check_plan(lengths, nkv, rng.random() < 0.5)


def test_dynamic_claims_take_every_chunk_once():
    rng = random.Random(1)
    for _ in range(50):
        n = rng.randint(1, 3000)
        grid = rng.choice([1, 7, 148, 296])
        speeds = [rng.uniform(0.7, 1.3) for _ in range(grid)]
        taken = schedule(n, grid, speeds)
        flat = sorted(g for t in taken for g in t)
        assert flat == list(range(n))
