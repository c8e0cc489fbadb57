"""Host side of the speculative decode path (the caller of the T > 1 verify attention).

The reference's engine can speculate (engine/engine.py:35-43, 48-90, 451-508; off unless
ENGINE_SPEC=1): each sequence drafts K tokens by looking up its latest n-gram in its own history
(prompt and generated tokens, longest n-gram first: 3, 2, 1), one verify forward runs the last
accepted token and the K drafts as T = K + 1 query rows per sequence at positions pos[b] ..
pos[b] + K, and the longest prefix of drafts that equals the verify forward's own greedy picks is
accepted, plus the pick after it. Every WINDOW verify steps the slowest sequence's advance per
step is compared with the break-even (verify step + host time over one-token step); below it the
engine finishes on the one-token path. Sequences advance at their own rates; tokens are handed to
the caller only as far as every sequence has them.

This module holds that logic without the GPU: ``Lookup`` (the n-gram index), ``draft_len`` and
``speculate``, which drives a verify callback and yields the emitted token lists, so the host logic
is testable on the CPU against a model stand-in.
"""

from __future__ import annotations

from typing import Callable, Iterator

NGRAMS = (3, 2, 1)      # draft lookup, longest match first (engine.py:35)
WINDOW = 8              # verify steps per break-even check (engine.py:36)
HOST_MS = 0.2           # host round trip per verify step, added to its time (engine.py:37)


def draft_len(B: int) -> int:
    """Draft tokens per sequence for a batch of B (engine.py:48-57): the verify rows B (K + 1)
    stay small."""
    if B <= 4:
        return 6
    if B <= 16:
        return 4
    if B <= 32:
        return 2
    return 0


class Lookup:
    """Incremental n-gram index over one sequence: n-gram -> index of its latest continuation."""

    __slots__ = ("seq", "maps")

    def __init__(self, seq: list[int]):
        self.seq = list(seq)
        self.maps: dict[int, dict[tuple, int]] = {n: {} for n in NGRAMS}
        for i in range(1, len(self.seq)):
            self._index(i)

    def _index(self, i: int) -> None:
        """Record that the n-grams ending at seq[i - 1] are continued at index i."""
        s = self.seq
        for n in NGRAMS:
            if i >= n:
                self.maps[n][tuple(s[i - n:i])] = i

    def append(self, toks) -> None:
        for t in toks:
            self.seq.append(int(t))
            self._index(len(self.seq) - 1)

    def draft(self, K: int) -> list[int]:
        """K tokens continuing the sequence's latest n-gram where it last occurred (a continuation
        that runs into the draft itself repeats the draft: loops); no match: the last token K
        times."""
        s = self.seq
        L = len(s)
        for n in NGRAMS:
            if L < n:
                continue
            j = self.maps[n].get(tuple(s[L - n:]))
            if j is None:
                continue
            out: list[int] = []
            for k in range(K):
                idx = j + k
                out.append(s[idx] if idx < L else out[idx - L])
            return out
        return [s[-1]] * K


def accept(drafts: list[int], picks: list[int]) -> list[int]:
    """Tokens a verify row accepts: the picks while each draft equals the pick before it, and the
    first pick that disagrees (always at least one token)."""
    K = len(drafts)
    a = 0
    while a < K and drafts[a] == picks[a]:
        a += 1
    return list(picks[:a + 1])


def speculate(prompts: list[list[int]], first: list[int], N: int, K: int,
              verify: Callable[[list[list[int]], list[int]], list[list[int]]],
              breakeven: float, window: int = WINDOW):
    """Generator: drive the verify forward until every sequence has N tokens or speculation stops
    paying; yields each emitted step (one token per sequence) and returns the per-sequence token
    lists (``outs``, first token included) for the one-token path to continue from.

    ``verify(rows, positions)`` runs rows[b] = [last accepted token] + K drafts at positions
    positions[b] .. positions[b] + K and returns each row's K + 1 greedy picks. A sequence that
    already has N tokens keeps its position and its picks are ignored (engine.py:480-481)."""
    B = len(prompts)
    S = len(prompts[0])
    look = [Lookup(list(p) + [first[b]]) for b, p in enumerate(prompts)]
    outs = [[int(t)] for t in first]
    emitted = 1
    steps = 0
    window_min = 1
    while emitted < N:
        rows = [[lk.seq[-1]] + lk.draft(K) for lk in look]
        positions = [len(lk.seq) - 1 for lk in look]
        picks = verify(rows, positions)
        steps += 1
        for b in range(B):
            if len(outs[b]) >= N:
                continue
            new = accept(rows[b][1:], picks[b])
            outs[b].extend(new)
            look[b].append(new)
        ready = min(len(o) for o in outs)
        while emitted < min(ready, N):
            yield [o[emitted] for o in outs]
            emitted += 1
        if steps % window == 0 and emitted < N:
            advance = (ready - window_min) / window
            window_min = ready
            if advance < breakeven:
                break
    assert all(len(lk.seq) == S + len(o) for lk, o in zip(look, outs))
    return outs


def drain_one_token(outs: list[list[int]], N: int, steps: Iterator[list[int]]):
    """Generator for the one-token path after speculation: each item of ``steps`` is one token per
    sequence, appended to its list; yields the steps every sequence has, from the first one not
    yet emitted."""
    emitted = min(min(len(o) for o in outs), N)
    for toks in steps:
        for o, t in zip(outs, toks):
            o.append(int(t))
        ready = min(N, min(len(o) for o in outs))
        while emitted < ready:
            yield [o[emitted] for o in outs]
            emitted += 1
        if emitted >= N:
            return
