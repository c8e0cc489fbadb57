"""Host mirror of the device-side work split of the decode-attention kernel.

The kernel (csrc/decode_attn.cu: compute_plan, chunk_range, chunk_of, unit_at, claim_chunk) decides
on the device, at every call, how the keys are divided between CTAs, from the live lengths
pos[b] + T. This module restates that arithmetic so the split can be inspected and property-tested
without a GPU:

* sequence b streams Ls_b keys from the cache (L_b, or L_b - 1 when the fused prologue appends the
  last key itself) = max(1, ceil(Ls_b / 16)) pages for each kv head;
* the pages of all pairs (b, kvh), pair index q = b * nkv + kvh, are laid end to end: T pages;
* with P = floor(pct T / 100) (0 when P < grid), chunk k < grid is CTA k's static piece
  [k P / grid, (k+1) P / grid); chunk k >= grid is the dynamic chunk [P + 32 (k - grid), ...)
  clipped to T, claimed at run time;
* with overlapped launches (skew) and long enough pieces, the last LATE_CTAS pieces are shorter by
  LATE_PAGES (the last CTA's most) and the first grid - LATE_CTAS pieces share the difference;
* a unit is a chunk's intersection with one pair; its partial result goes to workspace slot k + q,
  and the last of the pair's n units to finish merges slots c + q for c in c0 .. c0 + n - 1;
* when every pair has the same page count np, there are no more pairs than CTAs and the whole line
  is static, each pair is cut into k = min(grid // pairs, np) parts of its own instead (piece c =
  part c % k of pair c // k, [floor(i np / k), floor((i + 1) np / k)) within it), provided
  pairs * k >= 0.8 grid; the CTAs past pairs * k get nothing and the late-start allowance is off;
  with more pairs than CTAs, piece c is pairs [c m, (c + 1) m) instead, m = ceil(pairs / grid)
  when it divides the pair count and pairs / m >= 0.8 grid (no pair split, nothing merged).
"""

from __future__ import annotations

from dataclasses import dataclass

PAGE = 16
CHUNK_PAGES = 32
STATIC_PCT = 100
LATE_CTAS = 4
LATE_PAGES = (24, 12, 6, 6)     # taken off the pieces of the last, second-to-last, ... CTA


@dataclass(frozen=True)
class Unit:
    chunk: int
    b: int
    kvh: int
    q: int
    t0: int      # first key streamed from the cache
    t1: int      # one past the last key streamed from the cache
    c0: int      # first chunk holding the pair
    n: int       # chunks holding the pair
    last: bool   # this unit ends the pair (owns the appended key in the fused path)

    @property
    def slot(self) -> int:
        return self.chunk + self.q


@dataclass(frozen=True)
class Plan:
    npages: list
    pstart: list
    total_pages: int
    static_pages: int
    total_chunks: int
    grid: int
    late: bool = False
    parts: int = 0       # > 0: pair-aligned pieces, `parts` per pair of npg_eq pages
    npg_eq: int = 0
    group: int = 0       # > 0: pieces of `group` whole pairs of npg_eq pages

    def _late_front(self) -> int:
        q = self.static_pages // self.grid
        return self.static_pages - (LATE_CTAS * q - sum(LATE_PAGES))

    def chunk_range(self, k: int):
        G, P = self.grid, self.static_pages
        if self.parts:
            q, i = divmod(k, self.parts)
            np_ = self.npg_eq
            if q * np_ >= self.total_pages:
                return self.total_pages, self.total_pages
            return q * np_ + i * np_ // self.parts, q * np_ + (i + 1) * np_ // self.parts
        if self.group:
            w = self.group * self.npg_eq
            return min(k * w, self.total_pages), min((k + 1) * w, self.total_pages)
        if k < G and self.late:
            G4, F, q = G - LATE_CTAS, self._late_front(), P // G
            if k < G4:
                return k * F // G4, (k + 1) * F // G4
            x = F + sum(q - LATE_PAGES[LATE_CTAS - 1 - j] for j in range(k - G4))
            return x, x + q - LATE_PAGES[LATE_CTAS - 1 - (k - G4)]
        if k < G:
            return k * P // G, (k + 1) * P // G
        x0 = P + (k - G) * CHUNK_PAGES
        return x0, min(x0 + CHUNK_PAGES, self.total_pages)

    def chunk_of(self, y: int) -> int:
        G, P = self.grid, self.static_pages
        if self.parts:
            q, off = divmod(y, self.npg_eq)
            return q * self.parts + ((off + 1) * self.parts - 1) // self.npg_eq
        if self.group:
            return y // (self.npg_eq * self.group)
        if y < P and self.late:
            G4, F, q = G - LATE_CTAS, self._late_front(), P // G
            if y < F:
                return ((y + 1) * G4 - 1) // F
            x, i = F, 0
            while i < LATE_CTAS - 1 and x + q - LATE_PAGES[LATE_CTAS - 1 - i] <= y:
                x += q - LATE_PAGES[LATE_CTAS - 1 - i]
                i += 1
            return G4 + i
        return ((y + 1) * G - 1) // P if y < P else G + (y - P) // CHUNK_PAGES


def plan(lengths, nkv: int, grid: int, fused: bool, static_pct: int = STATIC_PCT,
         skew: bool = False) -> Plan:
    """skew: launched to overlap the previous kernel (KOPT_PLAN_OVERLAP_PREV)."""
    npages = [max(1, -(-((L - 1) if fused else L) // PAGE)) for L in lengths]
    pstart = [0]
    for n in npages:
        pstart.append(pstart[-1] + n * nkv)
    T = pstart[-1]
    P = T * static_pct // 100
    if P < grid:
        P = 0
    late = skew and grid > 2 * LATE_CTAS and P // grid >= 4 * LATE_PAGES[0]
    parts, group, pairs = 0, 0, len(lengths) * nkv
    if min(npages) == max(npages) and P == T:
        if pairs <= grid:
            k = min(grid // pairs, npages[0])
            if 5 * pairs * k >= 4 * grid:
                parts, late = k, False
        else:
            m = -(-pairs // grid)
            if pairs % m == 0 and 5 * (pairs // m) >= 4 * grid:
                group, late = m, False
    return Plan(npages, pstart, T, P, grid + -(-(T - P) // CHUNK_PAGES), grid, late, parts,
                npages[0], group)


def units_of_chunk(pl: Plan, lengths, nkv: int, fused: bool, k: int) -> list[Unit]:
    x, x1 = pl.chunk_range(k)
    out = []
    while x < x1:
        b = max(i for i in range(len(lengths)) if pl.pstart[i] <= x)
        np_ = pl.npages[b]
        kvh, pg = divmod(x - pl.pstart[b], np_)
        pair0 = pl.pstart[b] + kvh * np_
        pair1 = pair0 + np_
        ux1 = min(x1, pair1)
        ls = lengths[b] - 1 if fused else lengths[b]
        t0 = pg * PAGE
        c0 = pl.chunk_of(pair0)
        out.append(Unit(k, b, kvh, b * nkv + kvh, t0, max(t0, min((ux1 - pair0) * PAGE, ls)),
                        c0, pl.chunk_of(pair1 - 1) - c0 + 1, ux1 == pair1))
        x = ux1
    return out


def all_units(lengths, nkv: int, grid: int, fused: bool, static_pct: int = STATIC_PCT,
              skew: bool = False) -> list[Unit]:
    pl = plan(lengths, nkv, grid, fused, static_pct, skew)
    return [u for k in range(pl.total_chunks) for u in units_of_chunk(pl, lengths, nkv, fused, k)]


def max_units(B: int, nkv: int, max_len: int, grid: int) -> int:
    """Workspace slots of the host plan: grid + ceil(T_max / 32) + B * nkv."""
    pages = B * nkv * (-(-max_len // PAGE))
    return grid + -(-pages // CHUNK_PAGES) + B * nkv


def schedule(n_chunks: int, grid: int, speeds) -> list[list[int]]:
    """Simulate the claiming: CTA c starts with piece c and claims one dynamic chunk ahead; a CTA
    that finishes a chunk starts its claimed one and claims the next. speeds[c] is CTA c's time
    per chunk. Returns the chunks each CTA processed."""
    import heapq
    nxt = grid
    taken = [[c] for c in range(grid)]
    heap = [(speeds[c], c) for c in range(grid)]
    heapq.heapify(heap)
    while heap:
        t, c = heapq.heappop(heap)
        if nxt < n_chunks:
            taken[c].append(nxt)
            nxt += 1
            heapq.heappush(heap, (t + speeds[c], c))
    return taken
