"""Host mirror of the device-side work split of the decode-attention kernel.

The kernel (csrc/decode_attn.cu, compute_plan / chunk_unit / claim_chunk) decides on the device,
at every call, how the keys are divided between CTAs, from the live lengths pos[b] + T. This module
restates that arithmetic in Python so the split can be inspected and property-tested without a GPU:

* sequence b streams Ls_b keys from the cache (L_b, or L_b - 1 when the fused prologue appends the
  last key itself) = max(1, ceil(Ls_b / 16)) pages for each kv head;
* the pages of each pair (b, kvh), pair index q = b * nkv + kvh, are cut into chunks of 32 pages
  (512 keys); chunks are numbered pair after pair, b-major;
* CTA c processes chunk c first, then chunks it claims from a global counter (grid + 0, 1, 2 ...);
  which CTA gets which dynamic chunk depends on timing, not on this plan;
* chunk g's partial result goes to workspace slot g; the last of the pair's n chunks to finish
  merges slots c0 .. c0 + n - 1 (a pair with a single chunk writes its output directly).
"""

from __future__ import annotations

from dataclasses import dataclass

PAGE = 16
CHUNK_PAGES = 32
CHUNK_TOKENS = PAGE * CHUNK_PAGES


@dataclass(frozen=True)
class Chunk:
    g: int       # chunk index = workspace slot
    b: int
    kvh: int
    q: int
    t0: int      # first key streamed from the cache
    t1: int      # one past the last key streamed from the cache
    c0: int      # first chunk of the pair
    n: int       # chunks of the pair
    last: bool   # last chunk of the pair (owns the appended key in the fused path)


def chunks(lengths, nkv: int, fused: bool) -> list[Chunk]:
    """Every chunk of one call, in index order."""
    out = []
    g = 0
    for b, L in enumerate(lengths):
        ls = L - 1 if fused else L
        np_ = max(1, -(-ls // PAGE))
        nch = -(-np_ // CHUNK_PAGES)
        for kvh in range(nkv):
            c0 = g
            for j in range(nch):
                t0 = j * CHUNK_TOKENS
                t1 = max(t0, min((j + 1) * CHUNK_TOKENS, ls))
                out.append(Chunk(g, b, kvh, b * nkv + kvh, t0, t1, c0, nch, j == nch - 1))
                g += 1
    return out


def max_units(B: int, nkv: int, max_len: int) -> int:
    """Workspace slots a plan for caches of up to max_len keys needs (the host plan's max_units)."""
    pages = -(-max_len // PAGE)
    return B * nkv * (-(-pages // CHUNK_PAGES))


def schedule(n_chunks: int, grid: int, speeds) -> list[list[int]]:
    """Simulate the claiming: CTA c starts with chunk c; whenever a CTA starts a chunk it claims
    the next one (one ahead). `speeds[c]` is CTA c's time per chunk. Returns the chunks each CTA
    processed, to check that every chunk is taken exactly once."""
    import heapq
    nxt = grid
    taken = [[] for _ in range(grid)]
    heap = []
    for c in range(min(grid, n_chunks)):
        taken[c].append(c)
        heapq.heappush(heap, (speeds[c], c))
    while heap:
        t, c = heapq.heappop(heap)
        if nxt < n_chunks:
            taken[c].append(nxt)
            nxt += 1
            heapq.heappush(heap, (t + speeds[c], c))
    return taken
