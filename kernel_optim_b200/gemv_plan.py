"""Host mirror of the work split of the skinny-GEMM kernel (csrc/gemv.cu).

kopt_gemv_plan_make and gemv_kernel divide a projection between CTAs as follows; this module
restates that arithmetic so the split can be inspected and property-tested without a GPU. The
lines of csrc/gemv.cu restated here (a change there must be mirrored here):

* gemv_split       <- kopt_gemv_plan_make, gemv.cu:897-930 (tiles, units, per, grid)
* GemvSplit.run    <- gemv_kernel, gemv.cu:312-314 (a CTA's unit run)
* write_slot       <- gemv.cu:529-542 (a split segment's partial slot and the tile counter)
* holders, read_slot <- gemv.cu:548-590 (the merge's CTAs kfirst .. klast and kfirst_seg)

* the weight is cut into tiles of 128 rows (SWIGLU: 64 gate rows and their 64 up rows, so
  N / 64 tiles; otherwise ceil(N / 128)) and K into ceil(K / 64) chunks; a unit is one (tile,
  chunk), numbered tile-major: u = tile * nchunks + chunk;
* with C requested CTAs (by default the SM count times the resident CTAs per SM, one with this
  kernel's shared memory; at most one per unit), every CTA takes
  per = ceil(units / C) consecutive units; the grid is ceil(units / per) CTAs;
* CTA c's run [c per, min((c+1) per, units)) falls into segments, one per tile it touches; a
  segment that is not a whole tile writes its fp32 partial to workspace slot 2c (the CTA's first
  segment) or 2c + 1 (its last one);
* the CTAs holding tile t are kfirst = t nchunks // per .. klast = (t nchunks + nchunks - 1) // per;
  they count themselves on the tile's counter, and the one that arrives last adds the partials of
  CTAs kfirst .. klast in that order, CTA k's being slot 2k if k's run starts inside tile t (its
  first segment) and 2k + 1 otherwise.
"""

from __future__ import annotations

from dataclasses import dataclass

ROWS = 128      # weight rows per tile: the MMA's M
BK = 64         # k per chunk: one ring stage


@dataclass
class GemvSplit:
    tiles: int
    nchunks: int
    per: int
    grid: int

    @property
    def units(self) -> int:
        return self.tiles * self.nchunks

    def run(self, c: int) -> tuple[int, int]:
        """Units [u0, u1) of CTA c."""
        u0 = c * self.per
        return u0, min(u0 + self.per, self.units)

    def segments(self, c: int):
        """CTA c's segments in order: (tile, chunk a, chunk b, first_seg, whole)."""
        u0, u1 = self.run(c)
        u, out = u0, []
        while u < u1:
            tile, a = divmod(u, self.nchunks)
            b = min(self.nchunks, a + (u1 - u))
            out.append((tile, a, b, u == u0, a == 0 and b == self.nchunks))
            u += b - a
        return out

    def write_slot(self, c: int, first_seg: bool) -> int:
        """Partial slot a split segment of CTA c writes (gemv_kernel)."""
        return 2 * c + (0 if first_seg else 1)

    def holders(self, tile: int) -> range:
        """CTAs whose runs touch the tile, in the order the merge adds them."""
        tu0 = tile * self.nchunks
        return range(tu0 // self.per, (tu0 + self.nchunks - 1) // self.per + 1)

    def read_slot(self, k: int, tile: int) -> int:
        """Slot the merge of the tile reads for CTA k (gemv_kernel's kfirst_seg rule)."""
        return 2 * k + (0 if k * self.per >= tile * self.nchunks else 1)


def gemv_split(N: int, K: int, swiglu: bool = False, ctas: int = 148) -> GemvSplit:
    """kopt_gemv_plan_make's split for N outputs, K inputs and `ctas` CTAs asked for."""
    tiles = N // 64 if swiglu else (N + ROWS - 1) // ROWS
    nchunks = (K + BK - 1) // BK
    units = tiles * nchunks
    c = min(ctas, units)
    per = (units + c - 1) // c
    return GemvSplit(tiles, nchunks, per, (units + per - 1) // per)
