// Split-K GQA decode attention for Qwen3-4B on B200 (sm_100a), behind the C ABI in include/kopt.h.
//
// What the reference does (GodRishUniverse/kernel_optim, engine/kernels/fused.py):
//   _qk_norm_rope_kernel (fused.py:54-96): per (token, head) RMSNorm(128) -> weight -> RoPE with the
//     cast order bf16(w * bf16(x * rstd)), then bf16(bf16(xn*cos) + bf16(rot*sin)); q to q_out,
//     k/v into the cache slot pos[b] + t.
//   _decode_attn_kernel (fused.py:138-185): grid (B*NKV, NSPLIT); each program reads the 4 query
//     rows of a GQA group once per K/V tile, online softmax in fp32, stores un-normalised partials.
//   _decode_combine_kernel (fused.py:188-201): LSE merge of the splits, bf16 output.
//
// How this file does it on B200:
//   * One wave of one CTA per SM, balanced dynamically. Every CTA plans the call on the device from
//     the live lengths pos[b] + 1 (never from the capacity, unlike fused.py:211-214): the 16-token
//     pages of every (sequence, kv head) pair are laid end to end on one line. The first
//     static_pct of the line is cut into one equal piece per CTA; the rest into 32-page chunks that
//     CTAs claim from a global counter, one ahead, once their piece is done. SMs that the memory system serves
//     faster simply take more chunks. A pair cut by piece or chunk boundaries is split into units
//     whose partial results are merged by the last unit to finish. The last CTA to finish resets
//     the counter; no CTA ever waits for another.
//   * 8 warps; tile i of a unit is 128 keys = 8 pages and warp w owns page w of every tile. Each
//     warp streams its own pages with tiled TMA (cp.async.bulk.tensor, 128-byte swizzle, no
//     multicast) into a private 3-deep ring of shared-memory slots, each slot guarded by an
//     mbarrier; the refill of a slot is issued as soon as the warp has consumed it, two tiles ahead
//     and across unit boundaries. A page of one kv head arrives as two 16 x 64 boxes (dims 0-63,
//     64-127) for K and two for V. No warp waits on another warp between unit boundaries.
//   * Each warp consumes its page with mma.sync m16n8k16 (bf16 in, fp32
//     accumulate): S = Q K^T with the 4 query rows of the group in the 16-row A tile, an fp32
//     online softmax in the exp2 domain on the accumulator fragments (4-lane shuffles), then
//     O += P V with P rounded to bf16 as the reference does (fused.py:179). Swizzled ldmatrix loads
//     are bank-conflict free. The 12 idle rows of the A tile cost nothing: the path is HBM-bound.
//   * The fused variant computes the QK-norm/RoPE prologue in the CTA, appends the new token's K/V
//     to the cache from the CTA that owns position pos[b] and folds that token in from shared
//     memory (it is never read back from HBM).
//   * Splits of one (sequence, kv head) are merged by the last CTA to finish (atomic counter, no
//     waiting on other CTAs), so the reference's separate combine launch disappears.
//   * Every mbarrier wait is bounded in time; on expiry the kernel records KOPT_DEV_ERR_TIMEOUT,
//     stops issuing copies, waits (bounded) for copies in flight and runs to completion.
//
// The decode step's projections and row kernels are in gemv.cu; helpers both use, in common.cuh.

#include <mutex>

#include "common.cuh"

namespace kopt {

constexpr int kD = 128;                 // head dim
constexpr int kHalf = 64;               // dims per TMA box (128-byte rows for the 128B swizzle)
constexpr int kGroup = 4;               // query heads per kv head
constexpr int kPage = 16;               // tokens per page (and per consumer warp per tile)
constexpr int kNW = 8;                  // consumer warps
constexpr int kTile = kPage * kNW;      // tokens per pipeline stage
constexpr int kStages = 3;
constexpr int kThreads = kNW * 32;
constexpr int kMaxB = 256;
constexpr int kMaxRanks = KOPT_MAX_RANKS;   // fused gather: ranks of one node
constexpr int kBoxBytes = kPage * kHalf * 2;   // 2 KiB: one TMA box
constexpr int kChunkPages = 32;                // dynamic chunk: 512 keys of the page line
constexpr int kLateCtas = 4;                   // CTAs whose static piece is shortened (late start)
constexpr int kLateMax = 24;                   // pages taken off the last CTA's piece
constexpr int kMaxPend = 8;                    // partial units a CTA holds before releasing them
constexpr int kDefaultStaticPct = 100;         // share of the page line split statically
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1.0e30f;     // running-max seed (finite, as fused.py:164)


struct Params {
  CUtensorMap tmk;       // K cache: paged {128, pages*nkv*16} or contiguous {128, cap, nkv, B}
  CUtensorMap tmv;       // V cache, same geometry
  const bf16* q;         // [B*T, nq*128] (unfused)
  const bf16* qkv;       // [B, (nq + 2 nkv) * 128] (fused)
  const bf16* qw;        // q_norm weight [128]
  const bf16* kw;        // k_norm weight [128]
  const bf16* cos;       // [rope_len, 128]
  const bf16* sin;
  bf16* q_out;           // optional roped q [B, nq*128]
  bf16* kc;              // cache K (layer base or page pool), for the appended row
  bf16* vc;
  long long sb, sh;      // contiguous strides (elements)
  const int* bt;         // block table or nullptr
  const int* pos;        // [B]
  bf16* out;             // [B*T, nq*128] (when world == 0)
  // fused all-gather (world > 0): row b, head h of this rank go to out_peer[w] + b*out_row +
  // out_col + h*128 on every rank w; then flag_peer[w][rank] = epoch + 1
  bf16* out_peer[kMaxRanks];
  int* flag_peer[kMaxRanks];
  int* epoch;            // this rank's call counter, advanced by the last CTA
  long long out_row;     // elements per output row
  unsigned long long wait_ns;   // bound of the gather's flag wait
  int out_col;           // this rank's first column
  int rank, world;       // world == 0: no gather, write `out`
  float* ws_o;           // [max_units, 4, 128]
  float2* ws_ml;         // [max_units, 4]
  int* ws_cnt;           // [B * nkv]
  int* ws_err;           // error word; ws_err[1] = next dynamic chunk, ws_err[2] = CTAs done
  int bt_stride, num_pages, cap, rope_len;
  int B, T, nkv;
  int static_pct;        // share of the page line cut into one static piece per CTA
  int late_skew;         // launched to overlap the previous kernel: the last CTAs start late
  int nsplit, tblocks;   // verify kernel (T > 1): key splits, blocks of 4 query tokens
  float scale_log2, eps;
};

// One stage: [page 0..7][half 0..1][16 tokens x 64 dims] for K and for V. Every 2 KiB box starts
// on a 1 KiB boundary, as the 128-byte swizzle pattern (16-byte chunk ^= row % 8) requires.
struct __align__(1024) Smem {
  bf16 k[kStages][kNW][2][kPage * kHalf];
  bf16 v[kStages][kNW][2][kPage * kHalf];
  alignas(16) bf16 q[kGroup][kD];       // roped q rows of the current unit (the reference's q)
  float o[kNW][kGroup][kD + 4];         // unit epilogue: per-warp partial outputs (padded rows)
  alignas(16) bf16 rows[8][kD];         // next unit's prologue inputs, staged by cp.async:
                                        // q heads 0-3, k head, v head, cos row, sin row
  alignas(16) bf16 wq[kD];              // q_norm weight
  alignas(16) bf16 wk[kD];              // k_norm weight
  float red_m[kNW][kGroup];
  float red_l[kNW][kGroup];
  bf16 knew[kD];
  bf16 vnew[kD];
  int pstart[kMaxB + 1];                // first page of pair (b, kv head 0) on the page line
  int npages[kMaxB];                    // pages streamed per (b, kv head)
  int lens[kMaxB];                      // keys attended by sequence b
  int ring[4];                          // the CTA's k-th claimed chunk in ring[k % 4] (-1: none)
  unsigned long long full[kStages][kNW];   // per-warp ring: slot filled by this warp's TMA
  int total_pages;
  int static_pages;                     // P: pages of the line split into one piece per CTA
  int total_chunks;                     // grid static pieces + dynamic chunks
  int late;                             // the last kLateCtas pieces are shortened (see chunk_range)
  int parts;                            // > 0: every pair has npg_eq pages and is cut into this
  int npg_eq;                           //   many pieces of its own (see compute_plan)
  int group;                            // > 0: pieces of `group` whole pairs of npg_eq pages
  volatile int nclaimed;                // ring entries 0 .. nclaimed-1 are valid
  int npend;                            // partial units written, not yet released
  int pend[kMaxPend][5];                // their (pair, first chunk, chunks, sequence, kv head)
  int nmerge;                           // pending entries whose pair this CTA merges
  int merge[kMaxPend];
  int unext[12];                        // the look-ahead unit, parked across the tile loop
  int have_next;
  int err_bits;                         // errors found before the wait (reported at the end)
  volatile int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack to align the base to 1 KiB
static_assert(kSmemBytes <= 227 * 1024, "shared memory above the 227 KiB per-CTA limit");

// ---------------------------------------------------------------- QK-norm + RoPE of one head
// One warp; lane owns dims 4*lane .. 4*lane+3. Follows fused.py:79-87 with the sum of squares in
// a fixed order (per lane ((x0^2 + x1^2) + x2^2) + x3^2, then xor-butterfly 16, 8, 4, 2, 1),
// rstd = 1 / sqrt(mean + eps) with IEEE sqrt and division, and no FMA contraction anywhere.
__device__ __forceinline__ void norm_rope_head(const bf16* __restrict__ src, const bf16* __restrict__ w,
                                               const bf16* __restrict__ cs, const bf16* __restrict__ sn,
                                               float eps, int lane, float y[4]) {
  const uint2 raw = *reinterpret_cast<const uint2*>(src + 4 * lane);
  const float2 x01 = bf2f(raw.x), x23 = bf2f(raw.y);
  const float x[4] = {x01.x, x01.y, x23.x, x23.y};
  float ss = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1])),
                                 __fmul_rn(x[2], x[2])),
                       __fmul_rn(x[3], x[3]));
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const float var = __fmul_rn(ss, 1.0f / kD);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  const uint2 wr = *reinterpret_cast<const uint2*>(w + 4 * lane);
  const float2 w01 = bf2f(wr.x), w23 = bf2f(wr.y);
  const float wv[4] = {w01.x, w01.y, w23.x, w23.y};
  const uint2 cr = *reinterpret_cast<const uint2*>(cs + 4 * lane);
  const uint2 sr = *reinterpret_cast<const uint2*>(sn + 4 * lane);
  const float2 c01 = bf2f(cr.x), c23 = bf2f(cr.y), s01 = bf2f(sr.x), s23 = bf2f(sr.y);
  const float cv[4] = {c01.x, c01.y, c23.x, c23.y};
  const float sv[4] = {s01.x, s01.y, s23.x, s23.y};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float xn = bf16r(__fmul_rn(wv[j], bf16r(__fmul_rn(x[j], rstd))));
    const float xr = __shfl_xor_sync(0xffffffffu, xn, 16);  // dim d +- 64
    const float rh = lane < 16 ? -xr : xr;                   // rotate_half
    y[j] = bf16r(__fadd_rn(bf16r(__fmul_rn(xn, cv[j])), bf16r(__fmul_rn(rh, sv[j]))));
  }
}

__device__ __forceinline__ void store4_bf16(bf16* dst, const float y[4]) {
  uint2 u;
  u.x = pack_bf16(y[0], y[1]);
  u.y = pack_bf16(y[2], y[3]);
  *reinterpret_cast<uint2*>(dst) = u;
}

// ---------------------------------------------------------------------------- device plan
__device__ __forceinline__ int ceil_div_i(int a, int b) { return (a + b - 1) / b; }

// Warp 0 lays out the page line from pos[]: sequence b streams Ls_b keys from the cache (all L_b
// keys, or L_b - 1 when the fused prologue appends the last one itself) = max(1, ceil(Ls_b/16))
// pages per kv head; pair (b, kvh) owns pages [pstart[b] + kvh * npages[b], + npages[b]).
// Chunks: k < grid is CTA k's static piece [k*piece, (k+1)*piece); k >= grid is dynamic chunk
// k - grid covering [grid*piece + (k-grid)*32, ...) up to the end of the line.
template <bool FUSED>
__device__ void compute_plan(const Params& p, Smem& s, int lane) {
  int err = 0;
  for (int b = lane; b < p.B; b += 32) {
    int L = p.pos[b] + p.T;
    if (L < 1 || L > p.cap) {
      err |= KOPT_DEV_ERR_LEN;
      L = L < 1 ? 1 : p.cap;
    }
    s.lens[b] = L;
    const int Ls = FUSED ? L - 1 : L;
    s.npages[b] = Ls > 0 ? ceil_div_i(Ls, kPage) : 1;
  }
  err = __reduce_or_sync(0xffffffffu, err);
  if (lane == 0) s.err_bits = err;
  __syncwarp();
  // do all sequences stream the same number of pages?
  int nmin = 1 << 30, nmax = 0;
  for (int b = lane; b < p.B; b += 32) {
    nmin = min(nmin, s.npages[b]);
    nmax = max(nmax, s.npages[b]);
  }
  nmin = __reduce_min_sync(0xffffffffu, nmin);
  nmax = __reduce_max_sync(0xffffffffu, nmax);
  int carry = 0;
  for (int base = 0; base < p.B; base += 32) {
    const int b = base + lane;
    const int n = b < p.B ? s.npages[b] * p.nkv : 0;
    int incl = n;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += t;
    }
    if (b < p.B) s.pstart[b + 1] = carry + incl;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    const int G = gridDim.x;
    int P = static_cast<int>(static_cast<long long>(carry) * p.static_pct / 100);
    if (P < G) P = 0;   // too few pages for one per CTA: everything is dynamic
    s.pstart[0] = 0;
    s.total_pages = carry;
    s.static_pages = P;
    s.total_chunks = G + ceil_div_i(carry - P, kChunkPages);
    s.late = p.late_skew && G > 2 * kLateCtas && P / G >= 4 * kLateMax;
    // Pairs of equal length, no more of them than CTAs: cut each pair into the same number k of
    // pieces (CTA c takes part c % k of pair c / k) instead of one line cut into G pieces. Every
    // CTA then holds one unit, with no unit boundary inside its piece (measured on c2: 48.4 ->
    // 45.6 us; c4, k = 4: 347 -> 318 us). Only when the CTAs so used are >= 80% of the grid, a
    // part has at least one page, and the whole line is split statically; the CTAs beyond
    // pairs * k (the last ones, which start last under programmatic launch) get no pages.
    // More pairs than CTAs, all of one length: pieces of m whole pairs instead (m the smallest
    // that fits the grid and divides the pair count), under the same 80% rule, so that no pair is
    // split and nothing is merged.
    s.parts = 0;
    s.group = 0;
    s.npg_eq = nmin;
    const int pairs = p.B * p.nkv;
    if (nmin == nmax && P == carry) {
      if (pairs <= G) {
        const int k = min(G / pairs, nmin);
        if (5 * pairs * k >= 4 * G) {
          s.parts = k;
          s.late = 0;
        }
      } else {
        const int m = ceil_div_i(pairs, G);
        if (pairs % m == 0 && 5 * (pairs / m) >= 4 * G) {
          s.group = m;
          s.late = 0;
        }
      }
    }
  }
}

// Chunk k's page range on the line: k < grid is CTA k's static piece [k P / G, (k+1) P / G) of the
// first P pages (P >= G, so no piece is empty, or P = 0); k >= grid is dynamic chunk k - grid, 32
// pages from P + 32 (k - grid), clipped to the end of the line.
// With programmatic dependent launch the last CTAs of the grid are placed last, on the SMs the
// previous kernel frees last, and start late (device timestamps: ~4.5, ~2.5, ~1-1.5 us for the
// last, second-to-last and next two on c2); their pieces are shorter by kLatePages and the other
// CTAs share the difference. Measured on c2: 48.9 -> 48.5 us per call.
__device__ __forceinline__ int late_pages(int r) { return r == 0 ? kLateMax : r == 1 ? kLateMax / 2 : kLateMax / 4; }
__device__ __forceinline__ int late_front(const Smem& s) {   // pages of the first G - 4 pieces
  const int q = s.static_pages / static_cast<int>(gridDim.x);
  int d = 0;
  for (int r = 0; r < kLateCtas; ++r) d += late_pages(r);
  return s.static_pages - (kLateCtas * q - d);
}
__device__ __forceinline__ void chunk_range(const Smem& s, int k, int& x0, int& x1) {
  const int G = gridDim.x;
  const long long P = s.static_pages;
  if (s.parts > 0) {   // part k % parts of pair k / parts, or nothing past the last pair's part
    const int q = k / s.parts, i = k - q * s.parts, np = s.npg_eq;
    if (static_cast<long long>(q) * np >= s.total_pages) {
      x0 = x1 = s.total_pages;
    } else {
      x0 = q * np + static_cast<int>(static_cast<long long>(i) * np / s.parts);
      x1 = q * np + static_cast<int>(static_cast<long long>(i + 1) * np / s.parts);
    }
    return;
  }
  if (s.group > 0) {   // pairs [k m, (k + 1) m), or nothing past the last pair
    const long long w = static_cast<long long>(s.group) * s.npg_eq;
    x0 = static_cast<int>(min(static_cast<long long>(k) * w, static_cast<long long>(s.total_pages)));
    x1 = static_cast<int>(min(static_cast<long long>(k + 1) * w, static_cast<long long>(s.total_pages)));
    return;
  }
  if (k < G && s.late) {
    const int G4 = G - kLateCtas, F = late_front(s), q = s.static_pages / G;
    if (k < G4) {
      x0 = static_cast<int>(static_cast<long long>(k) * F / G4);
      x1 = static_cast<int>(static_cast<long long>(k + 1) * F / G4);
    } else {   // piece G4 + i is q - late_pages(3 - i) long: the last CTA's is the shortest
      int x = F;
      for (int j = 0; j < k - G4; ++j) x += q - late_pages(kLateCtas - 1 - j);
      x0 = x;
      x1 = x + q - late_pages(kLateCtas - 1 - (k - G4));
    }
  } else if (k < G) {
    x0 = static_cast<int>(k * P / G);
    x1 = static_cast<int>((k + 1) * P / G);
  } else {
    x0 = static_cast<int>(P) + (k - G) * kChunkPages;
    x1 = min(x0 + kChunkPages, s.total_pages);
  }
}
// The chunk holding page y.
__device__ __forceinline__ int chunk_of(const Smem& s, int y) {
  const long long G = gridDim.x;
  const long long P = s.static_pages;
  if (s.parts > 0) {   // the part of its pair holding page y
    const int q = y / s.npg_eq, off = y - q * s.npg_eq;
    return q * s.parts +
           static_cast<int>((static_cast<long long>(off + 1) * s.parts - 1) / s.npg_eq);
  }
  if (s.group > 0) return y / (s.npg_eq * s.group);   // the piece of the pair holding page y
  if (y < P && s.late) {
    const int G4 = static_cast<int>(G) - kLateCtas, F = late_front(s);
    const int q = s.static_pages / static_cast<int>(G);
    if (y < F) return static_cast<int>((static_cast<long long>(y + 1) * G4 - 1) / F);
    int x = F, i = 0;
    while (i < kLateCtas - 1 && x + q - late_pages(kLateCtas - 1 - i) <= y) {
      x += q - late_pages(kLateCtas - 1 - i);
      ++i;
    }
    return G4 + i;
  }
  return y < P ? static_cast<int>(((y + 1) * G - 1) / P)
               : static_cast<int>(G) + (y - static_cast<int>(P)) / kChunkPages;
}

struct Unit {
  int b, kvh, q;      // sequence, kv head, pair index b * nkv + kvh
  int t0, t1;         // keys streamed from the cache: [t0, t1)
  int L;              // keys attended by the sequence
  int slot;           // workspace slot of this unit's partial result: chunk + q
  int c0, n;          // chunks holding the pair: c0 .. c0 + n - 1 (slots c + q)
  bool last;          // this unit ends the pair (owns the appended token in the fused path)
};

// The unit starting at page x of chunk k (x is advanced past it, up to x1).
template <bool FUSED>
__device__ __forceinline__ Unit unit_at(const Params& p, const Smem& s, int k, int& x, int x1) {
  int lo = 0, hi = p.B;   // largest b with pstart[b] <= x
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s.pstart[mid] <= x) lo = mid; else hi = mid;
  }
  Unit U;
  const int b = lo, np = s.npages[b];
  const int off = x - s.pstart[b];
  const int kvh = off / np, pg = off % np;
  const int pair0 = s.pstart[b] + kvh * np, pair1 = pair0 + np;
  const int ux1 = min(x1, pair1);
  U.b = b;
  U.kvh = kvh;
  U.q = b * p.nkv + kvh;
  U.L = s.lens[b];
  const int Ls = FUSED ? U.L - 1 : U.L;
  U.t0 = pg * kPage;
  U.t1 = max(U.t0, min((ux1 - pair0) * kPage, Ls));
  U.slot = k + U.q;
  U.c0 = chunk_of(s, pair0);
  U.n = chunk_of(s, pair1 - 1) - U.c0 + 1;
  U.last = ux1 == pair1;
  x = ux1;
  return U;
}

// Claim the next dynamic chunk (thread 0 only). claim_issue returns the raw counter value so that
// the atomic's latency is only paid where claim_chunk turns it into a chunk index (or -1).
__device__ __forceinline__ int claim_issue(const Params& p) { return atomicAdd(p.ws_err + 1, 1); }
__device__ __forceinline__ int claim_chunk(int raw, int total) {
  const int k = static_cast<int>(gridDim.x) + raw;
  return k < total ? k : -1;
}

// Element offset of token t's row of (b, kvh) in the cache, or -1 for a page id out of range.
__device__ __forceinline__ long long row_offset(const Params& p, int b, int kvh, int t) {
  if (p.bt != nullptr) {
    const int pid = p.bt[static_cast<long long>(b) * p.bt_stride + t / kPage];
    if (pid < 0 || pid >= p.num_pages) return -1;
    return ((static_cast<long long>(pid) * p.nkv + kvh) * kPage + (t % kPage)) * kD;
  }
  return static_cast<long long>(b) * p.sb + static_cast<long long>(kvh) * p.sh +
         static_cast<long long>(t) * kD;
}

// Fused gather, run by the last CTA of this rank once every CTA's rows are out: raise this rank's
// flag on every rank (release at system scope, after a system fence covering the rows that the
// other CTAs ordered before their counter increment), then wait until every rank's flag for this
// call is up here (acquire; bounded by p.wait_ns, KOPT_DEV_ERR_TIMEOUT on expiry), so that this
// kernel's completion means the whole gathered row block has landed in local memory. The peers are
// other GPUs running the same kernel; nothing here waits on work of this GPU. When the error word
// already holds KOPT_DEV_ERR_TIMEOUT (an earlier call through this workspace gave up, and the host
// has not read the word since), the peers are taken as gone and the call does not wait again: a
// decode step after a peer's failure costs one bound, not one per layer.
__device__ __noinline__ void gather_signal_and_wait(const Params& p) {
  __threadfence_system();
  const int e = *p.epoch + 1;
  for (int w = 0; w < p.world; ++w)
    asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p.flag_peer[w] + p.rank), "r"(e)
                 : "memory");
  const int* mine = p.flag_peer[p.rank];
  const bool gone = (*reinterpret_cast<volatile int*>(p.ws_err) & KOPT_DEV_ERR_TIMEOUT) != 0;
  const unsigned long long t0 = globaltimer();
  for (int w = 0; !gone && w < p.world; ++w) {
    while (true) {
      int f;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(f) : "l"(mine + w) : "memory");
      if (f >= e) break;
      if (globaltimer() - t0 > p.wait_ns) {
        atomicOr(p.ws_err, KOPT_DEV_ERR_TIMEOUT);
        break;
      }
    }
  }
  *p.epoch = e;
}

// Final output of (sequence b, query head h, dims d, d+1): to `out`, or, for the fused gather, to
// this rank's columns of every rank's gathered buffer (plain stores; peers over NVLink).
__device__ __forceinline__ void store_out(const Params& p, int b, int h, int d, float x, float y) {
  const uint32_t v = pack_bf16(x, y);
  const long long off = static_cast<long long>(b) * p.out_row + p.out_col + h * kD + d;
  if (p.world == 0) {
    *reinterpret_cast<uint32_t*>(p.out + off) = v;
  } else {
    for (int w = 0; w < p.world; ++w) *reinterpret_cast<uint32_t*>(p.out_peer[w] + off) = v;
  }
}

// ---------------------------------------------------------------- consumer: one 16-token page
// Fragment layout (m16n8k16): lane l holds rows r = l/4 and r + 8, columns 2(l%4), 2(l%4)+1.
// Only rows 0-3 (the GQA group's query heads) are live, i.e. lanes 0-15 in c0/c1; the rest of
// the tile is zero and its results are ignored.
struct WarpState {
  float o[16][2];   // O[row l/4][8j + 2(l%4) + {0,1}]
  float m;          // running max of row l/4 (exp2 domain)
  float l;          // this lane's partial softmax denominator
};

__device__ __forceinline__ void page_step(uint32_t kbase, uint32_t vbase, int ntok,
                                          const uint32_t (&qa)[8][2], float scale_log2,
                                          WarpState& st, int lane) {
  const int mi = lane >> 3, ri = lane & 7;
  // ---- S = Q K^T over this page's 16 tokens: two n-blocks (tokens 0-7, 8-15), 8 k-steps.
  float s0a[2] = {0.f, 0.f}, s0b[2] = {0.f, 0.f};
  float s1a[2] = {0.f, 0.f}, s1b[2] = {0.f, 0.f};
  {
    // ldmatrix.x4 matrices: (tokens 0-7, chunk c), (0-7, c+1), (8-15, c), (8-15, c+1)
    const int tok = 8 * (mi >> 1) + ri;
    const uint32_t row = kbase + tok * 128;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int h = ks >> 2, c = 2 * (ks & 3) + (mi & 1);
      uint32_t b00, b01, b10, b11;
      ldsm_x4(row + h * kBoxBytes + ((c ^ ri) << 4), b00, b01, b10, b11);
      if (ks & 1) {
        mma16816(s0b[0], s0b[1], qa[ks][0], qa[ks][1], b00, b01);
        mma16816(s1b[0], s1b[1], qa[ks][0], qa[ks][1], b10, b11);
      } else {
        mma16816(s0a[0], s0a[1], qa[ks][0], qa[ks][1], b00, b01);
        mma16816(s1a[0], s1a[1], qa[ks][0], qa[ks][1], b10, b11);
      }
    }
  }
  const int t0 = 2 * (lane & 3);
  float sv[4];
  sv[0] = (t0 < ntok) ? (s0a[0] + s0b[0]) * scale_log2 : -INFINITY;
  sv[1] = (t0 + 1 < ntok) ? (s0a[1] + s0b[1]) * scale_log2 : -INFINITY;
  sv[2] = (t0 + 8 < ntok) ? (s1a[0] + s1b[0]) * scale_log2 : -INFINITY;
  sv[3] = (t0 + 9 < ntok) ? (s1a[1] + s1b[1]) * scale_log2 : -INFINITY;
  // ---- online softmax of row lane/4 (4 lanes share a row)
  float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float m_new = fmaxf(st.m, mx);
  const float alpha = exp2f(st.m - m_new);
  float pr[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) pr[i] = exp2f(sv[i] - m_new);
  st.l = st.l * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
  st.m = m_new;
  if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      st.o[j][0] *= alpha;
      st.o[j][1] *= alpha;
    }
  }
  const uint32_t pa0 = pack_bf16(pr[0], pr[1]);   // P[row][t0, t0+1]      (k 0-7)
  const uint32_t pa2 = pack_bf16(pr[2], pr[3]);   // P[row][t0+8, t0+9]    (k 8-15)
  // ---- rows past the live tokens may hold anything: zero them so 0 * V stays 0
  if (ntok < kPage) {
    for (int idx = lane; idx < (kPage - ntok) * 16; idx += 32) {
      const int r = ntok + (idx >> 4), part = idx & 15;   // 16 chunks of 16 B per row (2 boxes)
      const uint32_t a = vbase + (part >> 3) * kBoxBytes + r * 128 + ((part & 7) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
    }
    __syncwarp();
  }
  // ---- O += P V: 16 n-blocks of 8 dims, k = the page's 16 tokens
  {
    // ldmatrix.x4.trans matrices: (tokens 0-7, chunk j), (8-15, j), (0-7, j+1), (8-15, j+1)
    const int tok = 8 * (mi & 1) + ri;
    const uint32_t row = vbase + tok * 128;
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const int c = j + (mi >> 1);
      uint32_t b0a, b1a, b0b, b1b;
      ldsm_x4_t(row + (c >> 3) * kBoxBytes + (((c & 7) ^ ri) << 4), b0a, b1a, b0b, b1b);
      mma16816(st.o[j][0], st.o[j][1], pa0, pa2, b0a, b1a);
      mma16816(st.o[j + 1][0], st.o[j + 1][1], pa0, pa2, b0b, b1b);
    }
  }
}

// The appended token of the fused path, folded into warp 0's state on CUDA cores.
__device__ __forceinline__ void inject_token(const Smem& s, float scale_log2, WarpState& st,
                                             int lane) {
  // s_r = q_r . k_new for the 4 rows; lane covers dims 4*lane .. 4*lane+3
  const uint2 kr = *reinterpret_cast<const uint2*>(&s.knew[4 * lane]);
  const float2 k01 = bf2f(kr.x), k23 = bf2f(kr.y);
  float dot[kGroup];
#pragma unroll
  for (int r = 0; r < kGroup; ++r) {
    const uint2 qr = *reinterpret_cast<const uint2*>(&s.q[r][4 * lane]);
    const float2 q01 = bf2f(qr.x), q23 = bf2f(qr.y);
    dot[r] = q01.x * k01.x + q01.y * k01.y + q23.x * k23.x + q23.y * k23.y;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
    for (int r = 0; r < kGroup; ++r) dot[r] += __shfl_xor_sync(0xffffffffu, dot[r], off);
  const int row = (lane >> 2) & 3;
  const float sc = (row == 0 ? dot[0] : row == 1 ? dot[1] : row == 2 ? dot[2] : dot[3]) * scale_log2;
  const float m_new = fmaxf(st.m, sc);
  const float alpha = exp2f(st.m - m_new);
  const float pr = bf16r(exp2f(sc - m_new));
  st.l = st.l * alpha + ((lane & 3) == 0 ? pr : 0.f);
  st.m = m_new;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float2 vv = bf2f(*reinterpret_cast<const uint32_t*>(&s.vnew[8 * j + 2 * (lane & 3)]));
    st.o[j][0] = st.o[j][0] * alpha + pr * vv.x;
    st.o[j][1] = st.o[j][1] * alpha + pr * vv.y;
  }
}

// ------------------------------------------------------------------------------- main kernel
// Issue side of a warp's private pipeline: walks the CTA's claimed chunks in order and yields the
// tiles in which this warp owns a page (page jw of tile i = keys t0 + 128 i + 16 jw ...).
template <bool PAGED, bool FUSED>
struct Issuer {
  int k;              // next ring index to open
  int chunk, x, x1;   // current chunk and the unopened part of its page range [x, x1)
  Unit U;
  int ti, ntiles;     // current tile within U
  int npg;            // pages streamed by U
  int rot;            // pages the CTA streamed before U, mod 8
  int jw;             // this warp's page in each tile of U: (warp - rot) mod 8
  const int* bt_row;  // block-table row of U, from U's first page
  int win, win_next, win_base;  // page ids of this warp's pages of tiles win_base + lane

  __device__ __forceinline__ void open_window(int lane, int base) {
    win_base = base;
    const int a = 8 * (base + lane) + jw, b = 8 * (base + 32 + lane) + jw;
    win = a < npg ? bt_row[a] : 0;
    win_next = b < npg ? bt_row[b] : 0;
  }
  // Advance to the next tile with a page of this warp: 1 = found, 0 = the next chunk is not
  // claimed yet (retry later), -1 = no chunks left.
  __device__ __forceinline__ int next(const Params& p, const Smem& s, int warp, int lane) {
    while (true) {
      ++ti;
      while (ti >= ntiles) {
        if (x >= x1) {   // chunk exhausted: open the next claimed one
          if (k >= s.nclaimed) return 0;
          __threadfence_block();   // pairs with the fence between the ring write and nclaimed
          const int c = const_cast<const volatile int*>(s.ring)[k & 3];
          if (c < 0 || c >= s.total_chunks) return -1;
          ++k;
          chunk = c;
          chunk_range(s, c, x, x1);
          continue;
        }
        U = unit_at<FUSED>(p, s, chunk, x, x1);
        rot = (rot + npg) & 7;
        jw = (warp - rot) & 7;
        ntiles = ceil_div_i(U.t1 - U.t0, kTile);
        npg = ceil_div_i(U.t1 - U.t0, kPage);
        ti = 0;
        if (PAGED && ntiles > 0) {
          bt_row = p.bt + static_cast<long long>(U.b) * p.bt_stride + U.t0 / kPage;
          open_window(lane, 0);
        }
      }
      if (U.t0 + ti * kTile + jw * kPage < U.t1) return 1;
    }
  }
  // TMA of this warp's page of the current tile into ring slot `slot` (lane 0 issues).
  __device__ __forceinline__ void issue(const Params& p, Smem& s, int slot, int warp, int lane,
                                        uint64_t pol) {
    int row = 0;
    bool ok = true;
    if (PAGED) {
      if (ti >= win_base + 32) {   // window exhausted: move on, prefetch the one after
        win = win_next;
        win_base += 32;
        const int b = 8 * (win_base + 32 + lane) + jw;
        win_next = b < npg ? bt_row[b] : 0;
      }
      const int pid = __shfl_sync(0xffffffffu, win, ti - win_base);
      if (pid < 0 || pid >= p.num_pages) {
        ok = false;
      } else {
        row = (pid * p.nkv + U.kvh) * kPage;
      }
    }
    if (lane == 0) {
      const uint32_t fb = smem_u32(&s.full[slot][warp]);
      if (!ok) {
        atomicOr(&s.err_bits, KOPT_DEV_ERR_PAGE);
        mbar_arrive_expect_tx(fb, 0);   // completes the phase without data
        return;
      }
      // order this warp's earlier generic reads/writes of the slot before the async-proxy refill
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(fb, 4u * kBoxBytes);
      const int tq = U.t0 + ti * kTile + jw * kPage;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t dk = smem_u32(&s.k[slot][warp][h][0]);
        const uint32_t dv = smem_u32(&s.v[slot][warp][h][0]);
        if (PAGED) {
          tma_load_2d(dk, &p.tmk, h * kHalf, row, fb, pol);
          tma_load_2d(dv, &p.tmv, h * kHalf, row, fb, pol);
        } else {
          tma_load_4d(dk, &p.tmk, h * kHalf, tq, U.kvh, U.b, fb, pol);
          tma_load_4d(dv, &p.tmv, h * kHalf, tq, U.kvh, U.b, fb, pol);
        }
      }
    }
  }
};

template <bool PAGED, bool FUSED>
__global__ void __launch_bounds__(kThreads, 1) decode_attn_kernel(const __grid_constant__ Params p) {
  extern __shared__ unsigned char smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.nkv * kGroup;

  // Launched with programmatic dependent launch (KOPT_PLAN_OVERLAP_PREV), this CTA may start while
  // the previous kernel on the stream is still running. Before griddep_wait it reads only pos, the
  // block table and cache rows below pos (which that kernel must not write) and writes nothing
  // outside shared memory. The unfused variant reads the row at pos, which the standalone
  // prologue kernel before it writes, so it waits first.
  if (!FUSED) griddep_wait();
  if (warp == 0) compute_plan<FUSED>(p, s, lane);
  if (threadIdx.x == 32) {
    for (int i = 0; i < kStages; ++i)
      for (int w = 0; w < kNW; ++w) mbar_init(smem_u32(&s.full[i][w]), 1);
    s.abort = 0;
    s.npend = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x == 64) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmk) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&p.tmv) : "memory");
  }
  __syncwarp();
  if (threadIdx.x == 0) {   // the static piece; dynamic chunks are claimed from the prologues
    s.ring[0] = blockIdx.x;
    s.ring[1] = s.ring[2] = s.ring[3] = -1;
    s.nclaimed = 1;
    if (s.total_chunks == static_cast<int>(gridDim.x)) s.nclaimed = 2;   // piece, then end
  }
  __syncthreads();
  const uint64_t pol = evict_first_policy();
  // With no dynamic chunks nothing of the first unit touches the workspace, so its split and its
  // first page copies go out before the wait; otherwise all of it waits.
  const bool early = s.total_chunks == static_cast<int>(gridDim.x);

  const int ctid = threadIdx.x;
  // Consume cursor: ring index kc to open next, current chunk and its unvisited pages [cx, cx1).
  int kc = 0, chunk = -1, cx = 0, cx1 = 0;
  int pend_claim = -2;   // thread 0: raw claim in flight for ring index kc (published at a prologue)
  // Next unit along the cursor; opening a chunk claims the one after it.
  auto advance = [&](Unit& V) -> bool {
    while (cx >= cx1) {
      if (kc >= s.nclaimed) {   // never read a ring entry before it is published
        if (ctid == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PLAN);
        return false;
      }
      const int c = const_cast<const volatile int*>(s.ring)[kc & 3];
      if (c < 0) return false;
      if (c >= s.total_chunks) {
        if (ctid == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PLAN);
        return false;
      }
      chunk = c;
      chunk_range(s, c, cx, cx1);
      ++kc;
      // claim the chunk after this one, unless the piece was empty (then it was claimed up front)
      if (ctid == 0 && cx < cx1 && s.total_chunks > static_cast<int>(gridDim.x))
        pend_claim = claim_issue(p);
    }
    V = unit_at<FUSED>(p, s, chunk, cx, cx1);
    return true;
  };
  // Stage unit V's prologue inputs: warp w < 4 its q head row, warp 4 the k row, warp 5 the v row,
  // warps 6/7 the RoPE rows (16 lanes x 16 B each).
  auto stage = [&](const Unit& V) {
    const bf16* src = nullptr;
    if (warp < kGroup) {
      const int h = V.kvh * kGroup + warp;
      src = FUSED ? p.qkv + static_cast<long long>(V.b) * (nq + 2 * p.nkv) * kD + h * kD
                  : p.q + static_cast<long long>(V.b) * p.T * nq * kD + h * kD;
    } else if (FUSED) {
      const bf16* row = p.qkv + static_cast<long long>(V.b) * (nq + 2 * p.nkv) * kD;
      int rp = V.L - 1;
      if (rp >= p.rope_len) {
        if (lane == 0 && warp == 6) atomicOr(p.ws_err, KOPT_DEV_ERR_ROPE);
        rp = p.rope_len - 1;
      }
      if (warp == 4) src = row + (nq + V.kvh) * kD;
      else if (warp == 5) src = row + (nq + p.nkv + V.kvh) * kD;
      else if (warp == 6) src = p.cos + static_cast<long long>(rp) * kD;
      else src = p.sin + static_cast<long long>(rp) * kD;
    }
    if (src != nullptr && lane < 16) cp_async16(smem_u32(&s.rows[warp][8 * lane]), src + 8 * lane);
    cp_async_commit();
  };
  // Merge every partial of pair (q, b, kvh) held in slots c + q, c in c0 .. c0+n-1: online
  // log-sum-exp over the splits, loads issued four splits at a time.
  auto merge_pair = [&](int q, int c0, int n, int b, int kvh) {
    const int r = ctid >> 6, d = 2 * (ctid & 63);
    float M = kNegBig, L = 0.f;
    float2 O = make_float2(0.f, 0.f);
    for (int c = c0; c < c0 + n; c += 4) {
      float2 ml[4], oj[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (c + j < c0 + n) {
          const long long sl = static_cast<long long>(c + j) + q;
          ml[j] = __ldcg(&p.ws_ml[sl * kGroup + r]);
          oj[j] = __ldcg(reinterpret_cast<const float2*>(&p.ws_o[(sl * kGroup + r) * kD + d]));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (c + j < c0 + n) {
          const float mn = fmaxf(M, ml[j].x);
          const float a = exp2f(M - mn), f = exp2f(ml[j].x - mn);
          L = L * a + ml[j].y * f;
          O.x = O.x * a + oj[j].x * f;
          O.y = O.y * a + oj[j].y * f;
          M = mn;
        }
      }
    }
    const float inv = 1.0f / L;
    store_out(p, b, kvh * kGroup + r, d, O.x * inv, O.y * inv);
    if (ctid == 0) atomicExch(&p.ws_cnt[q], 0);
  };
  // Releasing a partial (fence, then the pair's counter) waits until this CTA's partial stores are
  // acknowledged, microseconds under full HBM load, and would stall the warp doing it and with it
  // the whole unit. So partial units are only recorded as they finish, and released together
  // once, when the CTA has streamed all its pages (or when the record is full); whoever releases
  // a pair's last partial merges it then. Collective: every thread calls flush.
  auto flush = [&]() {
    if (ctid == 0) {
      const int np = s.npend;
      int nm = 0;
      if (np > 0) {
        __threadfence();
        int prev[kMaxPend];
#pragma unroll
        for (int i = 0; i < kMaxPend; ++i) prev[i] = i < np ? atomicAdd(&p.ws_cnt[s.pend[i][0]], 1) : 0;
#pragma unroll
        for (int i = 0; i < kMaxPend; ++i)
          if (i < np && prev[i] == s.pend[i][2] - 1) s.merge[nm++] = i;
        if (nm > 0) __threadfence();   // acquire the other units' partials
      }
      s.nmerge = nm;
    }
    named_bar(1, kNW * 32);
    for (int i = 0; i < s.nmerge; ++i) {
      const int* e = s.pend[s.merge[i]];
      merge_pair(e[0], e[1], e[2], e[3], e[4]);
    }
    named_bar(1, kNW * 32);
    if (ctid == 0) s.npend = 0;
  };

  Unit U;
  bool have = false;
  // This warp's ring: `state` tells whether the issue cursor stands on an unissued tile.
  Issuer<PAGED, FUSED> iss;
  iss.k = 0;
  iss.chunk = 0;
  iss.x = iss.x1 = 0;
  iss.ti = 0;
  iss.ntiles = 0;
  iss.npg = 0;
  iss.rot = 0;
  iss.jw = warp;
  iss.bt_row = nullptr;
  iss.win = iss.win_next = iss.win_base = 0;
  int state = 0;
  int issued = 0, consumed = 0;
  auto pump = [&]() {
    while (issued - consumed < kStages && !__shfl_sync(0xffffffffu, s.abort, 0)) {
      if (state == 0) state = iss.next(p, s, warp, lane);
      if (state != 1) break;
      iss.issue(p, s, issued % kStages, warp, lane, pol);
      ++issued;
      state = iss.next(p, s, warp, lane);
    }
  };
  if (early) {
    have = advance(U);
    state = iss.next(p, s, warp, lane);
    pump();
  }
  if (FUSED) griddep_wait();
  griddep_launch_dependents();
  if (FUSED && (warp == 2 || warp == 3)) {   // q_norm / k_norm weights, once per CTA
    const bf16* w = warp == 2 ? p.qw : p.kw;
    bf16* dstw = warp == 2 ? s.wq : s.wk;
    *reinterpret_cast<uint2*>(dstw + 4 * lane) = *reinterpret_cast<const uint2*>(w + 4 * lane);
  }
  if (!early) {
    if (threadIdx.x == 0 && s.static_pages == 0) {
      // no pieces: the first dynamic chunk must be known up front (with P = 0 every chunk is
      // dynamic, so total_chunks > grid whenever there is work)
      s.ring[1] = claim_chunk(claim_issue(p), s.total_chunks);
      s.nclaimed = 2;
    }
    __syncthreads();
    have = advance(U);
    state = iss.next(p, s, warp, lane);
    pump();
  }
  if (have) stage(U);   // the first unit's prologue inputs travel while the rings fill

  int cbase = 0;   // pages streamed by the units before U, mod 8
  while (have) {
    const bool inject = FUSED && U.last;
    const int se = U.t1;                          // keys streamed from the cache end here
    const int ntiles = ceil_div_i(se - U.t0, kTile);
    // Pages go to the warps round-robin along the CTA's whole piece, not unit by unit, so that
    // the short last tiles of successive units do not all land on the same warps.
    const int jw = (warp - cbase) & 7;
    cbase = (cbase + ceil_div_i(se - U.t0, kPage)) & 7;

    // ---- prologue from the staged rows: q rows, and the new K/V for the unit ending the pair
    cp_async_wait_all();
    if (ctid == 0 && pend_claim != -2) {
      s.ring[kc & 3] = claim_chunk(pend_claim, s.total_chunks);
      __threadfence_block();
      s.nclaimed = kc + 1;
      pend_claim = -2;
    }
    named_bar(1, kNW * 32);
    pump();   // a chunk claimed in the previous unit is visible now
    if (FUSED) {
      float y[4];
      if (warp < kGroup) {
        norm_rope_head(s.rows[warp], s.wq, s.rows[6], s.rows[7], p.eps, lane, y);
        store4_bf16(&s.q[warp][4 * lane], y);
        if (p.q_out != nullptr && U.t0 == 0)
          store4_bf16(p.q_out + static_cast<long long>(U.b) * nq * kD +
                          (U.kvh * kGroup + warp) * kD + 4 * lane, y);
      } else if (inject && warp < kGroup + 2) {
        const long long off = row_offset(p, U.b, U.kvh, U.L - 1);
        if (warp == kGroup) {
          norm_rope_head(s.rows[4], s.wk, s.rows[6], s.rows[7], p.eps, lane, y);
          store4_bf16(&s.knew[4 * lane], y);
          if (off >= 0) store4_bf16(p.kc + off + 4 * lane, y);
        } else {
          const uint2 raw = *reinterpret_cast<const uint2*>(&s.rows[5][4 * lane]);
          *reinterpret_cast<uint2*>(&s.vnew[4 * lane]) = raw;
          if (off >= 0) *reinterpret_cast<uint2*>(p.vc + off + 4 * lane) = raw;
        }
        if (off < 0 && lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
      }
    } else if (warp < kGroup) {
      *reinterpret_cast<uint2*>(&s.q[warp][4 * lane]) =
          *reinterpret_cast<const uint2*>(&s.rows[warp][4 * lane]);
    }
    named_bar(1, kNW * 32);
    // A fragments of Q (rows 0-3 live on lanes 0-15): a0 = Q[r][16ks + 2(l%4) + {0,1}], a2 = +8
    uint32_t qa[8][2];
    {
      const int r = lane >> 2, c = 2 * (lane & 3);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qa[ks][0] = lane < 16 ? *reinterpret_cast<const uint32_t*>(&s.q[r & 3][16 * ks + c]) : 0u;
        qa[ks][1] = lane < 16 ? *reinterpret_cast<const uint32_t*>(&s.q[r & 3][16 * ks + 8 + c]) : 0u;
      }
    }

    WarpState st;
    st.m = kNegBig;
    st.l = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) st.o[j][0] = st.o[j][1] = 0.f;

    // Look one unit ahead and stage its inputs while this unit streams; done after this warp's
    // first tile so that it does not delay the start of the unit.
    bool looked = false;
    auto look_ahead = [&]() {
      Unit Un;
      const bool hn = advance(Un);
      if (hn) stage(Un);
      if (ctid == 0) {
        static_assert(sizeof(Unit) <= sizeof(s.unext), "look-ahead unit does not fit");
        *reinterpret_cast<Unit*>(s.unext) = Un;
        s.have_next = hn;
      }
      looked = true;
    };
    for (int i = 0; i < ntiles; ++i) {
      const int ntok = min(max(se - (U.t0 + i * kTile + jw * kPage), 0), kPage);
      if (ntok == 0) continue;          // no page of this warp in this tile
      if (issued == consumed) pump();   // this tile's copy must be in flight before waiting
      const int slot = consumed % kStages;
      mbar_wait(smem_u32(&s.full[slot][warp]), (consumed / kStages) & 1, s, p.ws_err, true);
      __syncwarp();   // lanes leave the bounded spin at different times: reconverge before mma.sync
      page_step(smem_u32(&s.k[slot][warp][0][0]), smem_u32(&s.v[slot][warp][0][0]), ntok, qa,
                p.scale_log2, st, lane);
      ++consumed;
      __syncwarp();
      pump();                           // refill the slot just consumed
      if (!looked) look_ahead();
    }
    if (!looked) look_ahead();          // this warp had no tile in this unit
    if (inject && warp == 0) inject_token(s, p.scale_log2, st, lane);

    // ---- epilogue: merge the 8 warps; a split pair's partial goes to the workspace
    float l = st.l;
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
    if (lane < 16) {
      const int r = lane >> 2, c = 2 * (lane & 3);
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2*>(&s.o[warp][r][8 * j + c]) = make_float2(st.o[j][0], st.o[j][1]);
      if ((lane & 3) == 0) {
        s.red_m[warp][r] = st.m;
        s.red_l[warp][r] = l;
      }
    }
    named_bar(1, kNW * 32);
    // thread -> (output row r = query head kvh*4 + r, dims d .. d+1)
    const int r = ctid >> 6, d = 2 * (ctid & 63);
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < kNW; ++w) M = fmaxf(M, s.red_m[w][r]);
    float Lsum = 0.f;
    float2 O = make_float2(0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float f = exp2f(s.red_m[w][r] - M);
      Lsum += f * s.red_l[w][r];
      const float2 ow = *reinterpret_cast<const float2*>(&s.o[w][r][d]);
      O.x += f * ow.x;
      O.y += f * ow.y;
    }
    if (U.n == 1) {
      const float inv = 1.0f / Lsum;
      store_out(p, U.b, U.kvh * kGroup + r, d, O.x * inv, O.y * inv);
    } else {
      const long long slot = U.slot;
      *reinterpret_cast<float2*>(&p.ws_o[(slot * kGroup + r) * kD + d]) = O;
      if ((ctid & 63) == 0) p.ws_ml[slot * kGroup + r] = make_float2(M, Lsum);
    }
    named_bar(1, kNW * 32);
    if (U.n > 1 && ctid == 0) {   // released by flush
      int* e = s.pend[s.npend++];
      e[0] = U.q; e[1] = U.c0; e[2] = U.n; e[3] = U.b; e[4] = U.kvh;
    }
    named_bar(1, kNW * 32);   // parked look-ahead unit visible
    if (s.npend == kMaxPend) flush();
    have = s.have_next != 0;
    U = *reinterpret_cast<const Unit*>(s.unext);
  }
  flush();   // release this CTA's partials; merge the pairs it completes
  // Drain: after an abort, copies issued into this warp's ring may still be in flight. The last
  // phase issued to each slot is the newest one on its barrier, so waiting on it is exact.
  if (lane == 0) {
    for (int k = issued > kStages ? issued - kStages : 0; k < issued; ++k)
      mbar_wait(smem_u32(&s.full[k % kStages][warp]), (k / kStages) & 1, s, p.ws_err, false);
  }
  // The last CTA to finish (all claims made) resets the chunk counter for the next call; with the
  // fused gather it also tells every rank that all of this rank's rows have landed there. A call
  // split statically only (no chunk is claimed) and without the gather needs neither, so its
  // CTAs skip the fence and the count (the whole grid takes the same branch: total_chunks is
  // the same in every CTA) and leave the SM sooner.
  if (p.world > 0) named_bar(1, kNW * 32);   // every output store of this CTA is issued
  if (threadIdx.x == 0 && p.world == 0 && s.total_chunks == static_cast<int>(gridDim.x)) {
    if (s.err_bits) atomicOr(p.ws_err, s.err_bits);
  } else if (threadIdx.x == 0) {
    if (s.err_bits) atomicOr(p.ws_err, s.err_bits);
    if (p.world > 0) __threadfence_system();   // this CTA's rows visible to the peers
    else __threadfence();
    if (atomicAdd(p.ws_err + 2, 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(p.ws_err + 1, 0);
      atomicExch(p.ws_err + 2, 0);
      if (p.world > 0) gather_signal_and_wait(p);
    }
  }
}

// ------------------------------------------------------------- standalone QK-norm/RoPE/append
// Grid (B*T, ceil((nq + 2 nkv) / 4)), 4 warps, one (token, head) per warp: fused.py:54-96.
__global__ void __launch_bounds__(128) qk_norm_rope_kernel(const __grid_constant__ Params p, int nheads) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y * 4 + warp;
  if (h >= nheads) return;
  const int m = blockIdx.x;
  const int b = m / p.T;
  const int nq = p.nkv * kGroup;
  const int row = (nq + 2 * p.nkv) * kD;
  int ps = p.pos[b] + m % p.T;
  if (ps < 0 || ps >= p.cap) {
    if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_LEN);
    ps = ps < 0 ? 0 : p.cap - 1;
  }
  const bf16* src = p.qkv + static_cast<long long>(m) * row + h * kD;
  if (h < nq + p.nkv) {
    int rp = ps;
    if (rp >= p.rope_len) {
      if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_ROPE);
      rp = p.rope_len - 1;
    }
    float y[4];
    norm_rope_head(src, h < nq ? p.qw : p.kw, p.cos + static_cast<long long>(rp) * kD,
                   p.sin + static_cast<long long>(rp) * kD, p.eps, lane, y);
    if (h < nq) {
      store4_bf16(p.q_out + static_cast<long long>(m) * nq * kD + h * kD + 4 * lane, y);
    } else {
      const long long off = row_offset(p, b, h - nq, ps);
      if (off >= 0) store4_bf16(p.kc + off + 4 * lane, y);
      else if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
    }
  } else {
    const long long off = row_offset(p, b, h - nq - p.nkv, ps);
    if (off >= 0)
      *reinterpret_cast<uint2*>(p.vc + off + 4 * lane) = *reinterpret_cast<const uint2*>(src + 4 * lane);
    else if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
  }
}

// ======================================================== verify attention (T > 1 query tokens)
// T query tokens per sequence at positions pos[b] .. pos[b] + T - 1, causal among themselves: the
// query at pos[b] + t sees keys 0 .. pos[b] + t (fused.py:130-185 with T > 1, the verify step of
// engine.py:403-415). Their K/V are already in the cache (qk_norm_rope appends all T). One CTA
// takes one (pair, split of the keys) and all 4 T query rows of the pair (T tokens x the 4 heads
// of the GQA group) on MT m16 MMA tiles (MT = 1 for T <= 4, 2 for T <= 8), so every key is read
// once. 4 page streams go round-robin over the split's pages through 3-deep TMA rings; each stream
// is consumed by MT warps, warp w taking row tile w / 4 of stream w % 4, so a warp carries one
// tile's state whatever T is. A ring slot is refilled once all its consumers are done with it.
// The split that finishes last merges the partials.
constexpr int kVW = 4;                       // page streams per verify CTA
constexpr int kVStages = 3;
constexpr int kVMaxT = 8;
template <int MT>
__host__ __device__ constexpr int verify_threads() { return kVW * MT * 32; }

template <int MT>
struct __align__(1024) VSmem {
  bf16 k[kVStages][kVW][2][kPage * kHalf];   // per stream and stage: one page, two 64-dim boxes
  bf16 v[kVStages][kVW][2][kPage * kHalf];
  alignas(16) bf16 q[16 * MT][kD + 8];       // query rows (padded rows: no ldmatrix conflicts)
  float red_m[kVW][16 * MT];
  float red_l[kVW][16 * MT];
  unsigned long long full[kVStages][kVW];    // slot filled by the stream's TMA
  unsigned long long empty[kVStages][kVW];   // slot consumed by the stream's MT warps
  int last;                                  // this CTA merges the splits of its pair
  volatile int abort;
};
template <int MT>
constexpr size_t vsmem_bytes() { return sizeof(VSmem<MT>) + 1024; }
inline int verify_tiles(int T) { return T > 4 ? 2 : 1; }

// D += A B, m16n8k16, all 16 rows live (4 accumulators).
__device__ __forceinline__ void mma16816_full(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                              uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <bool PAGED, int MT>
__global__ void __launch_bounds__(verify_threads<MT>()) verify_attn_kernel(const __grid_constant__ Params p) {
  constexpr int R = 16 * MT;                 // query rows
  constexpr int NT = verify_threads<MT>();
  // the warps' partial outputs reuse the rings once every page is consumed
  static_assert(sizeof(float) * kVW * R * (kD + 4) <= sizeof(bf16) * 2 * kVStages * kVW * 2 * kPage * kHalf,
                "verify partials do not fit in the rings");
  extern __shared__ unsigned char smem_raw[];
  VSmem<MT>& s = *reinterpret_cast<VSmem<MT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sw = warp % kVW;                 // this warp's page stream
  const int mt = warp / kVW;                 // and its row tile
  const bool issuer = mt == 0;               // the stream's first warp issues its copies
  const int nq = p.nkv * kGroup;
  const int split = blockIdx.x % p.nsplit;
  const int pair = blockIdx.x / p.nsplit;
  const int b = pair / p.nkv, kvh = pair % p.nkv;
  const int T = p.T;                                    // 2 .. 4 MT
  int p0 = p.pos[b];
  if (p0 < 0 || p0 + T > p.cap) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_LEN);
    p0 = min(max(p0, 0), p.cap - T);
  }
  const int Lb = p0 + T;                                // keys the last query sees
  const int per = ceil_div_i(ceil_div_i(Lb, p.nsplit), kPage) * kPage;
  const int s0 = split * per, s1 = min(Lb, s0 + per);   // this split's keys (s0 on a page edge)
  const int pg0 = s0 / kPage;
  const int npg = s1 > s0 ? ceil_div_i(s1, kPage) - pg0 : 0;
  const int mine = npg > sw ? ceil_div_i(npg - sw, kVW) : 0;   // pages of this stream

  if (threadIdx.x == 0) {
    for (int i = 0; i < kVStages; ++i)
      for (int w = 0; w < kVW; ++w) {
        mbar_init(smem_u32(&s.full[i][w]), 1);
        mbar_init(smem_u32(&s.empty[i][w]), MT);
      }
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const uint64_t pol = evict_first_policy();

  // page ids of this stream's pages k = base + lane, 32 at a time
  const int* bt_row = PAGED ? p.bt + static_cast<long long>(b) * p.bt_stride : nullptr;
  int win = 0, win_base = -32;
  auto issue = [&](int k) {
    const int pg = pg0 + sw + k * kVW;
    int row = 0;
    bool ok = true;
    if (PAGED) {
      if (k >= win_base + 32) {
        win_base = k - (k & 31);
        const int kk = win_base + lane;
        win = kk < mine ? bt_row[pg0 + sw + kk * kVW] : 0;
      }
      const int pid = __shfl_sync(0xffffffffu, win, k - win_base);
      if (pid < 0 || pid >= p.num_pages) ok = false;
      else row = (pid * p.nkv + kvh) * kPage;
    }
    if (lane == 0) {
      const int slot = k % kVStages;
      const uint32_t fb = smem_u32(&s.full[slot][sw]);
      if (!ok) {
        atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
        mbar_arrive_expect_tx(fb, 0);
        return;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_arrive_expect_tx(fb, 4u * kBoxBytes);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t dk = smem_u32(&s.k[slot][sw][h][0]);
        const uint32_t dv = smem_u32(&s.v[slot][sw][h][0]);
        if (PAGED) {
          tma_load_2d(dk, &p.tmk, h * kHalf, row, fb, pol);
          tma_load_2d(dv, &p.tmv, h * kHalf, row, fb, pol);
        } else {
          tma_load_4d(dk, &p.tmk, h * kHalf, pg * kPage, kvh, b, fb, pol);
          tma_load_4d(dv, &p.tmv, h * kHalf, pg * kPage, kvh, b, fb, pol);
        }
      }
    }
  };
  // the first copies go out before the query rows are read
  int issued = 0;
  if (issuer)
    for (; issued < min(mine, kVStages) && !__shfl_sync(0xffffffffu, s.abort, 0); ++issued) issue(issued);

  // query rows r = 4 j + g: token j, head kvh * 4 + g (rows of tokens past T are zero)
  for (int i = threadIdx.x; i < R * (kD / 8); i += NT) {
    const int r = i / (kD / 8), c = i % (kD / 8);
    const int j = r / kGroup, g = r % kGroup;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (j < T)
      v = *reinterpret_cast<const uint4*>(
          p.q + (static_cast<long long>(b) * T + j) * nq * kD + (kvh * kGroup + g) * kD + c * 8);
    *reinterpret_cast<uint4*>(&s.q[r][c * 8]) = v;
  }
  __syncthreads();

  // lane: in this warp's tile, rows 16 mt + lane / 4 (h = 0) and + 8 (h = 1), columns 2 (lane % 4) + {0, 1}
  float m[2], l[2];
  int lim[2];            // last key each row sees (-1: a row past the T tokens)
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int r = 16 * mt + 8 * h + (lane >> 2);
    m[h] = kNegBig;
    l[h] = 0.f;
    lim[h] = r / kGroup < T ? p0 + r / kGroup : -1;
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  const int mi = lane >> 3, ri = lane & 7;
  const uint32_t qaddr = smem_u32(&s.q[16 * mt + (lane & 15)][(lane >> 4) * 8]);

  for (int k = 0; k < mine; ++k) {
    const int slot = k % kVStages;
    mbar_wait(smem_u32(&s.full[slot][sw]), (k / kVStages) & 1, s, p.ws_err, true);
    __syncwarp();   // reconverge after the per-lane spin before ldmatrix / mma.sync
    const int key0 = (pg0 + sw + k * kVW) * kPage;
    const uint32_t kbase = smem_u32(&s.k[slot][sw][0][0]);
    const uint32_t vbase = smem_u32(&s.v[slot][sw][0][0]);
    // ---- S = Q K^T, this tile's 16 rows x 16 keys
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int tok = 8 * (mi >> 1) + ri;
      const uint32_t krow = kbase + tok * 128;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int h = ks >> 2, c = 2 * (ks & 3) + (mi & 1);
        uint32_t b00, b01, b10, b11, a0, a1, a2, a3;
        ldsm_x4(krow + h * kBoxBytes + ((c ^ ri) << 4), b00, b01, b10, b11);
        ldsm_x4(qaddr + ks * 32, a0, a1, a2, a3);
        mma16816_full(c0, a0, a1, a2, a3, b00, b01);
        mma16816_full(c1, a0, a1, a2, a3, b10, b11);
      }
    }
    const int kc = key0 + 2 * (lane & 3);
    // rows of the page past the split's keys may hold anything: zero them so 0 * V stays 0 (the
    // stream's first warp does it; its partner waits for it below)
    const int ntok = min(s1 - key0, kPage);
    if (ntok < kPage) {
      if (issuer) {
        for (int i = lane; i < (kPage - ntok) * 16; i += 32) {
          const int r = ntok + (i >> 4), part = i & 15;
          const uint32_t a = vbase + (part >> 3) * kBoxBytes + r * 128 + ((part & 7) << 4);
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
        }
      }
      if (MT > 1) named_bar(2 + sw, 32 * MT);   // the stream's warps: zeroed rows visible
      else __syncwarp();
    }
    const int tok = 8 * (mi & 1) + ri;
    const uint32_t vrow = vbase + tok * 128;
    // ---- online softmax, rows h = 0 / 1 of this tile (4 lanes share a row)
    uint32_t pa[4];
    float al[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int lm = lim[h];
      float sv[4];
      sv[0] = (kc < s1 && kc <= lm) ? c0[2 * h] * p.scale_log2 : -INFINITY;
      sv[1] = (kc + 1 < s1 && kc + 1 <= lm) ? c0[2 * h + 1] * p.scale_log2 : -INFINITY;
      sv[2] = (kc + 8 < s1 && kc + 8 <= lm) ? c1[2 * h] * p.scale_log2 : -INFINITY;
      sv[3] = (kc + 9 < s1 && kc + 9 <= lm) ? c1[2 * h + 1] * p.scale_log2 : -INFINITY;
      float x = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
      x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
      const float mn = fmaxf(m[h], x);
      al[h] = exp2f(m[h] - mn);
      float pr[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) pr[e] = exp2f(sv[e] - mn);
      l[h] = l[h] * al[h] + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
      m[h] = mn;
      // P as the A operand: a0 / a1 rows h = 0 / 1 keys 0-7, a2 / a3 keys 8-15
      pa[h] = pack_bf16(pr[0], pr[1]);
      pa[2 + h] = pack_bf16(pr[2], pr[3]);
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= al[0];
      o[j][1] *= al[0];
      o[j][2] *= al[1];
      o[j][3] *= al[1];
    }
    // ---- O += P V
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const int c = j + (mi >> 1);
      uint32_t b0a, b1a, b0b, b1b;
      ldsm_x4_t(vrow + (c >> 3) * kBoxBytes + (((c & 7) ^ ri) << 4), b0a, b1a, b0b, b1b);
      mma16816_full(o[j], pa[0], pa[1], pa[2], pa[3], b0a, b1a);
      mma16816_full(o[j + 1], pa[0], pa[1], pa[2], pa[3], b0b, b1b);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&s.empty[slot][sw]));   // this warp is done with the slot
    if (issuer && issued < mine && !__shfl_sync(0xffffffffu, s.abort, 0)) {
      // refill the slot once every consumer of the stream has left it
      const bool ok = mbar_wait(smem_u32(&s.empty[slot][sw]), (k / kVStages) & 1, s, p.ws_err, true);
      __syncwarp();
      if (ok) issue(issued++);
    }
  }
  // every copy this stream issued has landed (waited above, or drained here after an abort)
  if (issuer && lane == 0)
    for (int k = max(issued - kVStages, 0); k < issued; ++k)
      mbar_wait(smem_u32(&s.full[k % kVStages][sw]), (k / kVStages) & 1, s, p.ws_err, false);

  // ---- merge the streams (partials in the ring memory), then the splits of this pair
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  __syncthreads();   // every warp is done with the rings
  float* ob = reinterpret_cast<float*>(&s.k[0][0][0][0]);   // [kVW][R][kD + 4]
  {
    const int c = 2 * (lane & 3);
    const int rA = 16 * mt + (lane >> 2), rB = rA + 8;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      *reinterpret_cast<float2*>(&ob[(sw * R + rA) * (kD + 4) + 8 * j + c]) = make_float2(o[j][0], o[j][1]);
      *reinterpret_cast<float2*>(&ob[(sw * R + rB) * (kD + 4) + 8 * j + c]) = make_float2(o[j][2], o[j][3]);
    }
    if ((lane & 3) == 0) {
      s.red_m[sw][rA] = m[0];
      s.red_l[sw][rA] = l[0];
      s.red_m[sw][rB] = m[1];
      s.red_l[sw][rB] = l[1];
    }
  }
  __syncthreads();
  // thread -> row r, dims d0 .. d0 + DPT - 1
  constexpr int TPR = NT / R, DPT = kD / TPR;
  const int r = threadIdx.x / TPR, d0 = (threadIdx.x % TPR) * DPT;
  const int j = r / kGroup, g = r % kGroup;
  float M = kNegBig;
#pragma unroll
  for (int w = 0; w < kVW; ++w) M = fmaxf(M, s.red_m[w][r]);
  float Lsum = 0.f, O[DPT];
#pragma unroll
  for (int e = 0; e < DPT; ++e) O[e] = 0.f;
#pragma unroll
  for (int w = 0; w < kVW; ++w) {
    const float f = exp2f(s.red_m[w][r] - M);
    Lsum += f * s.red_l[w][r];
#pragma unroll
    for (int e = 0; e < DPT; e += 4) {
      const float4 x = *reinterpret_cast<const float4*>(&ob[(w * R + r) * (kD + 4) + d0 + e]);
      O[e] += f * x.x;
      O[e + 1] += f * x.y;
      O[e + 2] += f * x.z;
      O[e + 3] += f * x.w;
    }
  }
  bf16* dst = p.out + ((static_cast<long long>(b) * T + j) * nq + kvh * kGroup + g) * kD + d0;
  if (p.nsplit == 1) {
    if (j < T) {
      const float inv = 1.0f / Lsum;
#pragma unroll
      for (int e = 0; e < DPT; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16(O[e] * inv, O[e + 1] * inv);
    }
    return;
  }
  const long long slot = blockIdx.x;
  float* po = p.ws_o + (slot * R + r) * kD + d0;
#pragma unroll
  for (int e = 0; e < DPT; e += 4) *reinterpret_cast<float4*>(po + e) = make_float4(O[e], O[e + 1], O[e + 2], O[e + 3]);
  if ((threadIdx.x % TPR) == 0) p.ws_ml[slot * R + r] = make_float2(M, Lsum);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s.last = atomicAdd(&p.ws_cnt[pair], 1) == p.nsplit - 1;
    if (s.last) __threadfence();   // acquire the other splits' partials
  }
  __syncthreads();
  if (!s.last) return;
  // the last split of the pair: online log-sum-exp over every split's partial
  const long long first = blockIdx.x - split;
  float Mm = kNegBig, Lm = 0.f;
#pragma unroll
  for (int e = 0; e < DPT; ++e) O[e] = 0.f;
  for (int sp = 0; sp < p.nsplit; ++sp) {
    const long long sl = first + sp;
    const float2 ml = __ldcg(&p.ws_ml[sl * R + r]);
    const float mn = fmaxf(Mm, ml.x);
    const float a = exp2f(Mm - mn), f = exp2f(ml.x - mn);
    Lm = Lm * a + ml.y * f;
    const float* src = p.ws_o + (sl * R + r) * kD + d0;
#pragma unroll
    for (int e = 0; e < DPT; e += 4) {
      const float4 x = __ldcg(reinterpret_cast<const float4*>(src + e));
      O[e] = O[e] * a + x.x * f;
      O[e + 1] = O[e + 1] * a + x.y * f;
      O[e + 2] = O[e + 2] * a + x.z * f;
      O[e + 3] = O[e + 3] * a + x.w * f;
    }
    Mm = mn;
  }
  if (j < T) {
    const float inv = 1.0f / Lm;
#pragma unroll
    for (int e = 0; e < DPT; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack_bf16(O[e] * inv, O[e + 1] * inv);
  }
  if (threadIdx.x == 0) atomicExch(&p.ws_cnt[pair], 0);
}

// ------------------------------------------------- verify attention on tcgen05 (T = 5 .. 8)
// The same work split as verify_attn_kernel (one CTA per pair and split of the keys), with the
// arithmetic on the 5th-generation tensor cores. The pair's 4T query rows (row 4t + g: token t,
// head kvh * 4 + g; rows 4T .. 31 zero) fill 32 rows of a 128-row query tile, four times: copy w
// in rows 32w .. 32w + 31. S = Q K^T (M = 128, N = 128 keys) and O += P V (P from tensor memory)
// run as full-size tcgen05 MMAs, and the four copies split the softmax: warp w (tensor-memory
// lanes 32w ..) takes keys 32w .. 32w + 31 of each 128-key tile for its copy of the rows, with a
// row maximum shared through shared memory, and writes P for those keys only (zero elsewhere), so
// copy w's O and l are sums over its quarter of the keys; the four are added at the end. Keys go
// in tiles of 128 (8 pages) through a TMA ring; two S buffers, so the scores of tile j + 1
// are ready when the softmax of tile j ends. Per tile j the MMA order is O += P(j) V_j, then
// S(j + 2) into the buffer P(j) came from (the MMAs of one thread execute in issue order, and a
// commit tracks every MMA issued before it). K tiles are read two tiles before their V tiles, so
// the ring holds 2 K slots and 4 V slots: each copy then starts two to four tiles ahead of its use.
// The running maximum moves only when a row's maximum
// grows by more than 2^8. The epilogue writes the output when the pair has one split, else the
// split's partial (m, l, O), and the split that finishes last merges them. Launched with
// programmatic dependent launch (KOPT_PLAN_OVERLAP_PREV), the producer copies the tiles whose keys
// are all below pos before it waits for the previous kernel; the query rows, the rows at pos ..
// pos + T - 1 and the outputs are only touched after the wait.
//   warps 0-3  softmax, epilogue, merge;   warp 4  TMA producer;   warp 5  tensor memory + MMAs.
constexpr int kTcKeys = 128;
constexpr int kTcKStages = 2;                // K slots (a K tile is done with after its S)
constexpr int kTcVStages = 4;                // V slots (held until the P V two tiles later)
constexpr int kTcRows = 32;                  // query rows held (4 T <= 32)
constexpr int kTcSoft = 4;                   // softmax warps = row copies
constexpr int kTcThreads = 6 * 32;
constexpr uint32_t kTcCols = 512;            // S0, S1, O: 128 fp32 columns each
constexpr int kTcHalf = 128 * 64;            // elements of one 64-dim half of a 128-row tile
constexpr uint32_t kTcHalfBytes = kTcHalf * 2;
constexpr float kTcRescale = 8.f;
// kind::f16: fp32 accumulator, bf16 A and B, A K-major; M = 128, N = 128; B K-major (S) or
// MN-major (bit 16: V with dims contiguous)
constexpr uint32_t kTcIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kTcIdescO = kTcIdescS | (1u << 16);

struct __align__(1024) TcSmem {
  bf16 q[2][kTcHalf];                        // query tile: [dims half][128 rows][64], swizzled
  bf16 k[kTcKStages][2][kTcHalf];            // key tiles: [dims half][128 keys][64]
  bf16 v[kTcVStages][2][kTcHalf];            // value tiles, same layout (MN-major operand)
  float red[2][kTcSoft][kTcRows];            // per tile parity: each copy's row maxima
  float lsum[kTcSoft][kTcRows];              // each copy's row sums at the end
  unsigned long long kfull[kTcKStages], kempty[kTcKStages], vfull[kTcVStages], vempty[kTcVStages];
  unsigned long long sfull[2], pfull[2], pvdone[2], odone, drain;
  unsigned long long redbar[2], epibar, partbar, lastbar;   // among the softmax warps (bounded)
  unsigned long long qready;                                // the query tile is in
  uint32_t tmem;
  int last;
  volatile int abort;
};
constexpr size_t kTcSmemBytes = sizeof(TcSmem) + 1024;
static_assert(kTcSmemBytes <= 232448, "verify (tcgen05) shared memory above the per-CTA limit");
static_assert(sizeof(float) * kTcSoft * kTcRows * kD <= sizeof(bf16) * kTcKStages * 2 * kTcHalf,
              "the copies' outputs do not fit in the key ring");

template <bool PAGED>
__global__ void __launch_bounds__(kTcThreads, 1) verify_tc_kernel(const __grid_constant__ Params p) {
  extern __shared__ unsigned char smem_raw[];
  TcSmem& s = *reinterpret_cast<TcSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.nkv * kGroup;
  const int split = blockIdx.x % p.nsplit;
  const int pair = blockIdx.x / p.nsplit;
  const int b = pair / p.nkv, kvh = pair % p.nkv;
  const int T = p.T;                                    // 4 T <= kTcRows
  int p0 = p.pos[b];
  if (p0 < 0 || p0 + T > p.cap) {
    if (threadIdx.x == 0 && split == 0 && kvh == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_LEN);
    p0 = min(max(p0, 0), p.cap - T);
  }
  const int Lb = p0 + T;                                // keys the last query sees
  const int per = ceil_div_i(ceil_div_i(Lb, p.nsplit), kPage) * kPage;
  const int s0 = split * per, s1 = min(Lb, s0 + per);   // this split's keys (s0 on a page edge)
  const int pg0 = s0 / kPage;
  const int pg1 = s1 > s0 ? ceil_div_i(s1, kPage) : pg0;   // pages [pg0, pg1)
  const int nt = ceil_div_i(pg1 - pg0, kTcKeys / kPage);   // key tiles

  if (threadIdx.x == 0) {
    for (int i = 0; i < kTcKStages; ++i) {
      mbar_init(smem_u32(&s.kfull[i]), 1);
      mbar_init(smem_u32(&s.kempty[i]), 1);
    }
    for (int i = 0; i < kTcVStages; ++i) {
      mbar_init(smem_u32(&s.vfull[i]), 1);
      mbar_init(smem_u32(&s.vempty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s.sfull[i]), 1);
      mbar_init(smem_u32(&s.pfull[i]), 32 * kTcSoft);
      mbar_init(smem_u32(&s.pvdone[i]), 1);
    }
    mbar_init(smem_u32(&s.odone), 1);
    mbar_init(smem_u32(&s.drain), 1);
    mbar_init(smem_u32(&s.redbar[0]), 32 * kTcSoft);
    mbar_init(smem_u32(&s.redbar[1]), 32 * kTcSoft);
    mbar_init(smem_u32(&s.epibar), 32 * kTcSoft);
    mbar_init(smem_u32(&s.partbar), 32 * kTcSoft);
    mbar_init(smem_u32(&s.lastbar), 1);
    mbar_init(smem_u32(&s.qready), 32 * kTcSoft);
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(&s.tmem), kTcCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  if (warp < kTcSoft) {
    griddep_wait();   // q and the rows at pos .. are the previous kernel's
    // the query tile in the 128-byte-swizzled K-major layout (16-byte chunk c of row r at
    // c ^ (r % 8)): row r holds query row r % 32 (zero past 4 T)
    for (int i = threadIdx.x; i < 128 * 16; i += 32 * kTcSoft) {
      const int r = i >> 4, c = i & 15;              // row, 16-byte chunk of its 256 bytes
      const int qr = r % kTcRows, t = qr / kGroup, g = qr % kGroup;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (qr < kGroup * T)
        val = *reinterpret_cast<const uint4*>(p.q + (static_cast<long long>(b) * T + t) * nq * kD +
                                              (kvh * kGroup + g) * kD + c * 8);
      const int h = c >> 3, cc = c & 7;
      *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&s.q[h][0]) + r * 128 + ((cc ^ (r & 7)) << 4)) = val;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the MMA reads it
    mbar_arrive(smem_u32(&s.qready));
  }
  griddep_launch_dependents();

  if (warp == 4) {
    // ---- producer warp: K and V tiles of 8 pages, lane i copying page i of the tile (its id read
    // two tiles ahead, so the id loads are off the path of the copies); lane 0 waits for the slots
    // and sets the byte counts
    const uint64_t pol = evict_first_policy();
    constexpr int kTP = kTcKeys / kPage;
    const int* bt_row = PAGED ? p.bt + static_cast<long long>(b) * p.bt_stride : nullptr;
    auto fetch = [&](int j) {
      const int pg = pg0 + j * kTP + lane;
      return (PAGED && lane < kTP && pg < pg1) ? __ldg(bt_row + pg) : 0;
    };
    int nxt = nt > 0 ? fetch(0) : 0, nxt2 = nt > 1 ? fetch(1) : 0;
    int t = 0;
    bool ok = true, waited = false;
    for (; t < nt; ++t) {
      if (!waited && min(s1, s0 + (t + 1) * kTcKeys) > p0) {   // rows at pos and past: after the wait
        griddep_wait();
        waited = true;
      }
      const int npg = min(kTP, pg1 - pg0 - t * kTP);
      int row = 0;
      if (PAGED) {
        int pid = nxt;
        if (lane < npg && (pid < 0 || pid >= p.num_pages)) {   // recorded; a valid page keeps the count
          atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
          pid = 0;
        }
        row = (pid * p.nkv + kvh) * kPage;
        nxt = nxt2;
        if (t + 2 < nt) nxt2 = fetch(t + 2);
      }
      const int key = (pg0 + t * kTP + lane) * kPage;
      for (int kv = 0; kv < 2; ++kv) {
        unsigned long long* empty = kv == 0 ? s.kempty : s.vempty;
        unsigned long long* full = kv == 0 ? s.kfull : s.vfull;
        const int ns = kv == 0 ? kTcKStages : kTcVStages, st = t % ns, use = t / ns;
        ok = __all_sync(0xffffffffu, t < ns ||
                        mbar_wait(smem_u32(&empty[st]), (use - 1) & 1, s, p.ws_err, true));
        if (!ok) break;
        if (lane == 0) mbar_arrive_expect_tx(smem_u32(&full[st]), static_cast<uint32_t>(npg) * 2u * kBoxBytes);
        __syncwarp();
        if (lane < npg) {
          const CUtensorMap* map = kv == 0 ? &p.tmk : &p.tmv;
          bf16 (*dst)[kTcHalf] = kv == 0 ? s.k[st] : s.v[st];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t d = smem_u32(&dst[h][lane * kPage * kHalf]);
            if (PAGED) tma_load_2d(d, map, h * kHalf, row, smem_u32(&full[st]), pol);
            else tma_load_4d(d, map, h * kHalf, key, kvh, b, smem_u32(&full[st]), pol);
          }
        }
      }
      if (!ok) break;
    }
    // every copy issued has landed (the newest phase of each slot; after an abort the tile whose
    // V was not issued waits out its bound)
    if (lane == 0) {
      const int te = min(t + (ok ? 0 : 1), nt);
      for (int k = max(te - kTcKStages, 0); k < te; ++k)
        mbar_wait(smem_u32(&s.kfull[k % kTcKStages]), (k / kTcKStages) & 1, s, p.ws_err, false);
      for (int k = max(te - kTcVStages, 0); k < te; ++k)
        mbar_wait(smem_u32(&s.vfull[k % kTcVStages]), (k / kTcVStages) & 1, s, p.ws_err, false);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      // ---- MMAs: S(0), S(1), then per tile j: O += P(j) V_j, S(j + 2)
      auto issue_s = [&](int j) {
        const uint32_t qa = smem_u32(&s.q[0][0]), ka = smem_u32(&s.k[j % kTcKStages][0][0]);
#pragma unroll
        for (int kk = 0; kk < kD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kTcHalfBytes + (kk & 3) * 32;
          umma_bf16(tmem + 128u * (j & 1), sw128_desc(qa + off), sw128_desc(ka + off), kTcIdescS, kk > 0);
        }
        umma_commit(smem_u32(&s.sfull[j & 1]));
        umma_commit(smem_u32(&s.kempty[j % kTcKStages]));
      };
      bool ok = nt == 0 || mbar_wait(smem_u32(&s.qready), 0, s, p.ws_err, true);
      for (int j = 0; ok && j < 2 && j < nt; ++j) {
        if (!mbar_wait(smem_u32(&s.kfull[j % kTcKStages]), (j / kTcKStages) & 1, s, p.ws_err, true)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(j);
      }
      for (int j = 0; ok && j < nt; ++j) {
        if (!mbar_wait(smem_u32(&s.pfull[j & 1]), (j >> 1) & 1, s, p.ws_err, true) ||
            !mbar_wait(smem_u32(&s.vfull[j % kTcVStages]), (j / kTcVStages) & 1, s, p.ws_err, true))
          break;
        tc_fence_after();
        const uint32_t va = smem_u32(&s.v[j % kTcVStages][0][0]);
#pragma unroll
        for (int kk = 0; kk < kTcKeys / 16; ++kk)
          umma_bf16_ts(tmem + 256u, tmem + 128u * (j & 1) + 8 * kk,
                       sw128_mn_desc(va + kk * 16 * 128, kTcHalfBytes, 1024), kTcIdescO,
                       (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(smem_u32(&s.pvdone[j & 1]));
        umma_commit(smem_u32(&s.vempty[j % kTcVStages]));
        if (j == nt - 1) umma_commit(smem_u32(&s.odone));
        if (j + 2 < nt) {
          if (!mbar_wait(smem_u32(&s.kfull[(j + 2) % kTcKStages]), ((j + 2) / kTcKStages) & 1, s, p.ws_err, true))
            break;
          tc_fence_after();
          issue_s(j + 2);
        }
      }
      umma_commit(smem_u32(&s.drain));
      mbar_wait(smem_u32(&s.drain), 0, s, p.ws_err, false);
    }
    __syncwarp();
  } else {
    // ---- warps 0-3: warp w holds copy w of row r = lane (token r / 4, head kvh * 4 + r % 4) in
    // tensor-memory lane 32 w + r and takes keys 32 w .. 32 w + 31 of each tile
    const int w = warp, r = lane;
    const uint32_t lq = tmem + (static_cast<uint32_t>(32 * w) << 16);
    const int lim = r < kGroup * T ? p0 + r / kGroup : 0x7fffffff;   // last key the row sees
    float m = kNegBig, l = 0.f;
    bool ok = true;
    uint32_t zero[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) zero[e] = 0u;
    for (int j = 0; j < nt; ++j) {
      const int bb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.sfull[bb]), (j >> 1) & 1, s, p.ws_err, true));
      if (!ok) break;
      tc_fence_after();
      float sv[32];
      tmem_ld32(lq + 128u * bb + 32u * w, sv);
      const int key0 = s0 + j * kTcKeys + 32 * w;   // this warp's first key in the tile
      if (key0 + 32 > s1 || key0 + 31 > lim) {       // keys past the split or the row
        const int cl = min(s1 - 1, lim) - key0;
#pragma unroll
        for (int c = 0; c < 32; ++c)
          if (c > cl) sv[c] = -INFINITY;
      }
      float mx0 = sv[0], mx1 = sv[1];
#pragma unroll
      for (int c = 2; c < 32; c += 2) {
        mx0 = fmaxf(mx0, sv[c]);
        mx1 = fmaxf(mx1, sv[c + 1]);
      }
      s.red[bb][w][r] = fmaxf(mx0, mx1);
      mbar_arrive(smem_u32(&s.redbar[bb]));   // every copy's maximum of this tile is in
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.redbar[bb]), (j >> 1) & 1, s, p.ws_err, true));
      if (!ok) break;
      const float mx = fmaxf(fmaxf(s.red[bb][0][r], s.red[bb][1][r]), fmaxf(s.red[bb][2][r], s.red[bb][3][r])) *
                       p.scale_log2;
      const bool need = mx > m + kTcRescale;
      float alpha = 1.f;
      if (need) {
        alpha = ex2_fast(m - mx);
        m = mx;
        l *= alpha;
      }
      uint32_t pk[16];
      float sum0 = 0.f, sum1 = 0.f;
      const float nm = -m;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float a0 = ex2_fast(fmaf(sv[2 * e], p.scale_log2, nm));
        const float a1 = ex2_fast(fmaf(sv[2 * e + 1], p.scale_log2, nm));
        sum0 += a0;
        sum1 += a1;
        pk[e] = pack_bf16(a0, a1);
      }
      l += sum0 + sum1;
      // P of this copy over the first 64 columns: its keys' words 16 w .. 16 w + 15, zero elsewhere
#pragma unroll
      for (int q = 0; q < kTcSoft; ++q) tmem_st16u(lq + 128u * bb + 16u * q, q == w ? pk : zero);
      if (__any_sync(0xffffffffu, need) && j > 0) {
        // this copy's O row *= alpha, once the previous P V has completed
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.pvdone[bb ^ 1]), ((j - 1) >> 1) & 1, s, p.ws_err, true));
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kD; c += 32) {
          float o[32];
          tmem_ld32(lq + 256u + c, o);
#pragma unroll
          for (int q = 0; q < 32; ++q) o[q] *= alpha;
          tmem_st32(lq + 256u + c, o);
        }
      }
      if (s0 + (j + 1) * kTcKeys > s1) {
        // V rows past the split's keys may hold anything: zero them so 0 * V stays 0
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.vfull[j % kTcVStages]), (j / kTcVStages) & 1, s, p.ws_err, true));
        if (!ok) break;
        const int nv = s1 - (s0 + j * kTcKeys);
        for (int i = nv * 16 + 32 * w + lane; i < kTcKeys * 16; i += 32 * kTcSoft) {
          const int rr = i >> 4, part = i & 15;
          const uint32_t a = smem_u32(&s.v[j % kTcVStages][part >> 3][0]) + rr * 128 + ((part & 7) << 4);
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a), "r"(0u) : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&s.pfull[bb]));
    }
    // ---- epilogue: add the four copies (through the key ring, free once the last P V is done);
    // warp w then owns dims 32 w .. 32 w + 31 of row r
    float* ob = reinterpret_cast<float*>(&s.k[0][0][0]);   // [copy][row][kD]
    float O[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) O[c] = 0.f;
    float L = 0.f;
    const bool have = ok && nt > 0;
    if (have) {
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.odone), 0, s, p.ws_err, true));
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kD; c += 32) {
          float o[32];
          tmem_ld32(lq + 256u + c, o);
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(&ob[(w * kTcRows + r) * kD + c + e]) = make_float4(o[e], o[e + 1], o[e + 2], o[e + 3]);
        }
        s.lsum[w][r] = l;
      }
    }
    mbar_arrive(smem_u32(&s.epibar));
    ok = __all_sync(0xffffffffu, ok && mbar_wait(smem_u32(&s.epibar), 0, s, p.ws_err, true));
    const bool good = ok && have;
    if (good) {
#pragma unroll
      for (int q = 0; q < kTcSoft; ++q) {
        L += s.lsum[q][r];
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          const float4 x = *reinterpret_cast<const float4*>(&ob[(q * kTcRows + r) * kD + 32 * w + e]);
          O[e] += x.x;
          O[e + 1] += x.y;
          O[e + 2] += x.z;
          O[e + 3] += x.w;
        }
      }
    }
    const int t = r / kGroup, g = r % kGroup;
    bf16* dst = p.out + ((static_cast<long long>(b) * T + t) * nq + kvh * kGroup + g) * kD + 32 * w;
    if (p.nsplit == 1) {
      if (good && r < kGroup * T) {
        const float inv = 1.0f / L;
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 u;
          u.x = pack_bf16(O[c] * inv, O[c + 1] * inv);
          u.y = pack_bf16(O[c + 2] * inv, O[c + 3] * inv);
          u.z = pack_bf16(O[c + 4] * inv, O[c + 5] * inv);
          u.w = pack_bf16(O[c + 6] * inv, O[c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + c) = u;
        }
      }
    } else {
      // the split's partial (every split writes one, so the counts add up), then the merge
      const long long slot = blockIdx.x;
      float* po = p.ws_o + (slot * kTcRows + r) * kD + 32 * w;
#pragma unroll
      for (int c = 0; c < 32; c += 4) *reinterpret_cast<float4*>(po + c) = make_float4(O[c], O[c + 1], O[c + 2], O[c + 3]);
      if (w == 0) p.ws_ml[slot * kTcRows + r] = make_float2(good ? m : kNegBig, good ? L : 0.f);
      __threadfence();
      mbar_arrive(smem_u32(&s.partbar));
      if (threadIdx.x == 0) {
        s.last = mbar_wait(smem_u32(&s.partbar), 0, s, p.ws_err, false) &&
                 atomicAdd(&p.ws_cnt[pair], 1) == p.nsplit - 1;
        if (s.last) __threadfence();   // acquire the other splits' partials
        mbar_arrive(smem_u32(&s.lastbar));
      }
      const bool merge = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.lastbar), 0, s, p.ws_err, false)) && s.last;
      if (merge) {   // online log-sum-exp over every split's partial
        const long long first = blockIdx.x - split;
        float Mm = kNegBig, Lm = 0.f;
#pragma unroll
        for (int c = 0; c < 32; ++c) O[c] = 0.f;
        for (int sp = 0; sp < p.nsplit; ++sp) {
          const long long sl = first + sp;
          const float2 ml = __ldcg(&p.ws_ml[sl * kTcRows + r]);
          const float mn = fmaxf(Mm, ml.x);
          const float a = exp2f(Mm - mn), f = exp2f(ml.x - mn);
          Lm = Lm * a + ml.y * f;
          const float* src = p.ws_o + (sl * kTcRows + r) * kD + 32 * w;
#pragma unroll
          for (int c = 0; c < 32; c += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(src + c));
            O[c] = O[c] * a + x.x * f;
            O[c + 1] = O[c + 1] * a + x.y * f;
            O[c + 2] = O[c + 2] * a + x.z * f;
            O[c + 3] = O[c + 3] * a + x.w * f;
          }
          Mm = mn;
        }
        if (r < kGroup * T) {
          const float inv = 1.0f / Lm;
#pragma unroll
          for (int c = 0; c < 32; c += 8) {
            uint4 u;
            u.x = pack_bf16(O[c] * inv, O[c + 1] * inv);
            u.y = pack_bf16(O[c + 2] * inv, O[c + 3] * inv);
            u.z = pack_bf16(O[c + 4] * inv, O[c + 5] * inv);
            u.w = pack_bf16(O[c + 6] * inv, O[c + 7] * inv);
            *reinterpret_cast<uint4*>(dst + c) = u;
          }
        }
        if (threadIdx.x == 0) atomicExch(&p.ws_cnt[pair], 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kTcCols);
  }
}

// ------------------------------------------------------------------------------ host side

struct WsLayout {
  int64_t err, cnt, ml, o, total;
};
// counters: one per pair; partials: rows per slot = 4 (T = 1) or 16 / 32 (verify, T <= 4 / 8)
inline WsLayout ws_layout(int B, int nkv, int max_units, int T = 1) {
  const int rows = T > 1 ? 16 * verify_tiles(T) : kGroup;
  WsLayout w;
  w.err = 0;
  w.cnt = kHeaderBytes;
  w.ml = w.cnt + align256(static_cast<int64_t>(B) * nkv * 4);
  w.o = w.ml + align256(static_cast<int64_t>(max_units) * rows * 8);
  w.total = w.o + static_cast<int64_t>(max_units) * rows * kD * 4;
  return w;
}
inline WsLayout ws_layout(const kopt_plan* plan) {
  return ws_layout(plan->B, plan->nkv, plan->max_units, plan->T);
}

template <bool PAGED, bool FUSED>
int attn_occupancy(int device, int* blocks_per_sm) {
  static int configured[64] = {0};
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  auto kern = decode_attn_kernel<PAGED, FUSED>;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess)
      return KOPT_ERR_CUDA;
    configured[device] = 1;
  }
  if (blocks_per_sm) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kern, kThreads, kSmemBytes) !=
        cudaSuccess)
      return KOPT_ERR_CUDA;
  }
  return KOPT_OK;
}



int fill_cache(Params& p, const kopt_kv_cache* c) {
  if (c == nullptr || c->k == nullptr || c->v == nullptr) return KOPT_ERR_ARG;
  if (!aligned16(c->k) || !aligned16(c->v)) return KOPT_ERR_ARG;
  if (c->cap < 1) return KOPT_ERR_ARG;
  p.kc = static_cast<bf16*>(c->k);
  p.vc = static_cast<bf16*>(c->v);
  p.cap = c->cap;
  if (c->block_table != nullptr) {
    if (c->page_size != kPage || c->bt_stride < 1 || c->num_pages < 1) return KOPT_ERR_ARG;
    if (static_cast<long long>(c->bt_stride) * kPage < c->cap) return KOPT_ERR_ARG;
    p.bt = c->block_table;
    p.bt_stride = c->bt_stride;
    p.num_pages = c->num_pages;
    p.sb = p.sh = 0;
  } else {
    if ((c->stride_b % 8) != 0 || (c->stride_h % 8) != 0) return KOPT_ERR_ARG;
    p.bt = nullptr;
    p.bt_stride = 0;
    p.num_pages = 0;
    p.sb = c->stride_b;
    p.sh = c->stride_h;
  }
  return KOPT_OK;
}


// TMA maps over the K and V caches. Box = 16 tokens x 64 dims (128 B rows, 128-byte swizzle).
//   paged:      2-D {128 dims, num_pages * nkv * 16 rows}, row stride 256 B
//   contiguous: 4-D {128 dims, cap, nkv, B}, strides {256 B, stride_h * 2, stride_b * 2}
// Out-of-range boxes (past cap) are zero-filled by the hardware.
int encode_kv_maps(Params& p, int B, int nkv) {
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return KOPT_ERR_CUDA;
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  cuuint32_t box[4] = {kHalf, kPage, 1, 1};
  cuuint32_t rank;
  if (p.bt != nullptr) {
    const unsigned long long rows = static_cast<unsigned long long>(p.num_pages) * nkv * kPage;
    if (rows >= (1ull << 31)) return KOPT_ERR_ARG;
    rank = 2;
    dims[0] = kD;
    dims[1] = rows;
    strides[0] = kD * 2;
  } else {
    rank = 4;
    dims[0] = kD;
    dims[1] = static_cast<cuuint64_t>(p.cap);
    dims[2] = static_cast<cuuint64_t>(nkv);
    dims[3] = static_cast<cuuint64_t>(B);
    strides[0] = kD * 2;
    strides[1] = static_cast<cuuint64_t>(p.sh) * 2;
    strides[2] = static_cast<cuuint64_t>(p.sb) * 2;
  }
  for (int which = 0; which < 2; ++which) {
    CUtensorMap* map = which == 0 ? &p.tmk : &p.tmv;
    void* base = which == 0 ? static_cast<void*>(p.kc) : static_cast<void*>(p.vc);
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, base, dims, strides, box,
                           elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return KOPT_ERR_ARG;
  }
  return KOPT_OK;
}

// A plan is a plain struct that the caller may have edited or kept from another shape: its
// fields must agree with each other before they size a launch. The kernels index the workspace by
// chunk + pair (T = 1; chunks < grid + ceil(pages / 32)) or by CTA (T > 1), so grid, max_units and
// the shape must be those kopt_decode_attn_plan would give together.
int check_plan(const kopt_plan* plan) {
  if (plan->B < 1 || plan->B > kMaxB || plan->T < 1 || plan->T > kVMaxT || plan->nkv < 1 ||
      plan->grid < 1 || plan->max_len < 1 || plan->max_units < 1)
    return KOPT_ERR_ARG;
  const long long pairs = static_cast<long long>(plan->B) * plan->nkv;
  if (plan->T > 1) {
    if (plan->grid % pairs != 0 || plan->grid > plan->max_units) return KOPT_ERR_ARG;
    return KOPT_OK;
  }
  const long long pages = pairs * ((static_cast<long long>(plan->max_len) + kPage - 1) / kPage);
  const long long units = plan->grid + (pages + kChunkPages - 1) / kChunkPages + pairs;
  return units <= plan->max_units ? KOPT_OK : KOPT_ERR_ARG;
}

int fill_ws(Params& p, const kopt_plan* plan, void* ws) {
  if (check_plan(plan) != KOPT_OK) return KOPT_ERR_ARG;
  if (ws == nullptr || (reinterpret_cast<uintptr_t>(ws) & 255) != 0) return KOPT_ERR_WORKSPACE;
  const WsLayout w = ws_layout(plan);
  if (w.total != plan->ws_bytes) return KOPT_ERR_WORKSPACE;
  char* base = static_cast<char*>(ws);
  p.ws_err = reinterpret_cast<int*>(base + w.err);
  p.ws_cnt = reinterpret_cast<int*>(base + w.cnt);
  p.ws_ml = reinterpret_cast<float2*>(base + w.ml);
  p.ws_o = reinterpret_cast<float*>(base + w.o);
  return KOPT_OK;
}

template <bool PAGED, bool FUSED>
int launch_attn(const kopt_plan* plan, Params& p, void* stream) {
  int rc = set_device(plan->device);
  if (rc) return rc;
  rc = attn_occupancy<PAGED, FUSED>(plan->device, nullptr);
  if (rc) return rc;
  if (plan->flags & ~KOPT_PLAN_OVERLAP_PREV) return KOPT_ERR_ARG;
  p.late_skew = (plan->flags & KOPT_PLAN_OVERLAP_PREV) ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (plan->flags & KOPT_PLAN_OVERLAP_PREV) ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, decode_attn_kernel<PAGED, FUSED>, p) != cudaSuccess) {
    cudaGetLastError();
    return KOPT_ERR_CUDA;
  }
  return KOPT_OK;
}

template <bool PAGED, int MT>
int verify_occupancy(int device, int* blocks_per_sm) {
  static int configured[64] = {0};
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  auto kern = verify_attn_kernel<PAGED, MT>;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(vsmem_bytes<MT>())) != cudaSuccess)
      return KOPT_ERR_CUDA;
    configured[device] = 1;
  }
  if (blocks_per_sm &&
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kern, verify_threads<MT>(),
                                                    vsmem_bytes<MT>()) != cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}
template <bool PAGED>
int verify_tc_occupancy(int device, int* blocks_per_sm) {
  static int configured[64] = {0};
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  auto kern = verify_tc_kernel<PAGED>;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kTcSmemBytes)) != cudaSuccess)
      return KOPT_ERR_CUDA;
    configured[device] = 1;
  }
  if (blocks_per_sm &&
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kern, kTcThreads, kTcSmemBytes) !=
          cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}
// T > 4 runs on the tensor-memory kernel (verify_tc_kernel), T <= 4 on verify_attn_kernel
inline bool verify_on_tc(int T) { return T > 4; }
int verify_configure(int device, int T, int* blocks_per_sm) {
  if (verify_on_tc(T)) {
    const int rc = verify_tc_occupancy<true>(device, blocks_per_sm);
    return rc ? rc : verify_tc_occupancy<false>(device, nullptr);
  }
  int rc = verify_tiles(T) == 1 ? verify_occupancy<true, 1>(device, blocks_per_sm)
                                : verify_occupancy<true, 2>(device, blocks_per_sm);
  if (rc) return rc;
  return verify_tiles(T) == 1 ? verify_occupancy<false, 1>(device, nullptr)
                              : verify_occupancy<false, 2>(device, nullptr);
}

template <bool PAGED, int MT>
int launch_verify_t(const kopt_plan* plan, Params& p, void* stream) {
  int rc = verify_occupancy<PAGED, MT>(plan->device, nullptr);
  if (rc) return rc;
  verify_attn_kernel<PAGED, MT><<<plan->grid, verify_threads<MT>(), vsmem_bytes<MT>(),
                                  static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}
template <bool PAGED>
int launch_verify(const kopt_plan* plan, Params& p, void* stream) {
  int rc = set_device(plan->device);
  if (rc) return rc;
  p.tblocks = 1;
  p.nsplit = plan->grid / (plan->B * plan->nkv);
  if (verify_on_tc(plan->T)) {
    rc = verify_tc_occupancy<PAGED>(plan->device, nullptr);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(plan->grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = kTcSmemBytes;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (plan->flags & KOPT_PLAN_OVERLAP_PREV) ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, verify_tc_kernel<PAGED>, p) != cudaSuccess) {
      cudaGetLastError();
      return KOPT_ERR_CUDA;
    }
    return KOPT_OK;
  }
  return verify_tiles(plan->T) == 1 ? launch_verify_t<PAGED, 1>(plan, p, stream)
                                    : launch_verify_t<PAGED, 2>(plan, p, stream);
}


}  // namespace kopt

// =================================================================================== C ABI
using namespace kopt;

extern "C" {

int kopt_abi_version(void) { return 2; }

const char* kopt_strerror(int status) {
  switch (status) {
    case KOPT_OK: return "ok";
    case KOPT_ERR_ARG: return "invalid argument (shape, head_dim, group, alignment or pointer)";
    case KOPT_ERR_CUDA: return "CUDA runtime call failed";
    case KOPT_ERR_WORKSPACE: return "workspace missing, misaligned or sized for another plan";
    case KOPT_ERR_SCRATCH:
      return "plan needs more split scratch than the 8 MiB built into the library (use "
             "kopt_decode_attn_fused with a caller-owned workspace)";
    default: return "unknown kopt status";
  }
}

int kopt_decode_attn_plan(int device, int B, int T, int nq, int nkv, int d, int max_len,
                          int target_ctas, kopt_plan* plan) {
  if (plan == nullptr) return KOPT_ERR_ARG;
  if (d != kD || nkv < 1 || nq != nkv * kGroup || B < 1 || B > kMaxB || T < 1 || T > kVMaxT ||
      max_len < 1)
    return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  int sms = 0, occ = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return KOPT_ERR_CUDA;
  if (T > 1) {   // verify: grid = pairs x key splits, one wave
    if (max_len < T) return KOPT_ERR_ARG;
    rc = verify_configure(device, T, &occ);
    if (rc) return rc;
    if (occ < 1) return KOPT_ERR_CUDA;
    const long long blocks = static_cast<long long>(B) * nkv;
    const long long max_split = (static_cast<long long>(max_len) + 2 * kPage - 1) / (2 * kPage);
    // one wave: each CTA pays a fixed cost for its q rows and its merge, so fewer and longer
    // splits win (measured: B=16, T=3, 4099 keys, 52 us at 256 CTAs, 72 us at 1152)
    const long long slots = target_ctas > 0 ? target_ctas : static_cast<long long>(sms) * occ;
    long long nsplit = slots / blocks;
    nsplit = nsplit < 1 ? 1 : nsplit > max_split ? max_split : nsplit;
    if (blocks * nsplit >= (1ll << 31)) return KOPT_ERR_ARG;
    plan->B = B;
    plan->T = T;
    plan->nkv = nkv;
    plan->grid = static_cast<int32_t>(blocks * nsplit);
    plan->ctas_per_sm = occ;
    plan->tile_tokens = kVW * kPage;
    plan->max_units = plan->grid;
    plan->device = device;
    plan->max_len = max_len;
    plan->chunk_tokens = static_cast<int32_t>((max_len + nsplit - 1) / nsplit);
    plan->static_pct = 100;
    plan->flags = 0;
    plan->ws_bytes = ws_layout(plan).total;
    return KOPT_OK;
  }
  rc = attn_occupancy<true, true>(device, &occ);
  if (rc) return rc;
  // the four instantiations share block size and shared memory, so one occupancy serves all
  rc = attn_occupancy<true, false>(device, nullptr);
  if (rc) return rc;
  rc = attn_occupancy<false, true>(device, nullptr);
  if (rc) return rc;
  rc = attn_occupancy<false, false>(device, nullptr);
  if (rc) return rc;
  if (occ < 1) return KOPT_ERR_CUDA;
  // slot = chunk + pair < grid + ceil(T / 32) + B * nkv, T = total pages at max_len
  const int grid = target_ctas > 0 ? target_ctas : sms * occ;
  const long long pages = static_cast<long long>(B) * nkv * ((static_cast<long long>(max_len) + kPage - 1) / kPage);
  if (pages >= (1ll << 31)) return KOPT_ERR_ARG;
  const long long units = grid + (pages + kChunkPages - 1) / kChunkPages + static_cast<long long>(B) * nkv;
  plan->B = B;
  plan->T = T;
  plan->nkv = nkv;
  plan->grid = grid;
  plan->ctas_per_sm = occ;
  plan->tile_tokens = kTile;
  plan->max_units = static_cast<int32_t>(units);
  plan->device = device;
  plan->max_len = max_len;
  plan->chunk_tokens = kChunkPages * kPage;
  plan->static_pct = kDefaultStaticPct;
  plan->flags = 0;
  if (const char* e = getenv("KOPT_STATIC_PCT")) {
    const int v = atoi(e);
    if (v >= 0 && v <= 100) plan->static_pct = v;
  }
  plan->ws_bytes = ws_layout(B, nkv, plan->max_units).total;
  return KOPT_OK;
}

int kopt_workspace_init(const kopt_plan* plan, void* ws, void* stream) {
  if (plan == nullptr || ws == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(plan->device);
  if (rc) return rc;
  const WsLayout w = ws_layout(plan);
  // error word and split counters; partials need no initial value
  if (cudaMemsetAsync(ws, 0, static_cast<size_t>(w.ml), static_cast<cudaStream_t>(stream)) !=
      cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}

int kopt_read_error(const kopt_plan* plan, void* ws, int* err_out, void* stream) {
  if (plan == nullptr || ws == nullptr || err_out == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(plan->device);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int host = 0;
  if (cudaMemcpyAsync(&host, ws, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return KOPT_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return KOPT_ERR_CUDA;
  *err_out = host;
  if (host != 0) {
    const WsLayout w = ws_layout(plan);
    if (cudaMemsetAsync(ws, 0, static_cast<size_t>(w.ml), st) != cudaSuccess) return KOPT_ERR_CUDA;
  }
  return KOPT_OK;
}

int kopt_decode_attn(const kopt_plan* plan, const void* q, const kopt_kv_cache* cache,
                     const int32_t* pos, void* out, void* ws, float scale, void* stream) {
  if (plan == nullptr || q == nullptr || pos == nullptr || out == nullptr) return KOPT_ERR_ARG;
  if (!aligned16(q) || !aligned16(out)) return KOPT_ERR_ARG;
  Params p{};
  int rc = fill_cache(p, cache);
  if (rc) return rc;
  if (p.cap > plan->max_len) return KOPT_ERR_ARG;
  rc = fill_ws(p, plan, ws);
  if (rc) return rc;
  p.q = static_cast<const bf16*>(q);
  p.pos = pos;
  p.out = static_cast<bf16*>(out);
  p.out_row = static_cast<long long>(plan->T) * plan->nkv * kGroup * kD;
  p.out_col = 0;
  p.world = 0;
  p.B = plan->B;
  p.T = plan->T;
  p.nkv = plan->nkv;
  p.static_pct = plan->static_pct;
  p.scale_log2 = scale * kLog2e;
  rc = set_device(plan->device);
  if (rc) return rc;
  rc = encode_kv_maps(p, plan->B, plan->nkv);
  if (rc) return rc;
  if (plan->T > 1) {
    if (p.cap < plan->T) return KOPT_ERR_ARG;
    return p.bt ? launch_verify<true>(plan, p, stream) : launch_verify<false>(plan, p, stream);
  }
  return p.bt ? launch_attn<true, false>(plan, p, stream) : launch_attn<false, false>(plan, p, stream);
}

}  // extern "C"

namespace {
// Shared by kopt_decode_attn_fused (g == nullptr: write `out`) and kopt_decode_attn_fused_gather.
int fused_launch(const kopt_plan* plan, const void* qkv, const void* q_norm_w, const void* k_norm_w,
                 const void* cos, const void* sin, int rope_len, const kopt_kv_cache* cache,
                 const int32_t* pos, void* out, const kopt_gather* g, void* q_out, void* ws,
                 float scale, float eps, void* stream, size_t clear_bytes = 0) {
  if (plan == nullptr || qkv == nullptr || q_norm_w == nullptr || k_norm_w == nullptr ||
      cos == nullptr || sin == nullptr || pos == nullptr || (g == nullptr && out == nullptr) ||
      rope_len < 1 || plan->T != 1)   // the fused prologue appends one token per sequence
    return KOPT_ERR_ARG;
  if (plan->flags & ~KOPT_PLAN_OVERLAP_PREV) return KOPT_ERR_ARG;
  if (!aligned16(qkv) || (out && !aligned16(out)) || (q_out && !aligned16(q_out)) ||
      !aligned16(cos) || !aligned16(sin) || (reinterpret_cast<uintptr_t>(q_norm_w) & 7) ||
      (reinterpret_cast<uintptr_t>(k_norm_w) & 7))
    return KOPT_ERR_ARG;
  Params p{};
  int rc = fill_cache(p, cache);
  if (rc) return rc;
  if (p.cap > plan->max_len) return KOPT_ERR_ARG;
  rc = fill_ws(p, plan, ws);
  if (rc) return rc;
  p.qkv = static_cast<const bf16*>(qkv);
  p.qw = static_cast<const bf16*>(q_norm_w);
  p.kw = static_cast<const bf16*>(k_norm_w);
  p.cos = static_cast<const bf16*>(cos);
  p.sin = static_cast<const bf16*>(sin);
  p.rope_len = rope_len;
  p.q_out = static_cast<bf16*>(q_out);
  p.pos = pos;
  const long long heads = static_cast<long long>(plan->nkv) * kGroup * kD;   // this rank's columns
  if (g == nullptr) {
    p.out = static_cast<bf16*>(out);
    p.out_row = static_cast<long long>(plan->T) * heads;
    p.out_col = 0;
    p.world = 0;
  } else {
    if (g->world < 1 || g->world > kMaxRanks || g->rank < 0 || g->rank >= g->world ||
        g->epoch == nullptr || g->row_elems < (g->rank + 1) * heads || g->row_elems % 8 != 0 ||
        plan->T != 1 || g->wait_ns < 0 || g->wait_ns > 10 * static_cast<long long>(kTimeoutNs))
      return KOPT_ERR_ARG;
    for (int w = 0; w < g->world; ++w) {
      if (g->out[w] == nullptr || g->flags[w] == nullptr || !aligned16(g->out[w]))
        return KOPT_ERR_ARG;
      p.out_peer[w] = static_cast<bf16*>(g->out[w]);
      p.flag_peer[w] = g->flags[w];
    }
    p.out = nullptr;
    p.epoch = g->epoch;
    p.rank = g->rank;
    p.world = g->world;
    p.out_row = g->row_elems;
    p.out_col = static_cast<int>(g->rank * heads);
    p.wait_ns = g->wait_ns > 0 ? static_cast<unsigned long long>(g->wait_ns) : kTimeoutNs;
  }
  p.B = plan->B;
  p.T = plan->T;
  p.nkv = plan->nkv;
  p.static_pct = plan->static_pct;
  p.scale_log2 = scale * kLog2e;
  p.eps = eps;
  rc = set_device(plan->device);
  if (rc) return rc;
  rc = encode_kv_maps(p, plan->B, plan->nkv);
  if (rc) return rc;
  // every argument is checked: only now may a clear of the workspace header go on the stream
  if (clear_bytes > 0 &&
      cudaMemsetAsync(ws, 0, clear_bytes, static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return KOPT_ERR_CUDA;
  return p.bt ? launch_attn<true, true>(plan, p, stream) : launch_attn<false, true>(plan, p, stream);
}
}  // namespace

extern "C" {

int kopt_decode_attn_fused(const kopt_plan* plan, const void* qkv, const void* q_norm_w,
                           const void* k_norm_w, const void* cos, const void* sin, int rope_len,
                           const kopt_kv_cache* cache, const int32_t* pos, void* out, void* q_out,
                           void* ws, float scale, float eps, void* stream) {
  return fused_launch(plan, qkv, q_norm_w, k_norm_w, cos, sin, rope_len, cache, pos, out, nullptr,
                      q_out, ws, scale, eps, stream);
}

int kopt_decode_attn_fused_gather(const kopt_plan* plan, const void* qkv, const void* q_norm_w,
                                  const void* k_norm_w, const void* cos, const void* sin,
                                  int rope_len, const kopt_kv_cache* cache, const int32_t* pos,
                                  const kopt_gather* gather, void* q_out, void* ws, float scale,
                                  float eps, void* stream) {
  if (gather == nullptr) return KOPT_ERR_ARG;
  return fused_launch(plan, qkv, q_norm_w, k_norm_w, cos, sin, rope_len, cache, pos, nullptr,
                      gather, q_out, ws, scale, eps, stream);
}

int kopt_ipc_alloc(int device, int64_t bytes, void** ptr) {
  if (ptr == nullptr || bytes <= 0) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  if (cudaMalloc(ptr, static_cast<size_t>(bytes)) != cudaSuccess) return KOPT_ERR_CUDA;
  if (cudaMemset(*ptr, 0, static_cast<size_t>(bytes)) != cudaSuccess) return KOPT_ERR_CUDA;
  return cudaDeviceSynchronize() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

int kopt_ipc_free(int device, void* ptr) {
  if (ptr == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  return cudaFree(ptr) == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

int kopt_ipc_get_handle(const void* ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == KOPT_IPC_HANDLE_BYTES, "IPC handle size");
  if (ptr == nullptr || handle == nullptr) return KOPT_ERR_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return KOPT_ERR_CUDA;
  memcpy(handle, &h, sizeof(h));
  return KOPT_OK;
}

int kopt_ipc_open(int device, const void* handle, void** peer_ptr) {
  if (handle == nullptr || peer_ptr == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  if (cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}

int kopt_ipc_close(int device, void* peer_ptr) {
  if (peer_ptr == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  return cudaIpcCloseMemHandle(peer_ptr) == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

int kopt_qk_norm_rope(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                      const void* cos, const void* sin, int rope_len, const int32_t* pos,
                      void* q_out, const kopt_kv_cache* cache, int B, int T, int nq, int nkv,
                      int d, float eps, int* dev_err, int device, void* stream) {
  if (d != kD || nkv < 1 || nq != nkv * kGroup || B < 1 || T < 1 || rope_len < 1) return KOPT_ERR_ARG;
  if (qkv == nullptr || q_norm_w == nullptr || k_norm_w == nullptr || cos == nullptr ||
      sin == nullptr || pos == nullptr || q_out == nullptr || dev_err == nullptr)
    return KOPT_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(qkv) & 7) || (reinterpret_cast<uintptr_t>(q_out) & 7) ||
      (reinterpret_cast<uintptr_t>(cos) & 7) || (reinterpret_cast<uintptr_t>(sin) & 7) ||
      (reinterpret_cast<uintptr_t>(q_norm_w) & 7) || (reinterpret_cast<uintptr_t>(k_norm_w) & 7))
    return KOPT_ERR_ARG;
  Params p{};
  int rc = fill_cache(p, cache);
  if (rc) return rc;
  rc = set_device(device);
  if (rc) return rc;
  p.qkv = static_cast<const bf16*>(qkv);
  p.qw = static_cast<const bf16*>(q_norm_w);
  p.kw = static_cast<const bf16*>(k_norm_w);
  p.cos = static_cast<const bf16*>(cos);
  p.sin = static_cast<const bf16*>(sin);
  p.rope_len = rope_len;
  p.q_out = static_cast<bf16*>(q_out);
  p.pos = pos;
  p.ws_err = dev_err;
  p.B = B;
  p.T = T;
  p.nkv = nkv;
  p.eps = eps;
  const int nheads = nq + 2 * nkv;
  dim3 grid(B * T, (nheads + 3) / 4);
  qk_norm_rope_kernel<<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p, nheads);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

}  // extern "C"

// ====================================================================== allocation-free variant
// Some callers cannot allocate device memory for the split scratch: an engine that owns the whole
// memory budget and hands out only fixed buffers, a process whose allocator must not grow after
// start-up, or a plugin host whose memory calls are not reachable from the attention call site.
// For them the scratch of kopt_decode_attn_fused lives in a buffer built into this library.
namespace {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;   // 8 MiB, held by every GPU using the library
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_scratch_mutex;
void* g_static_scratch_ptr[64] = {};   // device address of g_static_scratch, per device

// Device address of the built-in scratch on the current device (resolved once per device).
int static_scratch(int device, void** out) {
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_ptr[device] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_static_scratch) != cudaSuccess || ptr == nullptr)
      return KOPT_ERR_CUDA;
    g_static_scratch_ptr[device] = ptr;
  }
  *out = g_static_scratch_ptr[device];
  return KOPT_OK;
}

}  // namespace

extern "C" int kopt_decode_attn_fused_noalloc(
    const kopt_plan* plan, const void* qkv, const void* q_norm_w, const void* k_norm_w,
    const void* cos, const void* sin, int rope_len, const kopt_kv_cache* cache,
    const int32_t* pos, void* out, void* q_out, float scale, float eps, int* dev_err,
    void* stream) {
  if (plan == nullptr) return KOPT_ERR_ARG;
  // The plan is a plain struct the caller may have edited: its shape fields, not only ws_bytes,
  // decide how much of the buffer the kernel and the clear below touch, so they are checked
  // against each other and against the buffer before anything is queued.
  if (plan->T != 1 || check_plan(plan) != KOPT_OK) return KOPT_ERR_ARG;
  const WsLayout w = ws_layout(plan);
  if (w.total != plan->ws_bytes) return KOPT_ERR_WORKSPACE;
  if (w.total > static_cast<int64_t>(kStaticScratchBytes)) return KOPT_ERR_SCRATCH;
  int rc = set_device(plan->device);
  if (rc) return rc;
  void* ws = nullptr;
  rc = static_scratch(plan->device, &ws);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The buffer keeps the previous call's contents: the error word and the split counters must
  // start at zero (the partial-result slots need no initial value). The clear is queued by the
  // launch itself, after every argument has been checked, right before the kernel.
  rc = fused_launch(plan, qkv, q_norm_w, k_norm_w, cos, sin, rope_len, cache, pos, out, nullptr,
                    q_out, ws, scale, eps, stream, static_cast<size_t>(w.ml));
  if (rc) return rc;
  if (dev_err != nullptr &&
      cudaMemcpyAsync(dev_err, ws, sizeof(int), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}
