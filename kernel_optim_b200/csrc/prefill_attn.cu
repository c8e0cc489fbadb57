// Causal GQA attention over a prompt (the prefill) on the 5th-generation tensor cores (sm_100a),
// behind the C ABI in include/kopt.h.
//
// What the reference does (GodRishUniverse/kernel_optim, engine/engine.py:343-386): per layer, after
// the q/k norm + RoPE of the prompt, F.scaled_dot_product_attention(q, k, v, is_causal=True) with
// GQA (engine.py:376-377), then the prompt's K/V go to the cache. Here the prologue writes the
// prompt's K/V straight into the (paged) cache and this kernel reads them from there.
//
// Persistent grid, one CTA per SM. A work item is one sequence, one kv head, one 128-row query
// tile and two of the kv head's four query heads (A and B): both query tiles sit at the same
// positions, so they need the same key tiles 0 .. qt (causal) and every K/V tile loaded serves
// both. Items are dealt round-robin, the longest (last query tiles) first. Per key tile j:
//   warp 8   TMA producer: the item's two query tiles, then K_j and V_j into a 2-deep ring
//            (128-byte swizzle; paged caches arrive as 16-row page boxes);
//   warp 9   allocates all 512 tensor-memory columns (S_A, S_B, O_A, O_B, fp32) and one thread
//            issues the MMAs in the order S_A(0) S_B(0), then per j: O_A += P_A(j) V_j,
//            S_A(j+1), O_B += P_B(j) V_j, S_B(j+1): while one softmax group works on its scores,
//            the tensor core computes the other group's. Each P V goes in two halves of 64 keys,
//            the first issued as soon as its half of P is written. S = Q K^T has M = 128 query rows,
//            N = 128 keys, K-major operands from shared memory; P V takes P from tensor memory
//            (the A operand) and V from shared memory as an MN-major operand;
//   warps 0-3 / 4-7: the softmax of tile A / B, one thread per query row (tensor-memory lane):
//            the row of S_j by tcgen05.ld, the diagonal tile masked, online softmax in fp32 in the
//            exp2 domain (packed two-lane FFMA / FADD), and P_j written back as bf16 pairs over
//            the first 64 columns of its S buffer by tcgen05.st, keys 0-63 handed over first.
//            The running maximum only moves when a row's maximum grows by more than 2^8, so O
//            is rescaled rarely, by the thread that needs it, before P_j is handed over; at the
//            end of the item O / l goes to the output as bf16.
// The MMAs of one thread execute in issue order, and a commit tracks every MMA issued before it:
// S_x(j+1) is issued after O_x += P_x(j) V_j, so when a softmax thread sees S_x(j+1) complete, the
// P V that read P_x(j) (same columns) is complete too, and O_x may be rescaled. Every wait is
// bounded in time; on expiry the kernel records KOPT_DEV_ERR_TIMEOUT, stops, waits (bounded) for
// what it issued and frees its tensor memory.

#include "common.cuh"

namespace kopt {
namespace {

constexpr int kPD = 128;                    // head dim
constexpr int kPGroup = 4;                  // query heads per kv head
constexpr int kPHeads = 2;                  // query heads (tiles A, B) per work item
constexpr int kPRows = 128;                 // query rows per tile: the MMAs' M
constexpr int kPKeys = 128;                 // keys per tile
constexpr int kPPage = 16;                  // tokens per cache page
constexpr int kPStages = 2;                 // K/V ring depth
constexpr int kPSoftWarps = 8;              // warps 0-3: rows of tile A, warps 4-7: rows of tile B
constexpr int kPProducer = 8;
constexpr int kPMma = 9;
constexpr int kPThreads = 10 * 32;
constexpr uint32_t kPCols = 512;            // tensor memory: S_A, S_B, O_A, O_B (128 columns each)
constexpr int kPHalf = kPRows * 64;         // elements of one 64-column half tile
constexpr uint32_t kPHalfBytes = kPHalf * 2;   // 16 KiB
constexpr float kPRescale = 8.f;            // log2 growth of a row's max that moves its running max
__host__ __device__ constexpr uint32_t col_s(int x) { return 128u * static_cast<uint32_t>(x); }
__host__ __device__ constexpr uint32_t col_o(int x) { return 256u + 128u * static_cast<uint32_t>(x); }

struct PrefillParams {
  CUtensorMap tmq;          // q [B*S, nq*128] as 4-D {128 dims, nq heads, S rows, B}: box {64, 1, 128, 1}
  CUtensorMap tmk;          // K cache: paged {128, pages*nkv*16} (box {64, 16}) or
  CUtensorMap tmv;          //   contiguous {128, cap, nkv, B} (box {64, 128, 1, 1}); V likewise
  bf16* out;                // [B*S, nq*128]
  const int* bt;            // block table (paged) or nullptr
  int* err;                 // device error word
  int bt_stride, num_pages;
  int B, S, nq, nkv, nqt;
  int items;                // nqt * B * nkv * 2 (query tile, sequence, kv head, head pair)
  float scale_log2;
};

struct __align__(1024) PSmem {
  bf16 q[kPHeads][2][kPHalf];       // the item's query tiles A, B: [dims 0-63 | 64-127][128 rows][64]
  bf16 k[kPStages][2][kPHalf];      // key tiles: [dims half][128 keys][64]
  bf16 v[kPStages][2][kPHalf];      // value tiles, same layout (read as an MN-major operand)
  unsigned long long qfull, qempty;
  unsigned long long kfull[kPStages], vfull[kPStages], kempty[kPStages], vempty[kPStages];
  unsigned long long sfull[kPHeads], plo[kPHeads], pfull[kPHeads], odone[kPHeads], oempty[kPHeads];
  unsigned long long drain;
  uint32_t tmem;
  volatile int abort;
};
constexpr size_t kPSmemBytes = sizeof(PSmem) + 1024;
static_assert(kPSmemBytes <= 232448, "prefill shared memory above the 227 KiB per-CTA limit");

// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, A K-major, B K-major (S) or
// MN-major (bit 16: V with dims contiguous), N = 128 (bits 17-22: N >> 3), M = 128 (24-28: M >> 4).
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((kPKeys >> 3) << 17) |
                             ((kPRows >> 4) << 24);
constexpr uint32_t kIdescO = kIdescS | (1u << 16);

// This CTA's work items: item w = blockIdx.x + i * gridDim.x of the list ordered longest first
// (query tile qt = nqt - 1 down to 0; within a tile sequence-major, then kv head, then head pair,
// so neighbouring items share their K/V tiles in L2).
struct Item {
  int b, kvh, h0, q0, nt;   // query heads h0 (tile A) and h0 + 1 (tile B)
};
__device__ __forceinline__ Item item_of(const PrefillParams& p, int w) {
  const int per_qt = p.B * p.nkv * kPHeads;
  const int qt = p.nqt - 1 - w / per_qt;
  const int rem = w - (w / per_qt) * per_qt;
  const int pairs_b = p.nkv * kPHeads;
  Item it;
  it.b = rem / pairs_b;
  const int r2 = rem - it.b * pairs_b;
  it.kvh = r2 / kPHeads;
  it.h0 = it.kvh * kPGroup + (r2 - it.kvh * kPHeads) * kPHeads;
  it.q0 = qt * kPRows;
  it.nt = qt + 1;   // causal: key tiles 0 .. qt
  return it;
}

// Two fp32 lanes per instruction (sm_100 packed FFMA / FADD).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

template <bool PAGED>
__global__ void __launch_bounds__(kPThreads, 1) prefill_attn_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ unsigned char smem_raw[];
  PSmem& s = *reinterpret_cast<PSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&s.qfull), 1);
    mbar_init(smem_u32(&s.qempty), 1);
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(smem_u32(&s.kfull[i]), 1);
      mbar_init(smem_u32(&s.vfull[i]), 1);
      mbar_init(smem_u32(&s.kempty[i]), 1);
      mbar_init(smem_u32(&s.vempty[i]), 1);
    }
    for (int x = 0; x < kPHeads; ++x) {
      mbar_init(smem_u32(&s.sfull[x]), 1);
      mbar_init(smem_u32(&s.plo[x]), kPRows);
      mbar_init(smem_u32(&s.pfull[x]), kPRows);
      mbar_init(smem_u32(&s.odone[x]), 1);
      mbar_init(smem_u32(&s.oempty[x]), kPRows);
    }
    mbar_init(smem_u32(&s.drain), 1);
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kPMma) {
    tmem_alloc(smem_u32(&s.tmem), kPCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;

  if (warp == kPProducer) {
    // ---- TMA producer warp: each item's two query tiles, then its K and V tiles through the
    // 2-deep ring, lane i copying page i of a tile (its id read two tiles ahead) while lane 0 waits
    // for the slots and sets the byte counts; tiles are counted across items (t), so the ring
    // never drains between items. Queries are read once (evict first); K/V tiles are read again by
    // the other head pair of the kv head and the later query tiles of the sequence (evict last).
    const uint64_t pol_q = evict_first_policy();
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    const int npg_all = (p.S + kPPage - 1) / kPPage;
    constexpr int kTilePages = kPKeys / kPPage;
    auto fetch = [&](int b, int j) {   // this lane's page id of tile j of sequence b
      const int pg = j * kTilePages + lane;
      return (PAGED && lane < kTilePages && pg < npg_all)
                 ? __ldg(p.bt + static_cast<long long>(b) * p.bt_stride + pg) : 0;
    };
    // the (sequence, tile) after (b, j) in this CTA's order, or b = -1 past its last item
    auto after = [&](int w, int j, int& b2, int& j2, int& w2) {
      const Item it = item_of(p, w);
      if (j + 1 < it.nt) {
        b2 = it.b; j2 = j + 1; w2 = w;
      } else if (w + G < p.items) {
        b2 = item_of(p, w + G).b; j2 = 0; w2 = w + G;
      } else {
        b2 = -1; j2 = 0; w2 = w;
      }
    };
    int nxt = 0, nxt2 = 0, fb2 = -1, fj2 = 0, fw2 = 0;   // ids of the next two tiles; where nxt2 is
    if (static_cast<int>(blockIdx.x) < p.items) {
      nxt = fetch(item_of(p, blockIdx.x).b, 0);
      after(blockIdx.x, 0, fb2, fj2, fw2);
      if (fb2 >= 0) nxt2 = fetch(fb2, fj2);
    }
    int t = 0, i = 0;
    bool ok = true;
    for (int w = blockIdx.x; ok && w < p.items; w += G, ++i) {
      const Item it = item_of(p, w);
      // the previous item's last scores are computed: its query tiles may be replaced
      ok = __all_sync(0xffffffffu, i == 0 || mbar_wait(smem_u32(&s.qempty), (i - 1) & 1, s, p.err, true));
      if (!ok) break;
      if (lane == 0) mbar_arrive_expect_tx(smem_u32(&s.qfull), 4 * kPHalfBytes);
      __syncwarp();
      if (lane < 4)
        tma_load_4d(smem_u32(&s.q[lane >> 1][lane & 1][0]), &p.tmq, 64 * (lane & 1), it.h0 + (lane >> 1),
                    it.q0, it.b, smem_u32(&s.qfull), pol_q);
      for (int j = 0; j < it.nt; ++j) {
        const int st = t & 1, use = t >> 1;
        const int npg = PAGED ? min(kTilePages, npg_all - j * kTilePages) : 0;
        int row = 0;
        if (PAGED) {
          int pid = nxt;
          if (lane < npg && (pid < 0 || pid >= p.num_pages)) {   // recorded; a valid page keeps the count
            atomicOr(p.err, KOPT_DEV_ERR_PAGE);
            pid = 0;
          }
          row = (pid * p.nkv + it.kvh) * kPPage;
          nxt = nxt2;
          if (fb2 >= 0) {   // the ids of the tile after the next one
            after(fw2, fj2, fb2, fj2, fw2);
            if (fb2 >= 0) nxt2 = fetch(fb2, fj2);
          }
        }
        for (int kv = 0; kv < 2; ++kv) {
          unsigned long long* empty = kv == 0 ? s.kempty : s.vempty;
          unsigned long long* full = kv == 0 ? s.kfull : s.vfull;
          ok = __all_sync(0xffffffffu, t < kPStages ||
                          mbar_wait(smem_u32(&empty[st]), (use - 1) & 1, s, p.err, true));
          if (!ok) break;
          const CUtensorMap* map = kv == 0 ? &p.tmk : &p.tmv;
          bf16 (*dst)[kPHalf] = kv == 0 ? s.k[st] : s.v[st];
          const uint32_t fb = smem_u32(&full[st]);
          if (lane == 0)
            mbar_arrive_expect_tx(fb, PAGED ? static_cast<uint32_t>(npg) * 2u * kPPage * 64u * 2u : 2 * kPHalfBytes);
          __syncwarp();
          if (PAGED) {
            if (lane < npg) {
              tma_load_2d(smem_u32(&dst[0][lane * kPPage * 64]), map, 0, row, fb, pol);
              tma_load_2d(smem_u32(&dst[1][lane * kPPage * 64]), map, 64, row, fb, pol);
            }
          } else if (lane < 2) {
            tma_load_4d(smem_u32(&dst[lane][0]), map, 64 * lane, j * kPKeys, it.kvh, it.b, fb, pol);
          }
        }
        if (!ok) break;
        ++t;
      }
    }
    // every copy issued has landed before the CTA ends (the newest phase of each barrier; after
    // an abort a copy that was never issued waits out its bound)
    if (lane == 0) {
      if (i > 0) mbar_wait(smem_u32(&s.qfull), (i - 1) & 1, s, p.err, false);
      for (int k = max(t - kPStages, 0); k < t + (ok ? 0 : 1); ++k) {
        mbar_wait(smem_u32(&s.kfull[k & 1]), (k >> 1) & 1, s, p.err, false);
        mbar_wait(smem_u32(&s.vfull[k & 1]), (k >> 1) & 1, s, p.err, false);
      }
    }
  } else if (warp == kPMma) {
    if (lane == 0) {
      // ---- MMA issuer. Per item: S_A(0), S_B(0); then per key tile j: O_A += P_A(j) V_j,
      // S_A(j+1), O_B += P_B(j) V_j, S_B(j+1), each P V in two halves of 64 keys (plo: the
      // first half of P is written; pfull: all of it). Tiles are counted across items (T).
      auto issue_s = [&](int x, int st) {   // S_x = Q_x K^T
        const uint32_t qa = smem_u32(&s.q[x][0][0]), ka = smem_u32(&s.k[st][0][0]);
#pragma unroll
        for (int kk = 0; kk < kPD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPHalfBytes + (kk & 3) * 32;
          umma_bf16(tmem + col_s(x), sw128_desc(qa + off), sw128_desc(ka + off), kIdescS, kk > 0);
        }
      };
      auto issue_pv = [&](int x, int st, bool acc, int half) {   // O_x (+)= P_x V (keys of one half)
        const uint32_t va = smem_u32(&s.v[st][0][0]);
#pragma unroll
        for (int kk = half * kPKeys / 32; kk < (half + 1) * kPKeys / 32; ++kk) {
          const uint64_t bdesc = sw128_mn_desc(va + kk * 16 * 128, kPHalfBytes, 1024);
          umma_bf16_ts(tmem + col_o(x), tmem + col_s(x) + 8 * kk, bdesc, kIdescO,
                       (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      int t0 = 0, i = 0;
      for (int w = blockIdx.x; ok && w < p.items; w += G, ++i) {
        const int nt = item_of(p, w).nt;
        ok = mbar_wait(smem_u32(&s.qfull), i & 1, s, p.err, true) &&
             mbar_wait(smem_u32(&s.kfull[t0 & 1]), (t0 >> 1) & 1, s, p.err, true);
        if (!ok) break;
        tc_fence_after();
        issue_s(0, t0 & 1);
        umma_commit(smem_u32(&s.sfull[0]));
        issue_s(1, t0 & 1);
        umma_commit(smem_u32(&s.sfull[1]));
        umma_commit(smem_u32(&s.kempty[t0 & 1]));
        if (nt == 1) umma_commit(smem_u32(&s.qempty));
        for (int j = 0; j < nt; ++j) {
          const int T = t0 + j, st = T & 1, st1 = (T + 1) & 1;
          const bool more = j + 1 < nt;
          // O_A += P_A(j) V_j (the first P V of an item overwrites O_A, once the previous item's
          // output has been read out of it)
          if (!mbar_wait(smem_u32(&s.plo[0]), T & 1, s, p.err, true) ||
              !mbar_wait(smem_u32(&s.vfull[st]), (T >> 1) & 1, s, p.err, true) ||
              (j == 0 && i > 0 && !mbar_wait(smem_u32(&s.oempty[0]), (i - 1) & 1, s, p.err, true))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, st, j > 0, 0);
          if (!mbar_wait(smem_u32(&s.pfull[0]), T & 1, s, p.err, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(0, st, true, 1);
          if (!more) umma_commit(smem_u32(&s.odone[0]));
          if (more) {   // S_A(j+1): after the P V that read P_A(j) from the same columns
            if (!mbar_wait(smem_u32(&s.kfull[st1]), ((T + 1) >> 1) & 1, s, p.err, true)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(0, st1);
            umma_commit(smem_u32(&s.sfull[0]));
          }
          // O_B += P_B(j) V_j
          if (!mbar_wait(smem_u32(&s.plo[1]), T & 1, s, p.err, true) ||
              (j == 0 && i > 0 && !mbar_wait(smem_u32(&s.oempty[1]), (i - 1) & 1, s, p.err, true))) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(1, st, j > 0, 0);
          if (!mbar_wait(smem_u32(&s.pfull[1]), T & 1, s, p.err, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_pv(1, st, true, 1);
          umma_commit(smem_u32(&s.vempty[st]));
          if (!more) umma_commit(smem_u32(&s.odone[1]));
          if (more) {   // S_B(j+1); then K_{j+1} has been read by both
            issue_s(1, st1);
            umma_commit(smem_u32(&s.sfull[1]));
            umma_commit(smem_u32(&s.kempty[st1]));
            if (j + 2 == nt) umma_commit(smem_u32(&s.qempty));   // the item's last scores
          }
        }
        t0 += nt;
      }
      // every MMA issued has completed before the tensor memory is released
      umma_commit(smem_u32(&s.drain));
      mbar_wait(smem_u32(&s.drain), 0, s, p.err, false);
    }
    __syncwarp();
  } else {
    // ---- softmax: warps 0-3 tile A, warps 4-7 tile B; thread r owns query row q0 + r (tensor
    // memory lane r) of every item
    const int x = warp >> 2;
    const int r = 32 * (warp & 3) + lane;
    const uint32_t lrow = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
    bool ok = true;
    int T = 0, i = 0;
    for (int w = blockIdx.x; ok && w < p.items; w += G, ++i) {
      const Item it = item_of(p, w);
      const int row = it.q0 + r;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.nt; ++j, ++T) {
        // S_x(j) complete, and with it every MMA issued before (the P V that read P_x(j-1))
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.sfull[x]), T & 1, s, p.err, true));
        if (!ok) break;
        tc_fence_after();
        float sv[kPKeys];
        tmem_ld128(lrow + col_s(x), sv);
        const bool diag = j == it.nt - 1;
        if (diag) {   // causal: key <= query position
          const int lim = row - j * kPKeys;
#pragma unroll
          for (int c = 0; c < kPKeys; ++c)
            if (c > lim) sv[c] = -INFINITY;
        }
        // the row max on the raw scores (the scale is positive), then the exp2-domain max m
        float mx0 = sv[0], mx1 = sv[1];
#pragma unroll
        for (int c = 2; c < kPKeys; c += 2) {
          mx0 = fmaxf(mx0, sv[c]);
          mx1 = fmaxf(mx1, sv[c + 1]);
        }
        const float mx = fmaxf(mx0, mx1) * p.scale_log2;
        const bool need = mx > m + kPRescale;
        float alpha = 1.f;
        if (need) {
          alpha = ex2_fast(m - mx);
          m = mx;
          l *= alpha;
        }
        if (__any_sync(0xffffffffu, need) && j > 0) {   // O_x row *= alpha (1 where not needed)
#pragma unroll 1
          for (int c = 0; c < kPD; c += 16) {
            float o[16];
            uint32_t u[16];
            tmem_ld16(lrow + col_o(x) + c, o);
#pragma unroll
            for (int q = 0; q < 16; ++q) u[q] = __float_as_uint(o[q] * alpha);
            tmem_st16u(lrow + col_o(x) + c, u);
          }
        }
        if (x == 0 && diag && (j + 1) * kPKeys > p.S) {
          // keys past the prompt: their P is 0, but their V rows may hold anything (0 * inf);
          // tile A's threads clear them before either P V of this tile is issued
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.vfull[T & 1]), (T >> 1) & 1, s, p.err, true));
          if (!ok) break;
          if (j * kPKeys + r >= p.S) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t a = smem_u32(&s.v[T & 1][hh][r * 64]);
#pragma unroll
              for (int c = 0; c < 8; ++c)
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a + 16 * c), "r"(0u) : "memory");
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // visible to the MMA
        }
        // P = 2^(s * scale * log2(e) - m) as bf16 pairs, written over the first 64 columns of
        // S_x 16 words at a time (word e holds keys 2e, 2e + 1; the scores are all in registers
        // already); l sums the fp32 p. The first 64 keys are handed over before the rest, so
        // their half of P V runs while the second half is computed.
        float2 sum = make_float2(0.f, 0.f);
        const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m, -m);
#pragma unroll
        for (int ch = 0; ch < kPKeys / 32; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float2 x2 = fma2(make_float2(sv[32 * ch + 2 * e], sv[32 * ch + 2 * e + 1]), sc2, nm2);
            const float2 p2 = make_float2(ex2_fast(x2.x), ex2_fast(x2.y));
            sum = add2(sum, p2);
            pk[e] = pack_bf16(p2.x, p2.y);
          }
          tmem_st16u(lrow + col_s(x) + 16 * ch, pk);
          if (ch == 1) {
            tmem_wait_st();   // P_x(j) of keys 0-63 (and a rescaled O_x row) in tensor memory
            tc_fence_before();
            mbar_arrive(smem_u32(&s.plo[x]));
          }
        }
        l += sum.x + sum.y;
        tmem_wait_st();   // P_x(j) in tensor memory
        tc_fence_before();
        mbar_arrive(smem_u32(&s.pfull[x]));
      }
      if (!ok) break;
      // the item's output: O_x / l once its last P V is done; then O_x is free for the next item
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.odone[x]), i & 1, s, p.err, true));
      if (!ok) break;
      tc_fence_after();
      // the whole row in one load; O_x is handed back before the stores, so the next item's
      // first P V may start while they go out
      float o[kPD];
      tmem_ld128(lrow + col_o(x), o);
      tc_fence_before();
      mbar_arrive(smem_u32(&s.oempty[x]));
      const float inv = 1.0f / l;
      bf16* dst = p.out + (static_cast<long long>(it.b) * p.S + row) * p.nq * kPD + (it.h0 + x) * kPD;
      if (row < p.S) {
#pragma unroll
        for (int e = 0; e < kPD; e += 8) {
          uint4 u;
          u.x = pack_bf16(o[e] * inv, o[e + 1] * inv);
          u.y = pack_bf16(o[e + 2] * inv, o[e + 3] * inv);
          u.z = pack_bf16(o[e + 4] * inv, o[e + 5] * inv);
          u.w = pack_bf16(o[e + 6] * inv, o[e + 7] * inv);
          *reinterpret_cast<uint4*>(dst + e) = u;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kPMma) {
    tc_fence_after();
    tmem_dealloc(tmem, kPCols);
  }
}

template <bool PAGED>
int prefill_configure(int device) {
  static int configured[64] = {0};
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(prefill_attn_kernel<PAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPSmemBytes)) != cudaSuccess)
      return KOPT_ERR_CUDA;
    configured[device] = 1;
  }
  return KOPT_OK;
}

}  // namespace
}  // namespace kopt

using namespace kopt;

extern "C" int kopt_prefill_attn(const void* q, const kopt_kv_cache* cache, void* out, int B, int S,
                                 int nq, int nkv, int d, float scale, int* dev_err, int device,
                                 void* stream) {
  if (q == nullptr || cache == nullptr || out == nullptr || dev_err == nullptr) return KOPT_ERR_ARG;
  if (d != kPD || nkv < 1 || nq != kPGroup * nkv || B < 1 || S < 1) return KOPT_ERR_ARG;
  if (!aligned16(q) || !aligned16(out) || (reinterpret_cast<uintptr_t>(dev_err) & 3)) return KOPT_ERR_ARG;
  if (cache->k == nullptr || cache->v == nullptr || !aligned16(cache->k) || !aligned16(cache->v) ||
      cache->cap < S)
    return KOPT_ERR_ARG;
  const bool paged = cache->block_table != nullptr;
  if (paged) {
    if (cache->page_size != kPPage || cache->num_pages < 1 || cache->bt_stride < 1 ||
        static_cast<long long>(cache->bt_stride) * kPPage < S)
      return KOPT_ERR_ARG;
  } else if ((cache->stride_b % 8) != 0 || (cache->stride_h % 8) != 0) {
    return KOPT_ERR_ARG;
  }
  const long long nqt = (S + kPRows - 1) / kPRows;
  const long long items = nqt * B * nkv * kPHeads;
  if (items >= (1ll << 31)) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  rc = paged ? prefill_configure<true>(device) : prefill_configure<false>(device);
  if (rc) return rc;
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return KOPT_ERR_CUDA;
  PrefillParams p{};
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  {   // q: {128 dims, nq heads, S rows, B sequences}, box one head x 128 rows x 64 dims
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kPD), static_cast<cuuint64_t>(nq),
                                static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(B)};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kPD) * 2,
                                   static_cast<cuuint64_t>(nq) * kPD * 2,
                                   static_cast<cuuint64_t>(S) * nq * kPD * 2};
    const cuuint32_t box[4] = {64, 1, kPRows, 1};
    if (enc(&p.tmq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(q), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return KOPT_ERR_ARG;
  }
  for (int which = 0; which < 2; ++which) {
    CUtensorMap* map = which == 0 ? &p.tmk : &p.tmv;
    void* base = which == 0 ? cache->k : cache->v;
    CUresult r;
    if (paged) {
      const unsigned long long rows = static_cast<unsigned long long>(cache->num_pages) * nkv * kPPage;
      if (rows >= (1ull << 31)) return KOPT_ERR_ARG;
      const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kPD), rows};
      const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kPD) * 2};
      const cuuint32_t box[2] = {64, kPPage};
      r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const cuuint64_t dims[4] = {static_cast<cuuint64_t>(kPD), static_cast<cuuint64_t>(cache->cap),
                                  static_cast<cuuint64_t>(nkv), static_cast<cuuint64_t>(B)};
      const cuuint64_t strides[3] = {static_cast<cuuint64_t>(kPD) * 2,
                                     static_cast<cuuint64_t>(cache->stride_h) * 2,
                                     static_cast<cuuint64_t>(cache->stride_b) * 2};
      const cuuint32_t box[4] = {64, kPKeys, 1, 1};
      r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box, elem,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return KOPT_ERR_ARG;
  }
  p.out = static_cast<bf16*>(out);
  p.bt = paged ? cache->block_table : nullptr;
  p.err = dev_err;
  p.bt_stride = paged ? cache->bt_stride : 0;
  p.num_pages = paged ? cache->num_pages : 0;
  p.B = B;
  p.S = S;
  p.nq = nq;
  p.nkv = nkv;
  p.nqt = static_cast<int>(nqt);
  p.items = static_cast<int>(items);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return KOPT_ERR_CUDA;
  const long long grid = items < sms ? items : sms;   // persistent: one CTA per SM
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (paged)
    prefill_attn_kernel<true><<<static_cast<unsigned>(grid), kPThreads, kPSmemBytes, st>>>(p);
  else
    prefill_attn_kernel<false><<<static_cast<unsigned>(grid), kPThreads, kPSmemBytes, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}
