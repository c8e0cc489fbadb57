// Causal GQA attention over a prompt (the prefill) on the 5th-generation tensor cores (sm_100a),
// behind the C ABI in include/kopt.h.
//
// What the reference does (GodRishUniverse/kernel_optim, engine/engine.py:343-386): per layer, after
// the q/k norm + RoPE of the prompt, F.scaled_dot_product_attention(q, k, v, is_causal=True) with
// GQA (engine.py:376-377), then the prompt's K/V go to the cache. Here the prologue writes the
// prompt's K/V straight into the (paged) cache and this kernel reads them from there.
//
// One CTA per (sequence, query head, 128-row query tile), the longest tiles first. For key tile j
// (128 keys) of the tiles 0 .. qt the tile needs (causal):
//   warp 4   TMA producer: the query tile once, then K and V tiles into a 2-deep ring (128-byte
//            swizzle; paged caches arrive as 16-row page boxes);
//   warp 5   allocates tensor memory and one thread issues the MMAs:
//            S_j = Q K_j^T into one of two fp32 S buffers in tensor memory (M = 128 query rows,
//            N = 128 keys, K-major operands), then O += P_j V_j (P from shared memory, V as an
//            MN-major operand) into the fp32 O accumulator in tensor memory;
//   warps 0-3 one thread per query row (tensor-memory lane): read the row of S_j with tcgen05.ld,
//            mask the diagonal tile, online softmax in fp32 in the exp2 domain, write P_j to shared
//            memory as bf16 (the K-major layout the MMA reads). The running maximum only moves
//            when a row's maximum grows by more than 2^8, so O (in tensor memory) is rescaled
//            rarely, by the warp that needs it, between the two MMAs that touch it; at the end
//            O / l goes to the output as bf16.
// S_{j+1} is computed while the softmax works on S_j. Every wait is bounded in time; on expiry
// the kernel records KOPT_DEV_ERR_TIMEOUT, stops, waits (bounded) for what it issued and frees
// its tensor memory.

#include "common.cuh"

namespace kopt {
namespace {

constexpr int kPD = 128;                    // head dim
constexpr int kPGroup = 4;                  // query heads per kv head
constexpr int kPRows = 128;                 // query rows per tile: the MMAs' M
constexpr int kPKeys = 128;                 // keys per tile
constexpr int kPPage = 16;                  // tokens per cache page
constexpr int kPStages = 2;                 // K/V ring depth
constexpr int kPSoftWarps = 4;              // warps 0-3: one thread per query row
constexpr int kPProducer = 4;
constexpr int kPMma = 5;
constexpr int kPThreads = 6 * 32;
constexpr uint32_t kPCols = 512;            // tensor memory: S double buffer + O
constexpr uint32_t kPColO = 256;
constexpr int kPHalf = kPRows * 64;         // elements of one 64-column half tile
constexpr uint32_t kPHalfBytes = kPHalf * 2;   // 16 KiB
constexpr float kPRescale = 8.f;            // log2 growth of a row's max that moves its running max

struct PrefillParams {
  CUtensorMap tmq;          // q [B*S, nq*128] as 4-D {128 dims, nq heads, S rows, B}: box {64, 1, 128, 1}
  CUtensorMap tmk;          // K cache: paged {128, pages*nkv*16} (box {64, 16}) or
  CUtensorMap tmv;          //   contiguous {128, cap, nkv, B} (box {64, 128, 1, 1}); V likewise
  bf16* out;                // [B*S, nq*128]
  const int* bt;            // block table (paged) or nullptr
  int* err;                 // device error word
  int bt_stride, num_pages;
  int B, S, nq, nkv, nqt;
  int items;                // B * nq * nqt (sequence, query head, query tile) work items
  float scale_log2;
};

struct __align__(1024) PSmem {
  bf16 q[2][2][kPHalf];             // two query tiles, each [dims 0-63 | 64-127][128 rows][64]
  bf16 k[kPStages][2][kPHalf];      // key tiles: [dims half][128 keys][64]
  bf16 v[kPStages][2][kPHalf];      // value tiles, same layout (read as an MN-major operand)
  bf16 pm[2][kPHalf];               // P: [keys 0-63 | 64-127][128 rows][64], bf16
  unsigned long long qfull[2], qempty[2];
  unsigned long long kfull[kPStages], vfull[kPStages], kempty[kPStages], vempty[kPStages];
  unsigned long long sfull[2], sempty[2], pfull, odone, drain;
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

// Shared-memory descriptor of an MN-major operand written with the 128-byte swizzle: 64-element
// (128-byte) rows along MN, 8 rows of K per 1024-byte atom; lbo = distance between 64-wide MN
// groups, sbo = distance between 8-row K groups; version 1, layout 2 (128-byte swizzle).
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// 32 consecutive fp32 columns of this thread's tensor-memory lane (waits for the load).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* r) {
  uint32_t v[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
        "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
        "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) r[j] = __uint_as_float(v[j]);
}
// 128 consecutive fp32 columns of this thread's tensor-memory lane in one load and one wait.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float* r) {
  uint32_t v[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31]),
        "=r"(v[32]), "=r"(v[33]), "=r"(v[34]), "=r"(v[35]), "=r"(v[36]), "=r"(v[37]), "=r"(v[38]), "=r"(v[39]),
        "=r"(v[40]), "=r"(v[41]), "=r"(v[42]), "=r"(v[43]), "=r"(v[44]), "=r"(v[45]), "=r"(v[46]), "=r"(v[47]),
        "=r"(v[48]), "=r"(v[49]), "=r"(v[50]), "=r"(v[51]), "=r"(v[52]), "=r"(v[53]), "=r"(v[54]), "=r"(v[55]),
        "=r"(v[56]), "=r"(v[57]), "=r"(v[58]), "=r"(v[59]), "=r"(v[60]), "=r"(v[61]), "=r"(v[62]), "=r"(v[63]),
        "=r"(v[64]), "=r"(v[65]), "=r"(v[66]), "=r"(v[67]), "=r"(v[68]), "=r"(v[69]), "=r"(v[70]), "=r"(v[71]),
        "=r"(v[72]), "=r"(v[73]), "=r"(v[74]), "=r"(v[75]), "=r"(v[76]), "=r"(v[77]), "=r"(v[78]), "=r"(v[79]),
        "=r"(v[80]), "=r"(v[81]), "=r"(v[82]), "=r"(v[83]), "=r"(v[84]), "=r"(v[85]), "=r"(v[86]), "=r"(v[87]),
        "=r"(v[88]), "=r"(v[89]), "=r"(v[90]), "=r"(v[91]), "=r"(v[92]), "=r"(v[93]), "=r"(v[94]), "=r"(v[95]),
        "=r"(v[96]), "=r"(v[97]), "=r"(v[98]), "=r"(v[99]), "=r"(v[100]), "=r"(v[101]), "=r"(v[102]), "=r"(v[103]),
        "=r"(v[104]), "=r"(v[105]), "=r"(v[106]), "=r"(v[107]), "=r"(v[108]), "=r"(v[109]), "=r"(v[110]), "=r"(v[111]),
        "=r"(v[112]), "=r"(v[113]), "=r"(v[114]), "=r"(v[115]), "=r"(v[116]), "=r"(v[117]), "=r"(v[118]), "=r"(v[119]),
        "=r"(v[120]), "=r"(v[121]), "=r"(v[122]), "=r"(v[123]), "=r"(v[124]), "=r"(v[125]), "=r"(v[126]), "=r"(v[127])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int j = 0; j < 128; ++j) r[j] = __uint_as_float(v[j]);
}
// Store 32 fp32 columns of this thread's lane; completes at the next tmem_wait_st.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
      "%29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(r[0])), "r"(__float_as_uint(r[1])), "r"(__float_as_uint(r[2])),
      "r"(__float_as_uint(r[3])), "r"(__float_as_uint(r[4])), "r"(__float_as_uint(r[5])),
      "r"(__float_as_uint(r[6])), "r"(__float_as_uint(r[7])), "r"(__float_as_uint(r[8])),
      "r"(__float_as_uint(r[9])), "r"(__float_as_uint(r[10])), "r"(__float_as_uint(r[11])),
      "r"(__float_as_uint(r[12])), "r"(__float_as_uint(r[13])), "r"(__float_as_uint(r[14])),
      "r"(__float_as_uint(r[15])), "r"(__float_as_uint(r[16])), "r"(__float_as_uint(r[17])),
      "r"(__float_as_uint(r[18])), "r"(__float_as_uint(r[19])), "r"(__float_as_uint(r[20])),
      "r"(__float_as_uint(r[21])), "r"(__float_as_uint(r[22])), "r"(__float_as_uint(r[23])),
      "r"(__float_as_uint(r[24])), "r"(__float_as_uint(r[25])), "r"(__float_as_uint(r[26])),
      "r"(__float_as_uint(r[27])), "r"(__float_as_uint(r[28])), "r"(__float_as_uint(r[29])),
      "r"(__float_as_uint(r[30])), "r"(__float_as_uint(r[31]))
      : "memory");
}
// 2^x by the hardware's approximate exponential (one MUFU op; subnormal results flush to zero,
// which bf16 P cannot hold with any meaning anyway).
__device__ __forceinline__ float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// This CTA's work items: item w = blockIdx.x + i * gridDim.x of the list ordered longest first
// (query tile qt = nqt - 1 down to 0; within a tile, sequence-major, head-minor, so the 4 heads of
// a kv head are neighbours and share its K/V tiles in L2).
struct Item {
  int b, h, kvh, q0, nt;
};
__device__ __forceinline__ Item item_of(const PrefillParams& p, int w) {
  const int per_qt = p.B * p.nq;
  const int qt = p.nqt - 1 - w / per_qt;
  const int rem = w - (w / per_qt) * per_qt;
  Item it;
  it.b = rem / p.nq;
  it.h = rem - it.b * p.nq;
  it.kvh = it.h / kPGroup;
  it.q0 = qt * kPRows;
  it.nt = qt + 1;   // causal: key tiles 0 .. qt
  return it;
}

template <bool PAGED>
__global__ void __launch_bounds__(kPThreads, 1) prefill_attn_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ unsigned char smem_raw[];
  PSmem& s = *reinterpret_cast<PSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&s.qfull[i]), 1);
      mbar_init(smem_u32(&s.qempty[i]), 1);
      mbar_init(smem_u32(&s.kfull[i]), 1);
      mbar_init(smem_u32(&s.vfull[i]), 1);
      mbar_init(smem_u32(&s.kempty[i]), 1);
      mbar_init(smem_u32(&s.vempty[i]), 1);
      mbar_init(smem_u32(&s.sfull[i]), 1);
      mbar_init(smem_u32(&s.sempty[i]), kPSoftWarps * 32);
    }
    mbar_init(smem_u32(&s.pfull), kPSoftWarps * 32);
    mbar_init(smem_u32(&s.odone), 1);
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
    if (lane == 0) {
      // ---- TMA producer: each item's query tile (two buffers, so the next item's arrives while
      // this one computes), then its K and V tiles through the 2-deep ring; tiles are counted
      // across items (t), so the ring never drains between items
      // queries are read once (evict first); K/V tiles are read again by the other heads of the
      // kv head and the later query tiles of the sequence (evict last)
      const uint64_t pol_q = evict_first_policy();
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
      const int npg_all = (p.S + kPPage - 1) / kPPage;
      int t = 0, i = 0;
      bool ok = true;
      auto load_tile = [&](const CUtensorMap* map, bf16 (*dst)[kPHalf], uint32_t bar, const Item& it, int j) {
        if (PAGED) {
          const int npg = min(kPKeys / kPPage, npg_all - j * (kPKeys / kPPage));
          mbar_arrive_expect_tx(bar, static_cast<uint32_t>(npg) * 2u * kPPage * 64u * 2u);
          for (int pg = 0; pg < npg; ++pg) {
            int pid = p.bt[static_cast<long long>(it.b) * p.bt_stride + j * (kPKeys / kPPage) + pg];
            if (pid < 0 || pid >= p.num_pages) {   // recorded; a valid page keeps the byte count
              atomicOr(p.err, KOPT_DEV_ERR_PAGE);
              pid = 0;
            }
            const int row = (pid * p.nkv + it.kvh) * kPPage;
            tma_load_2d(smem_u32(&dst[0][pg * kPPage * 64]), map, 0, row, bar, pol);
            tma_load_2d(smem_u32(&dst[1][pg * kPPage * 64]), map, 64, row, bar, pol);
          }
        } else {
          mbar_arrive_expect_tx(bar, 2 * kPHalfBytes);
          tma_load_4d(smem_u32(&dst[0][0]), map, 0, j * kPKeys, it.kvh, it.b, bar, pol);
          tma_load_4d(smem_u32(&dst[1][0]), map, 64, j * kPKeys, it.kvh, it.b, bar, pol);
        }
      };
      for (int w = blockIdx.x; ok && w < p.items; w += G, ++i) {
        const Item it = item_of(p, w);
        const int qb = i & 1;
        if (i >= 2 && !mbar_wait(smem_u32(&s.qempty[qb]), ((i >> 1) - 1) & 1, s, p.err, true)) break;
        mbar_arrive_expect_tx(smem_u32(&s.qfull[qb]), 2 * kPHalfBytes);
        tma_load_4d(smem_u32(&s.q[qb][0][0]), &p.tmq, 0, it.h, it.q0, it.b, smem_u32(&s.qfull[qb]), pol_q);
        tma_load_4d(smem_u32(&s.q[qb][1][0]), &p.tmq, 64, it.h, it.q0, it.b, smem_u32(&s.qfull[qb]), pol_q);
        for (int j = 0; j < it.nt; ++j) {
          const int st = t & 1, use = t >> 1;
          if (t >= kPStages && !mbar_wait(smem_u32(&s.kempty[st]), (use - 1) & 1, s, p.err, true)) {
            ok = false;
            break;
          }
          load_tile(&p.tmk, s.k[st], smem_u32(&s.kfull[st]), it, j);
          if (t >= kPStages && !mbar_wait(smem_u32(&s.vempty[st]), (use - 1) & 1, s, p.err, true)) {
            ++t;   // its K is in flight: drained below
            ok = false;
            break;
          }
          load_tile(&p.tmv, s.v[st], smem_u32(&s.vfull[st]), it, j);
          ++t;
        }
      }
      // every copy issued has landed before the CTA ends (the newest phase of each barrier)
      for (int k = max(i - 2, 0); k < i; ++k)
        mbar_wait(smem_u32(&s.qfull[k & 1]), (k >> 1) & 1, s, p.err, false);
      for (int k = max(t - kPStages, 0); k < t; ++k) {
        mbar_wait(smem_u32(&s.kfull[k & 1]), (k >> 1) & 1, s, p.err, false);
        mbar_wait(smem_u32(&s.vfull[k & 1]), (k >> 1) & 1, s, p.err, false);
      }
    }
  } else if (warp == kPMma) {
    if (lane == 0) {
      // ---- MMA issuer, one tile sequence across items: S of tile t + 1 is issued before P V of
      // tile t, so the tensor core computes the next scores while the softmax works
      int ntiles = 0;
      for (int w = blockIdx.x; w < p.items; w += G) ntiles += item_of(p, w).nt;
      int si = 0, sw = blockIdx.x, sj = 0, st_t = 0;   // next S: item si (index sw), its tile sj
      Item sit = item_of(p, min(sw, p.items - 1));
      auto issue_s = [&]() -> bool {
        const int qb = si & 1, st = st_t & 1;
        if (sj == 0 && !mbar_wait(smem_u32(&s.qfull[qb]), (si >> 1) & 1, s, p.err, true)) return false;
        if (!mbar_wait(smem_u32(&s.kfull[st]), (st_t >> 1) & 1, s, p.err, true)) return false;
        if (st_t >= 2 && !mbar_wait(smem_u32(&s.sempty[st]), ((st_t >> 1) - 1) & 1, s, p.err, true))
          return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(&s.q[qb][0][0]), ka = smem_u32(&s.k[st][0][0]);
#pragma unroll
        for (int kk = 0; kk < kPD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPHalfBytes + (kk & 3) * 32;
          umma_bf16(tmem + st * kPKeys, sw128_desc(qa + off), sw128_desc(ka + off), kIdescS, kk > 0);
        }
        umma_commit(smem_u32(&s.sfull[st]));
        umma_commit(smem_u32(&s.kempty[st]));
        if (sj == sit.nt - 1) {   // the item's last scores: its query buffer may take item si + 2
          umma_commit(smem_u32(&s.qempty[qb]));
          ++si;
          sw += G;
          sj = 0;
          if (sw < p.items) sit = item_of(p, sw);
        } else {
          ++sj;
        }
        ++st_t;
        return true;
      };
      bool ok = ntiles == 0 || issue_s();
      int pj = 0, pnt = item_of(p, min(static_cast<int>(blockIdx.x), p.items - 1)).nt, pw = blockIdx.x;
      for (int t = 0; ok && t < ntiles; ++t) {
        if (t + 1 < ntiles && !issue_s()) break;
        const int st = t & 1;
        if (!mbar_wait(smem_u32(&s.pfull), t & 1, s, p.err, true)) break;
        if (!mbar_wait(smem_u32(&s.vfull[st]), (t >> 1) & 1, s, p.err, true)) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(&s.pm[0][0]), va = smem_u32(&s.v[st][0][0]);
#pragma unroll
        for (int kk = 0; kk < kPKeys / 16; ++kk) {
          const uint64_t adesc = sw128_desc(pa + (kk >> 2) * kPHalfBytes + (kk & 3) * 32);
          const uint64_t bdesc = sw128_mn_desc(va + kk * 16 * 128, kPHalfBytes, 1024);
          umma_bf16(tmem + kPColO, adesc, bdesc, kIdescO, (pj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(smem_u32(&s.odone));
        umma_commit(smem_u32(&s.vempty[st]));
        if (++pj == pnt) {   // next item: its first P V overwrites O
          pj = 0;
          pw += G;
          if (pw < p.items) pnt = item_of(p, pw).nt;
        }
      }
      // every MMA issued has completed before the tensor memory is released
      umma_commit(smem_u32(&s.drain));
      mbar_wait(smem_u32(&s.drain), 0, s, p.err, false);
    }
    __syncwarp();
  } else {
    // ---- softmax: thread r owns query row q0 + r (tensor-memory lane r) of every item
    const int r = 32 * warp + lane;
    const uint32_t lrow = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    bool ok = true;
    int t = 0;
    for (int w = blockIdx.x; ok && w < p.items; w += G) {
      const Item it = item_of(p, w);
      const int row = it.q0 + r;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < it.nt; ++j, ++t) {
        const int sb = t & 1;
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.sfull[sb]), (t >> 1) & 1, s, p.err, true));
        if (!ok) break;
        tc_fence_after();
        float sv[kPKeys];
        tmem_ld128(lrow + sb * kPKeys, sv);
        tc_fence_before();
        mbar_arrive(smem_u32(&s.sempty[sb]));   // the S buffer may take S_{t+2}
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
        // P = 2^(s * scale * log2(e) - m), in registers (bf16 pairs) before waiting for the P
        // buffer; l sums the fp32 p
        uint32_t pk[kPKeys / 2];
        float sum0 = 0.f, sum1 = 0.f;
        const float nm = -m;
#pragma unroll
        for (int e = 0; e < kPKeys / 2; ++e) {
          const float p0 = ex2_fast(fmaf(sv[2 * e], p.scale_log2, nm));
          const float p1 = ex2_fast(fmaf(sv[2 * e + 1], p.scale_log2, nm));
          sum0 += p0;
          sum1 += p1;
          pk[e] = pack_bf16(p0, p1);
        }
        l += sum0 + sum1;
        const bool wresc = __any_sync(0xffffffffu, need) && j > 0;
        if (t > 0) {   // P V of the previous tile done: P may be rewritten, O is stable
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.odone), (t - 1) & 1, s, p.err, true));
          if (!ok) break;
          tc_fence_after();
        }
        if (wresc) {
#pragma unroll
          for (int c = 0; c < kPD; c += 32) {
            float o[32];
            tmem_ld32(lrow + kPColO + c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(lrow + kPColO + c, o);
          }
          tmem_wait_st();
        }
        if (diag && (j + 1) * kPKeys > p.S) {
          // keys past the prompt: their P is 0, but their V rows may hold anything (0 * inf)
          ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.vfull[sb]), (t >> 1) & 1, s, p.err, true));
          if (!ok) break;
          if (j * kPKeys + r >= p.S) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint32_t a = smem_u32(&s.v[sb][hh][r * 64]);
#pragma unroll
              for (int c = 0; c < 8; ++c)
                asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(a + 16 * c), "r"(0u) : "memory");
            }
          }
        }
        // P row r in the 128-byte swizzled K-major layout (16-byte chunk c of row r at c ^ (r % 8))
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t base = smem_u32(&s.pm[hh][r * 64]);
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const int e = hh * 32 + cc * 4;
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((cc ^ (r & 7)) << 4)),
                         "r"(pk[e]), "r"(pk[e + 1]), "r"(pk[e + 2]), "r"(pk[e + 3])
                         : "memory");
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // P visible to the MMA
        tc_fence_before();
        mbar_arrive(smem_u32(&s.pfull));
      }
      if (!ok) break;
      // the item's output: O / l once its last P V is done
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.odone), (t - 1) & 1, s, p.err, true));
      if (!ok) break;
      tc_fence_after();
      const float inv = 1.0f / l;
      bf16* dst = p.out + (static_cast<long long>(it.b) * p.S + row) * p.nq * kPD + it.h * kPD;
#pragma unroll
      for (int c = 0; c < kPD; c += 32) {
        float o[32];
        tmem_ld32(lrow + kPColO + c, o);
        if (row < p.S) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 u;
            u.x = pack_bf16(o[e] * inv, o[e + 1] * inv);
            u.y = pack_bf16(o[e + 2] * inv, o[e + 3] * inv);
            u.z = pack_bf16(o[e + 4] * inv, o[e + 5] * inv);
            u.w = pack_bf16(o[e + 6] * inv, o[e + 7] * inv);
            *reinterpret_cast<uint4*>(dst + c + e) = u;
          }
        }
      }
      tc_fence_before();   // O read before the next item's first P V overwrites it
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
  const long long items = nqt * B * nq;
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
