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
  float scale_log2;
};

struct __align__(1024) PSmem {
  bf16 q[2][kPHalf];                // query tile: [dims 0-63 | 64-127][128 rows][64]
  bf16 k[kPStages][2][kPHalf];      // key tiles: [dims half][128 keys][64]
  bf16 v[kPStages][2][kPHalf];      // value tiles, same layout (read as an MN-major operand)
  bf16 pm[2][kPHalf];               // P: [keys 0-63 | 64-127][128 rows][64], bf16
  unsigned long long qfull, kfull[kPStages], vfull[kPStages], kempty[kPStages], vempty[kPStages];
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
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <bool PAGED>
__global__ void __launch_bounds__(kPThreads, 1) prefill_attn_kernel(const __grid_constant__ PrefillParams p) {
  extern __shared__ unsigned char smem_raw[];
  PSmem& s = *reinterpret_cast<PSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // work item, the longest query tiles first
  const int per_qt = p.B * p.nq;
  const int qt = p.nqt - 1 - static_cast<int>(blockIdx.x) / per_qt;
  const int rem = static_cast<int>(blockIdx.x) % per_qt;
  const int b = rem / p.nq, h = rem % p.nq, kvh = h / kPGroup;
  const int q0 = qt * kPRows;
  const int nt = qt + 1;   // key tiles 0 .. qt

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&s.qfull), 1);
    for (int i = 0; i < kPStages; ++i) {
      mbar_init(smem_u32(&s.kfull[i]), 1);
      mbar_init(smem_u32(&s.vfull[i]), 1);
      mbar_init(smem_u32(&s.kempty[i]), 1);
      mbar_init(smem_u32(&s.vempty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
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
      const uint64_t pol = evict_first_policy();
      mbar_arrive_expect_tx(smem_u32(&s.qfull), 2 * kPHalfBytes);
      tma_load_4d(smem_u32(&s.q[0][0]), &p.tmq, 0, h, q0, b, smem_u32(&s.qfull), pol);
      tma_load_4d(smem_u32(&s.q[1][0]), &p.tmq, 64, h, q0, b, smem_u32(&s.qfull), pol);
      const int npg_all = (p.S + kPPage - 1) / kPPage;
      // one K or V tile: 8 page boxes per 64-dim half (paged) or one 128-row box per half
      auto load_tile = [&](const CUtensorMap* map, bf16 (*dst)[kPHalf], uint32_t bar, int j) {
        if (PAGED) {
          const int npg = min(kPKeys / kPPage, npg_all - j * (kPKeys / kPPage));
          mbar_arrive_expect_tx(bar, static_cast<uint32_t>(npg) * 2u * kPPage * 64u * 2u);
          for (int pg = 0; pg < npg; ++pg) {
            int pid = p.bt[static_cast<long long>(b) * p.bt_stride + j * (kPKeys / kPPage) + pg];
            if (pid < 0 || pid >= p.num_pages) {   // recorded; a valid page keeps the byte count
              atomicOr(p.err, KOPT_DEV_ERR_PAGE);
              pid = 0;
            }
            const int row = (pid * p.nkv + kvh) * kPPage;
            tma_load_2d(smem_u32(&dst[0][pg * kPPage * 64]), map, 0, row, bar, pol);
            tma_load_2d(smem_u32(&dst[1][pg * kPPage * 64]), map, 64, row, bar, pol);
          }
        } else {
          mbar_arrive_expect_tx(bar, 2 * kPHalfBytes);
          tma_load_4d(smem_u32(&dst[0][0]), map, 0, j * kPKeys, kvh, b, bar, pol);
          tma_load_4d(smem_u32(&dst[1][0]), map, 64, j * kPKeys, kvh, b, bar, pol);
        }
      };
      int j = 0;
      for (; j < nt; ++j) {
        const int st = j & 1, use = j >> 1;
        if (j >= kPStages && !mbar_wait(smem_u32(&s.kempty[st]), (use - 1) & 1, s, p.err, true)) break;
        load_tile(&p.tmk, s.k[st], smem_u32(&s.kfull[st]), j);
        if (j >= kPStages && !mbar_wait(smem_u32(&s.vempty[st]), (use - 1) & 1, s, p.err, true)) break;
        load_tile(&p.tmv, s.v[st], smem_u32(&s.vfull[st]), j);
      }
      // every copy issued has landed before this CTA ends (waits on the newest phase per stage)
      mbar_wait(smem_u32(&s.qfull), 0, s, p.err, false);
      for (int i = max(j - kPStages, 0); i < j; ++i) {
        mbar_wait(smem_u32(&s.kfull[i & 1]), (i >> 1) & 1, s, p.err, false);
        mbar_wait(smem_u32(&s.vfull[i & 1]), (i >> 1) & 1, s, p.err, false);
      }
    }
  } else if (warp == kPMma) {
    if (lane == 0) {
      const uint32_t qa = smem_u32(&s.q[0][0]);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(smem_u32(&s.kfull[st]), (j >> 1) & 1, s, p.err, true)) return false;
        if (j >= 2 && !mbar_wait(smem_u32(&s.sempty[st]), ((j >> 1) - 1) & 1, s, p.err, true))
          return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(&s.k[st][0][0]);
#pragma unroll
        for (int kk = 0; kk < kPD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kPHalfBytes + (kk & 3) * 32;
          umma_bf16(tmem + st * kPKeys, sw128_desc(qa + off), sw128_desc(ka + off), kIdescS, kk > 0);
        }
        umma_commit(smem_u32(&s.sfull[st]));
        umma_commit(smem_u32(&s.kempty[st]));
        return true;
      };
      bool ok = mbar_wait(smem_u32(&s.qfull), 0, s, p.err, true);
      if (ok) {
        tc_fence_after();
        ok = issue_s(0);
      }
      for (int j = 0; ok && j < nt; ++j) {
        if (j + 1 < nt && !issue_s(j + 1)) break;
        const int st = j & 1;
        if (!mbar_wait(smem_u32(&s.pfull), j & 1, s, p.err, true)) break;
        if (!mbar_wait(smem_u32(&s.vfull[st]), (j >> 1) & 1, s, p.err, true)) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(&s.pm[0][0]), va = smem_u32(&s.v[st][0][0]);
#pragma unroll
        for (int kk = 0; kk < kPKeys / 16; ++kk) {
          const uint64_t adesc = sw128_desc(pa + (kk >> 2) * kPHalfBytes + (kk & 3) * 32);
          const uint64_t bdesc = sw128_mn_desc(va + kk * 16 * 128, kPHalfBytes, 1024);
          umma_bf16(tmem + kPColO, adesc, bdesc, kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(smem_u32(&s.odone));
        umma_commit(smem_u32(&s.vempty[st]));
      }
      // every MMA issued has completed before the tensor memory is released
      umma_commit(smem_u32(&s.drain));
      mbar_wait(smem_u32(&s.drain), 0, s, p.err, false);
    }
    __syncwarp();
  } else {
    // ---- softmax: thread r owns query row q0 + r (tensor-memory lane r)
    const int r = 32 * warp + lane;
    const int row = q0 + r;
    const uint32_t lrow = tmem + (static_cast<uint32_t>(32 * warp) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt && ok; ++j) {
      const int sb = j & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.sfull[sb]), (j >> 1) & 1, s, p.err, true));
      if (!ok) break;
      tc_fence_after();
      float sv[kPKeys];
#pragma unroll
      for (int c = 0; c < kPKeys; c += 32) tmem_ld32(lrow + sb * kPKeys + c, sv + c);
      tc_fence_before();
      mbar_arrive(smem_u32(&s.sempty[sb]));   // the S buffer may take S_{j+2}
      const bool diag = j == nt - 1;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < kPKeys; ++c) {
        float x = sv[c] * p.scale_log2;
        if (diag && j * kPKeys + c > row) x = -INFINITY;   // causal: key <= query position
        sv[c] = x;
        mx = fmaxf(mx, x);
      }
      const bool need = mx > m + kPRescale;
      float alpha = 1.f;
      if (need) {
        alpha = exp2f(m - mx);
        m = mx;
        l *= alpha;
      }
      const bool wresc = __any_sync(0xffffffffu, need) && j > 0;
      if (j > 0) {   // PV_{j-1} done: P may be rewritten and O is stable
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.odone), (j - 1) & 1, s, p.err, true));
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
        ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.vfull[sb]), (j >> 1) & 1, s, p.err, true));
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
      // P row r: bf16 in the 128-byte swizzled K-major layout (16-byte chunk c of row r at
      // c ^ (r % 8)); l sums the fp32 p
      float sum = 0.f;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t base = smem_u32(&s.pm[hh][r * 64]);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int c = hh * 64 + cc * 8 + 2 * e;
            const float p0 = exp2f(sv[c] - m), p1 = exp2f(sv[c + 1] - m);
            sum += p0 + p1;
            w[e] = pack_bf16(p0, p1);
          }
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(base + ((cc ^ (r & 7)) << 4)),
                       "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                       : "memory");
        }
      }
      l += sum;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // P visible to the MMA
      tc_fence_before();
      mbar_arrive(smem_u32(&s.pfull));
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(smem_u32(&s.odone), (nt - 1) & 1, s, p.err, true));
    if (ok) {
      tc_fence_after();
      const float inv = 1.0f / l;
      bf16* dst = p.out + (static_cast<long long>(b) * p.S + row) * p.nq * kPD + h * kPD;
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
  const long long grid = nqt * B * nq;
  if (grid >= (1ll << 31)) return KOPT_ERR_ARG;
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
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (paged)
    prefill_attn_kernel<true><<<static_cast<unsigned>(grid), kPThreads, kPSmemBytes, st>>>(p);
  else
    prefill_attn_kernel<false><<<static_cast<unsigned>(grid), kPThreads, kPSmemBytes, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}
