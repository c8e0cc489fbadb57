// Decode-step projections on B200 (sm_100a) and the row kernels around them, behind the C ABI in
// include/kopt.h (the reference's engine/kernels/gemv.py and the norm / SwiGLU wrappers of
// engine/kernels/fused.py): the residual add + RMSNorm, SwiGLU and row sum-of-squares kernels,
// and the tcgen05 skinny GEMM with its epilogues.
#include "common.cuh"

namespace kopt {

// ============================================================ decode-step epilogue kernels
// The two small ops around the projections of a decode step, in the reference's cast order
// (fused.py:13-46, 107-127, itself Transformers' Qwen3RMSNorm and Qwen3MLP): fp32 arithmetic,
// rounded to bf16 where the reference rounds.

// res <- bf16(res + delta) (if delta); out = bf16(w * bf16(res * rsqrt(mean(res^2) + eps))).
// One CTA per row; a thread holds 8-element vectors. Launched with programmatic dependent launch:
// it waits for the kernel before it before touching memory, then lets the next kernel's CTAs
// start (a projection streams its weights while the rows are normalised).
__global__ void add_rms_norm_kernel(bf16* __restrict__ res, const bf16* __restrict__ delta,
                                    const bf16* __restrict__ w, bf16* __restrict__ out, int n,
                                    float eps) {
  __shared__ float part[32];
  griddep_wait();
  griddep_launch_dependents();
  const long long row = blockIdx.x;
  const int nv = n / 8;
  bf16* x = res + row * n;
  float ss = 0.f;
  uint4 keep[4];   // up to 4 vectors per thread (n <= 32 * blockDim)
  uint4 wkeep[4];  // their weights, loaded with them: no second memory round trip after the sum
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v >= nv) break;
    wkeep[i] = __ldg(reinterpret_cast<const uint4*>(w + v * 8));
    uint4 a = *reinterpret_cast<const uint4*>(x + v * 8);
    if (delta != nullptr) {
      const uint4 d = *reinterpret_cast<const uint4*>(delta + row * n + v * 8);
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
      const uint32_t* pd = reinterpret_cast<const uint32_t*>(&d);
      uint4 sum;
      uint32_t* ps = reinterpret_cast<uint32_t*>(&sum);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 fa = bf2f(pa[e]), fd = bf2f(pd[e]);
        ps[e] = pack_bf16(__fadd_rn(fa.x, fd.x), __fadd_rn(fa.y, fd.y));
      }
      a = sum;
      *reinterpret_cast<uint4*>(x + v * 8) = a;
    }
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = bf2f(pa[e]);
      ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(f.x, f.x), __fmul_rn(f.y, f.y)));
    }
    keep[i] = a;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = (blockDim.x + 31) >> 5;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? part[lane] : 0.f;
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, off));
    if (lane == 0) part[0] = t;
  }
  __syncthreads();
  const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(part[0], static_cast<float>(n)), eps));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v >= nv) break;
    const uint4 wv = wkeep[i];
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&keep[i]);
    const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
    uint4 y;
    uint32_t* py = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = bf2f(pa[e]), fw = bf2f(pw[e]);
      py[e] = pack_bf16(__fmul_rn(fw.x, bf16r(__fmul_rn(f.x, rstd))),
                        __fmul_rn(fw.y, bf16r(__fmul_rn(f.y, rstd))));
    }
    *reinterpret_cast<uint4*>(out + row * n + v * 8) = y;
  }
}

// out[m, i] = bf16(bf16(silu(g)) * u), g = gu[m, i], u = gu[m, I + i]; a thread per 8 columns.
__global__ void silu_mul_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int I) {
  const long long m = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;
  if (v >= I / 8) return;
  const uint4 g = *reinterpret_cast<const uint4*>(gu + m * 2 * I + v * 8);
  const uint4 u = *reinterpret_cast<const uint4*>(gu + m * 2 * I + I + v * 8);
  const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
  const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
  uint4 y;
  uint32_t* py = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 fg = bf2f(pg[e]), fu = bf2f(pu[e]);
    const float s0 = bf16r(__fdiv_rn(fg.x, __fadd_rn(1.0f, expf(-fg.x))));
    const float s1 = bf16r(__fdiv_rn(fg.y, __fadd_rn(1.0f, expf(-fg.y))));
    py[e] = pack_bf16(__fmul_rn(s0, fu.x), __fmul_rn(s1, fu.y));
  }
  *reinterpret_cast<uint4*>(out + m * I + v * 8) = y;
}

// out[m] = sum over the row of x[m]^2 (bf16 x, fp32 sums), one CTA per row: each thread its 8-element
// vectors in order, then a warp xor tree and the warps in order. The row sums of squares a fused
// RMSNorm needs when no residual projection has produced them (the embedded rows of layer 0).
__global__ void row_sumsq_kernel(const bf16* __restrict__ x, int n, float* __restrict__ out) {
  __shared__ float part[32];
  griddep_wait();
  const long long row = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * n);
  float ss = 0.f;
  for (int v = threadIdx.x; v < n / 8; v += blockDim.x) {
    const uint4 a = xr[v];
    const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = bf2f(pa[e]);
      ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(f.x, f.x), __fmul_rn(f.y, f.y)));
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t = __fadd_rn(t, part[w]);
    out[row] = t;
  }
  griddep_launch_dependents();
}

// ============================================================= decode-step skinny GEMM (GEMV)
// y[M, N] = x[M, K] . W[N, K]^T for M <= 64 rows (the decode batch), fp32 accumulation, with the
// reference's epilogues (gemv.py:1-20, 29-106): F32 (fp32 store), BF16 (rounded store), RESID
// (h <- bf16(h + bf16(acc)), in place) and SWIGLU (W = [gate; up] of [2N, K], out =
// bf16(bf16(silu(bf16 g)) * bf16 u)), plus ARGMAX for the LM head: the index of each row's largest
// bf16-rounded logit, the first one on ties, as argmax over the reference's bf16 logits
// (engine.py:263 and the greedy pick after it) without writing the logits. Only the fp32
// accumulation order differs from cuBLAS.
//
// The weight is the MMA's A operand and the decode rows its B operand: D[128 weight rows][16 MT
// decode rows] += W[128][K] . x[16 MT][K]^T on the 5th-generation tensor cores (tcgen05.mma,
// kind::f16, bf16 in, fp32 accumulators in tensor memory). Persistent stream-K, one CTA per SM:
// the weight is cut into 128-row tiles (SWIGLU: 64 gate rows + the matching 64 up rows) of 64-wide
// K chunks; the (tile, chunk) units, tile-major, are dealt to the CTAs in equal contiguous runs.
//   warp 4  TMA producer: each unit's 128 x 64 weight tile and the matching x tile into a deep
//           ring (128-byte swizzle, the layout the MMA descriptors name);
//   warp 5  allocates tensor memory and one thread issues the MMAs, 4 of K = 16 per chunk, into
//           one of two accumulators, releasing each stage and each finished accumulator with
//           tcgen05.commit;
//   warps 0-3 read a finished accumulator (tcgen05.ld, lanes 32w..32w+31), hand it back, and run
//           the epilogue while the next segment accumulates in the other one.
// Where a run ends inside a tile, that segment's fp32 partial goes to the workspace and the CTA
// that arrives last at the tile adds the segments in CTA order (fixed, whichever finishes first)
// before the epilogue.
//
// Launched with programmatic stream serialization, the producer issues the weight copies of the
// first ring stages before griddepcontrol.wait: weights never depend on the previous kernel, so
// they stream while it drains. x, h and the workspace are touched only after the wait.
constexpr int kGEpiWarps = 4;            // epilogue warps: tensor-memory lanes 0-127
constexpr int kGProducerWarp = 4;
constexpr int kGMmaWarp = 5;
constexpr int kGNormWarp0 = 6;           // warps 6-9: RMSNorm of x in shared memory (when fused)
constexpr int kGNormThreads = 128;
constexpr int kGNormSmemK = 4096;        // norm weights up to this K are staged in shared memory
constexpr int kGThreads = 10 * 32;
constexpr int kGRows = 128;              // weight rows per tile = the MMA's M
constexpr int kGBK = 64;                 // k per chunk (one ring stage: 4 MMAs of K = 16)
constexpr int kGLd = kGRows + 4;         // fp32 tile row stride in shared memory (floats)
constexpr int GEMV_F32 = KOPT_GEMV_F32, GEMV_BF16 = KOPT_GEMV_BF16, GEMV_RESID = KOPT_GEMV_RESID,
              GEMV_SWIGLU = KOPT_GEMV_SWIGLU, GEMV_ARGMAX = KOPT_GEMV_ARGMAX;
// ring depth: as many stages as fit in shared memory next to the fp32 tile
template <int MT>
__host__ __device__ constexpr int gemv_stages() { return MT == 1 ? 11 : MT == 2 ? 10 : 7; }

struct GemvParams {
  CUtensorMap tmw;                       // W [rows, K]: box 64 k x 128 rows (SWIGLU: 64 rows)
  CUtensorMap tmx;                       // x [M, K]: box 64 k x 16 MT rows (rows >= M read as 0)
  void* y;                               // F32: float [M, N]; BF16, SWIGLU: bf16 [M, N];
                                         // RESID: the residual h [M, N], updated in place;
                                         // ARGMAX: int64 [M]
  float* part;                           // segment partials [2 grid][M][128]: 2c = CTA c's first
                                         // segment, 2c + 1 = its last
  int* cnt;                              // arrivals per tile, then tiles done (zero between launches)
  unsigned long long* keys;              // ARGMAX: per row, the best (bf16 logit, -index) so far
  int* err;
  const bf16* xg;                        // x in global memory (the norm's own sums of squares)
  const bf16* nw;                        // RMSNorm weight [K] applied to x; NULL: x used as it is
  const float* ss_in;                    // row sums of squares of x, [ss_tiles][M]; NULL: from x
  float* ss_out;                         // RESID: row sums of squares of the new h, [tiles][M]
  float eps;
  int ss_tiles;
  long long units;                       // tiles x nchunks
  int M, N, K, nchunks, tiles, per;      // per: units per CTA
};

template <int MT>
struct __align__(1024) GSmem {
  static constexpr int S = gemv_stages<MT>();
  bf16 w[S][kGRows * kGBK];              // 16 KB per stage
  bf16 x[S][16 * MT * kGBK];             // 2 KB per 16 decode rows per stage
  float ct[16 * MT][kGLd];               // a finished segment's fp32 sums, [decode row][weight row]
  unsigned long long full[S], empty[S], xready[S], tfull[2], tempty[2], fin, mrg;
  float rstd[64];                        // fused RMSNorm: 1 / rms of each row of x
  alignas(16) bf16 nws[kGNormSmemK];     // fused RMSNorm: its weight, when K <= kGNormSmemK
  uint32_t tmem;                         // tensor-memory base from tcgen05.alloc
  int last;
  int last_all;
  volatile int abort;
};
template <int MT>
constexpr size_t gsmem_bytes() { return sizeof(GSmem<MT>) + 1024; }
static_assert(gsmem_bytes<1>() <= 232448 && gsmem_bytes<2>() <= 232448 && gsmem_bytes<4>() <= 232448,
              "GEMV shared memory above the 227 KiB per-CTA limit");

__device__ __forceinline__ float silu_bf16(float g) {   // bf16(g / (1 + exp(-g))), g a bf16 value
  return bf16r(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B bf16 (7-9, 10-12 =
// 1), both K-major (15, 16 = 0), N >> 3 (17-22), M >> 4 (24-28).
__host__ __device__ constexpr uint32_t gemv_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kGRows >> 4) << 24);
}

template <int MT, int EPI>
__global__ void __launch_bounds__(kGThreads, 1) gemv_kernel(const __grid_constant__ GemvParams p) {
  constexpr int S = gemv_stages<MT>();
  const bool norm = p.nw != nullptr;   // x is normalised in shared memory before the MMAs read it
  constexpr int NM = 16 * MT;                  // the MMA's N: decode rows, padded
  constexpr uint32_t kCols = 2 * NM;           // two accumulators (32, 64 or 128 columns)
  extern __shared__ unsigned char smem_raw[];
  GSmem<MT>& s = *reinterpret_cast<GSmem<MT>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long u0 = static_cast<long long>(blockIdx.x) * p.per;
  const long long u1 = min(u0 + p.per, p.units);
  const int n = static_cast<int>(u1 - u0);   // >= 1: the grid is ceil(units / per)
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(smem_u32(&s.full[i]), 1);
      mbar_init(smem_u32(&s.empty[i]), 1);
      mbar_init(smem_u32(&s.xready[i]), kGNormThreads);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&s.tfull[b]), 1);
      mbar_init(smem_u32(&s.tempty[b]), kGEpiWarps);
    }
    mbar_init(smem_u32(&s.fin), 1);
    mbar_init(smem_u32(&s.mrg), 1);
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kGMmaWarp) {
    tmem_alloc(smem_u32(&s.tmem), kCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem;
  constexpr uint32_t kStageBytes = (kGRows + NM) * kGBK * 2;
  if (warp == kGProducerWarp) {   // --------------------------------------------------- producer
    if (lane == 0) {
      const uint64_t pol = evict_first_policy();
      auto load_w = [&](int i) {
        const long long u = u0 + i;
        const int tile = static_cast<int>(u / p.nchunks);
        const int k = static_cast<int>(u % p.nchunks) * kGBK;
        const int st = i % S;
        const uint32_t fb = smem_u32(&s.full[st]);
        if (EPI == GEMV_SWIGLU) {   // gate rows, then the up rows N further on
          tma_load_2d(smem_u32(&s.w[st][0]), &p.tmw, k, tile * 64, fb, pol);
          tma_load_2d(smem_u32(&s.w[st][64 * kGBK]), &p.tmw, k, p.N + tile * 64, fb, pol);
        } else {
          tma_load_2d(smem_u32(&s.w[st][0]), &p.tmw, k, tile * kGRows, fb, pol);
        }
      };
      auto load_x = [&](int i) {
        const int st = i % S;
        const int k = static_cast<int>((u0 + i) % p.nchunks) * kGBK;
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(&s.x[st][0])),
            "l"(&p.tmx), "r"(k), "r"(0), "r"(smem_u32(&s.full[st]))
            : "memory");
      };
      const int pre = n < S ? n : S;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(smem_u32(&s.full[i]), kStageBytes);
        load_w(i);
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i) load_x(i);
      int issued = pre;
      for (int i = pre; i < n; ++i) {
        const int st = i % S;
        if (!mbar_wait(smem_u32(&s.empty[st]), ((i / S) - 1) & 1, s, p.err, true)) break;
        mbar_arrive_expect_tx(smem_u32(&s.full[st]), kStageBytes);
        load_w(i);
        load_x(i);
        issued = i + 1;
      }
      // every copy issued has landed before the CTA may exit (bounded)
      for (int i = issued > S ? issued - S : 0; i < issued; ++i)
        mbar_wait(smem_u32(&s.full[i % S]), (i / S) & 1, s, p.err, false);
    } else {
      griddep_wait();
    }
    griddep_launch_dependents();
  } else if (warp == kGMmaWarp) {   // ----------------------------------------------- MMA issue
    griddep_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = gemv_idesc(NM);
      int i = 0, seg = 0;
      bool ok = true;
      for (long long u = u0; ok && u < u1; ++seg) {
        const int a = static_cast<int>(u % p.nchunks);
        const long long rest = u1 - u;
        const int b = rest < p.nchunks - a ? a + static_cast<int>(rest) : p.nchunks;
        const int buf = seg & 1;
        if (seg >= 2 && !mbar_wait(smem_u32(&s.tempty[buf]), ((seg >> 1) - 1) & 1, s, p.err, true))
          break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * NM);
        for (int c = a; c < b; ++c, ++i) {
          const int st = i % S;
          if (!mbar_wait(smem_u32(norm ? &s.xready[st] : &s.full[st]), (i / S) & 1, s, p.err, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wa = smem_u32(&s.w[st][0]), xa = smem_u32(&s.x[st][0]);
#pragma unroll
          for (int ks = 0; ks < kGBK / 16; ++ks)
            umma_bf16(d, sw128_desc(wa + 32 * ks), sw128_desc(xa + 32 * ks), idesc,
                      (c > a || ks > 0) ? 1u : 0u);
          umma_commit(smem_u32(&s.empty[st]));   // the stage is free once these MMAs read it
        }
        if (!ok) break;
        umma_commit(smem_u32(&s.tfull[buf]));   // the accumulator is complete
        u += b - a;
      }
      umma_commit(smem_u32(&s.fin));   // every MMA issued has completed: tensor memory may go
      mbar_wait(smem_u32(&s.fin), 0, s, p.err, false);
    }
    __syncwarp();
    griddep_launch_dependents();
  } else if (warp >= kGNormWarp0) {   // ------------------------------------- RMSNorm of x (fused)
    griddep_wait();
    if (norm) {
      const int t = threadIdx.x - kGNormWarp0 * 32;   // 0 .. 127
      // rstd of each row: from the producer's per-tile sums in tile order, or from x itself
      // (tpr threads per row, each a contiguous K range, then a fixed shuffle tree)
      constexpr int tpr = kGNormThreads / NM;        // 8, 4 or 2
      const int m = t / tpr, part = t % tpr;
      float ss = 0.f;
      if (m < p.M) {
        if (p.ss_in != nullptr) {   // the row's threads take contiguous runs of tiles, in order
          const int per_t = (p.ss_tiles + tpr - 1) / tpr;
          const int t0 = part * per_t, t1 = min(p.ss_tiles, t0 + per_t);
#pragma unroll 8
          for (int tt = t0; tt < t1; ++tt) ss = __fadd_rn(ss, __ldcg(p.ss_in + tt * p.M + m));
        } else {
          const int kv = p.K / 8, per_t = (kv + tpr - 1) / tpr;
          const int v0 = part * per_t, v1 = min(kv, v0 + per_t);
          const uint4* row = reinterpret_cast<const uint4*>(p.xg + static_cast<long long>(m) * p.K);
#pragma unroll 8
          for (int v = v0; v < v1; ++v) {
            const uint4 a = __ldg(row + v);
            const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 f = bf2f(pa[e]);
              ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(f.x, f.x), __fmul_rn(f.y, f.y)));
            }
          }
        }
      }
#pragma unroll
      for (int off = 1; off < tpr; off <<= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
      if (part == 0) s.rstd[m] = m < p.M ? rsqrtf(__fadd_rn(__fdiv_rn(ss, static_cast<float>(p.K)), p.eps)) : 0.f;
      const bool wsm = p.K <= kGNormSmemK;   // the weight read once into shared memory
      if (wsm)
        for (int v = t; v < p.K / 8; v += kGNormThreads)
          reinterpret_cast<uint4*>(s.nws)[v] = __ldg(reinterpret_cast<const uint4*>(p.nw) + v);
      named_bar(2, kGNormThreads);
      // every stage: x <- bf16(w * bf16(x * rstd)) in place (fused.py:39-46's cast order), in the
      // 128-byte-swizzled layout TMA wrote (16-byte chunk c of row r sits at chunk c ^ (r % 8))
      for (int i = 0; i < n; ++i) {
        const int st = i % S;
        if (!mbar_wait(smem_u32(&s.full[st]), (i / S) & 1, s, p.err, true)) break;
        const int kb = static_cast<int>((u0 + i) % p.nchunks) * kGBK;
        unsigned char* xs = reinterpret_cast<unsigned char*>(&s.x[st][0]);
        for (int c = t; c < NM * 8; c += kGNormThreads) {
          const int r = c >> 3, pc = c & 7;
          const int k0 = kb + 8 * (pc ^ (r & 7));
          uint4* cp = reinterpret_cast<uint4*>(xs + r * 128 + pc * 16);
          uint4 a = *cp;
          const uint4 wv = k0 >= p.K ? make_uint4(0, 0, 0, 0)
                           : wsm ? *reinterpret_cast<const uint4*>(s.nws + k0)
                                 : __ldg(reinterpret_cast<const uint4*>(p.nw + k0));
          const float rs = s.rstd[r];
          uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
          const uint32_t* pw = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = bf2f(pa[e]), fw = bf2f(pw[e]);
            pa[e] = pack_bf16(__fmul_rn(fw.x, bf16r(__fmul_rn(f.x, rs))),
                              __fmul_rn(fw.y, bf16r(__fmul_rn(f.y, rs))));
          }
          *cp = a;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // generic writes -> MMA reads
        mbar_arrive(smem_u32(&s.xready[st]));
      }
    }
    griddep_launch_dependents();
  } else {   // ------------------------------------------------------------- epilogue warps 0-3
    griddep_wait();
    const int tid = threadIdx.x, q = tid & 3;
    // epilogue layout: row r0 + tid / 4, two 16-column segments of the tile
    const int sa = EPI == GEMV_SWIGLU ? 16 * q : 32 * q;            // gate (or first) segment
    const int sb = EPI == GEMV_SWIGLU ? 64 + 16 * q : 32 * q + 16;   // up (or second) segment
    int seg = 0;
    for (long long u = u0; u < u1; ++seg) {
      const int tile = static_cast<int>(u / p.nchunks);
      const int a = static_cast<int>(u % p.nchunks);
      const long long rest = u1 - u;
      const int b = rest < p.nchunks - a ? a + static_cast<int>(rest) : p.nchunks;
      const bool first_seg = u == u0;
      const int buf = seg & 1;
      mbar_wait(smem_u32(&s.tfull[buf]), (seg >> 1) & 1, s, p.err, true);
      __syncwarp();   // tcgen05.ld is .aligned: the lanes leave the bounded spin at other times
      tc_fence_after();
      float r[NM];    // D[weight row 32 warp + lane][decode rows 0 .. NM)
#pragma unroll
      for (int c = 0; c < NM; c += 16)
        tmem_ld16(tmem + (static_cast<uint32_t>(32 * warp) << 16) + static_cast<uint32_t>(buf * NM + c),
                  r + c);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.tempty[buf]));
      u += b - a;
      if (u >= u1) griddep_launch_dependents();
      named_bar(1, kGEpiWarps * 32);   // the previous segment's epilogue is done with ct
#pragma unroll
      for (int j = 0; j < NM; ++j) s.ct[j][32 * warp + lane] = r[j];
      named_bar(1, kGEpiWarps * 32);
      // ---- a tile split between CTAs: partial out, the last arriver adds the segments
      const bool whole = a == 0 && b == p.nchunks;
      const long long tu0 = static_cast<long long>(tile) * p.nchunks;
      const int kfirst = static_cast<int>(tu0 / p.per);                    // CTAs holding the tile
      const int klast = static_cast<int>((tu0 + p.nchunks - 1) / p.per);
      if (!whole) {
        // partial out and, for the last arriver, the segments' sum back into ct, both with a warp
        // on whole 512-byte rows (lane l: columns 4l .. 4l + 3; warp w: rows w, w + 4, ...)
        const int slot = 2 * blockIdx.x + (first_seg ? 0 : 1);
        const int rows = NM < p.M ? NM : p.M;
        for (int m = warp; m < rows; m += kGEpiWarps)
          __stcg(reinterpret_cast<float4*>(p.part + (static_cast<long long>(slot) * p.M + m) * kGRows) + lane,
                 *reinterpret_cast<const float4*>(&s.ct[m][4 * lane]));
        __threadfence();
        named_bar(1, kGEpiWarps * 32);
        if (tid == 0) {
          s.last = atomicAdd(&p.cnt[tile], 1) == klast - kfirst;
          if (s.last) __threadfence();   // acquire the other segments' partials
        }
        named_bar(1, kGEpiWarps * 32);
        if (!s.last) continue;
        if (tid == 0) atomicExch(&p.cnt[tile], 0);
        constexpr int kR = (NM + kGEpiWarps - 1) / kGEpiWarps;   // rows per warp
        float4 acc4[kR];
#pragma unroll
        for (int r = 0; r < kR; ++r) acc4[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        auto seg_src = [&](int k) {
          const bool kfirst_seg = static_cast<long long>(k) * p.per >= tu0;
          return reinterpret_cast<const float4*>(
              p.part + static_cast<long long>(2 * k + (kfirst_seg ? 0 : 1)) * p.M * kGRows);
        };
        const int nseg = klast - kfirst + 1;
        const uint32_t seg_bytes = static_cast<uint32_t>(p.M) * kGRows * 4;
        if (u >= u1 && static_cast<long long>(nseg) * seg_bytes <= static_cast<long long>(sizeof(s.w))) {
          // this CTA's last segment: the ring is idle (every stage has been read by the MMAs), so
          // all the tile's partials come in at once by bulk copies, one L2 round trip, and are
          // added from shared memory in the same fixed order
          const float4* stage = reinterpret_cast<const float4*>(&s.w[0][0]);
          if (tid == 0) {
            asm volatile("fence.proxy.async.global;" ::: "memory");   // generic writes -> bulk reads
            const uint32_t mb = smem_u32(&s.mrg);
            mbar_arrive_expect_tx(mb, static_cast<uint32_t>(nseg) * seg_bytes);
            for (int j = 0; j < nseg; ++j)
              bulk_g2s(smem_u32(&s.w[0][0]) + static_cast<uint32_t>(j) * seg_bytes, seg_src(kfirst + j),
                       seg_bytes, mb);
          }
          mbar_wait(smem_u32(&s.mrg), 0, s, p.err, true);   // once per launch: phase 0
          __syncwarp();
          for (int j = 0; j < nseg; ++j)
#pragma unroll
            for (int r = 0; r < kR; ++r) {
              const int m = warp + kGEpiWarps * r;
              if (m < rows) {
                const float4 x = stage[(j * p.M + m) * (kGRows / 4) + lane];
                acc4[r].x += x.x;
                acc4[r].y += x.y;
                acc4[r].z += x.z;
                acc4[r].w += x.w;
              }
            }
        } else {
        // segments in a fixed order (the tile's first CTA first), KP of them per round so that
        // KP x kR loads are in flight together
        constexpr int KP = kR <= 8 ? 2 : 1;
        for (int k = kfirst; k <= klast; k += KP) {
          float4 x4[KP][kR];
#pragma unroll
          for (int j = 0; j < KP; ++j) {
            const bool have = k + j <= klast;
            const float4* src = seg_src(have ? k + j : k);
#pragma unroll
            for (int r = 0; r < kR; ++r) {
              const int m = warp + kGEpiWarps * r;
              x4[j][r] = have && m < rows
                             ? __ldcg(src + static_cast<long long>(m) * (kGRows / 4) + lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
          }
#pragma unroll
          for (int j = 0; j < KP; ++j)
#pragma unroll
            for (int r = 0; r < kR; ++r) {
              acc4[r].x += x4[j][r].x;
              acc4[r].y += x4[j][r].y;
              acc4[r].z += x4[j][r].z;
              acc4[r].w += x4[j][r].w;
            }
        }
        }
#pragma unroll
        for (int r = 0; r < kR; ++r) {
          const int m = warp + kGEpiWarps * r;
          if (m < rows) *reinterpret_cast<float4*>(&s.ct[m][4 * lane]) = acc4[r];
        }
        named_bar(1, kGEpiWarps * 32);
      }
      const int tcol = EPI == GEMV_SWIGLU ? tile * 64 : tile * kGRows;   // first output column
      // SWIGLU covers its 64 columns whole (N % 64 == 0); otherwise a 16-column segment is
      // either inside N or past it (N % 16 == 0)
      const bool va = EPI == GEMV_SWIGLU || tcol + sa < p.N;
      const bool vb = EPI == GEMV_SWIGLU || tcol + sb < p.N;
      for (int r0 = 0; r0 < NM; r0 += 32) {
        const int m = r0 + (tid >> 2);
        const bool act = m < NM && m < p.M;
        // ARGMAX and RESID: every lane takes part in the shuffles
        if (EPI != GEMV_ARGMAX && EPI != GEMV_RESID && !act) continue;
        float v[32];
        if (!act) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = -INFINITY;
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            v[j] = s.ct[m][sa + j];
            v[16 + j] = s.ct[m][sb + j];
          }
        }
        const long long row = static_cast<long long>(m) * p.N + tcol;
        if (EPI == GEMV_F32) {
          float* y = static_cast<float*>(p.y) + row;
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            if (va) *reinterpret_cast<float4*>(y + sa + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            if (vb)
              *reinterpret_cast<float4*>(y + sb + j) =
                  make_float4(v[16 + j], v[17 + j], v[18 + j], v[19 + j]);
          }
        } else if (EPI == GEMV_BF16) {
          bf16* y = static_cast<bf16*>(p.y) + row;
#pragma unroll
          for (int seg2 = 0; seg2 < 2; ++seg2) {
            if (!(seg2 == 0 ? va : vb)) continue;
            uint4 o0, o1;
            uint32_t* p0 = reinterpret_cast<uint32_t*>(&o0);
            uint32_t* p1 = reinterpret_cast<uint32_t*>(&o1);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              p0[e] = pack_bf16(v[16 * seg2 + 2 * e], v[16 * seg2 + 2 * e + 1]);
              p1[e] = pack_bf16(v[16 * seg2 + 8 + 2 * e], v[16 * seg2 + 9 + 2 * e]);
            }
            bf16* dst = y + (seg2 == 0 ? sa : sb);
            *reinterpret_cast<uint4*>(dst) = o0;
            *reinterpret_cast<uint4*>(dst + 8) = o1;
          }
        } else if (EPI == GEMV_RESID) {   // h <- bf16(h + bf16(acc)) (gemv.py:95-97)
          bf16* h = static_cast<bf16*>(p.y) + row;
          float sq = 0.f;   // sum of squares of this thread's new h values (gemv.py:97-98)
#pragma unroll
          for (int seg2 = 0; seg2 < 2; ++seg2) {
            if (!act || !(seg2 == 0 ? va : vb)) continue;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              bf16* hp = h + (seg2 == 0 ? sa : sb) + 8 * half;
              uint4 hv = *reinterpret_cast<const uint4*>(hp);
              uint32_t* ph = reinterpret_cast<uint32_t*>(&hv);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 f = bf2f(ph[e]);
                const int j = 16 * seg2 + 8 * half + 2 * e;
                ph[e] = pack_bf16(__fadd_rn(f.x, bf16r(v[j])), __fadd_rn(f.y, bf16r(v[j + 1])));
                const float2 hn = bf2f(ph[e]);
                sq = __fadd_rn(sq, __fadd_rn(__fmul_rn(hn.x, hn.x), __fmul_rn(hn.y, hn.y)));
              }
              *reinterpret_cast<uint4*>(hp) = hv;
            }
          }
          // the row's 4 threads, then one partial per (tile, row): the next projection's norm adds
          // the tiles in order, so the result does not depend on timing
          sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 1));
          sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, 2));
          if (p.ss_out != nullptr && act && q == 0) p.ss_out[static_cast<long long>(tile) * p.M + m] = sq;
        } else if (EPI == GEMV_ARGMAX) {
          // this thread's 32 columns, then the row's 4 threads, then all tiles through one 64-bit
          // atomicMax per row: key = (order-preserving bits of the bf16 logit) << 32 | ~index, so
          // the larger logit wins and, on equal logits, the smaller index
          float best = -INFINITY;
          int bi = 0x7fffffff;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int col = tcol + (j < 16 ? sa + j : sb + j - 16);
            const float l = bf16r(v[j]) + 0.0f;   // -0 -> +0: equal logits compare equal
            if (col < p.N && (l > best || (l == best && col < bi))) {
              best = l;
              bi = col;
            }
          }
          const uint32_t ub = __float_as_uint(best);
          const uint32_t ord = (ub & 0x80000000u) ? ~ub : (ub | 0x80000000u);
          unsigned long long key = (static_cast<unsigned long long>(ord) << 32) |
                                   static_cast<uint32_t>(0xffffffffu - static_cast<uint32_t>(bi));
          key = max(key, __shfl_xor_sync(0xffffffffu, key, 1));
          key = max(key, __shfl_xor_sync(0xffffffffu, key, 2));
          if (q == 0 && act) atomicMax(p.keys + m, key);
        } else {   // SWIGLU: output columns 64 tile + 16 q .. + 16 (gemv.py:101-105)
          bf16* y = static_cast<bf16*>(p.y) + static_cast<long long>(m) * p.N + tcol + 16 * q;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint4 o;
            uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int j = 8 * half + 2 * e;
              const float s0 = silu_bf16(bf16r(v[j])), s1 = silu_bf16(bf16r(v[j + 1]));
              po[e] = pack_bf16(__fmul_rn(s0, bf16r(v[16 + j])), __fmul_rn(s1, bf16r(v[17 + j])));
            }
            *reinterpret_cast<uint4*>(y + 8 * half) = o;
          }
        }
      }
      if (EPI == GEMV_ARGMAX) {   // the tile that finishes last turns the keys into token ids
        __threadfence();
        named_bar(1, kGEpiWarps * 32);
        if (tid == 0) {
          s.last_all = atomicAdd(&p.cnt[p.tiles], 1) == p.tiles - 1;
          if (s.last_all) __threadfence();
        }
        named_bar(1, kGEpiWarps * 32);
        if (s.last_all) {
          if (tid < p.M) {
            const unsigned long long key = atomicExch(p.keys + tid, 0ull);   // read and re-arm
            static_cast<long long*>(p.y)[tid] =
                static_cast<long long>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffu));
          }
          if (tid == 0) atomicExch(&p.cnt[p.tiles], 0);
        }
      }
    }
  }
  // ---- tensor memory goes back once every MMA has completed and every load from it is done
  tc_fence_before();
  __syncthreads();
  if (warp == kGMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

// ------------------------------------------------------------------------------- GEMV host side
// Workspace: [0, 256) the error word; one arrival counter per tile and one for tiles done; the
// ARGMAX keys of up to 64 rows; then two fp32 segment partials [M][128] per CTA.
struct GemvWs { int64_t cnt, keys, part, total; };
GemvWs gemv_ws_layout(int M, int tiles, int grid) {
  GemvWs w;
  w.cnt = kHeaderBytes;
  w.keys = w.cnt + (static_cast<int64_t>(tiles + 1) * 4 + 255) / 256 * 256;
  w.part = w.keys + 64 * 8;
  w.total = w.part + 2 * static_cast<int64_t>(grid) * M * kGRows * 4;
  return w;
}
inline int gemv_mt(int M) { return M <= 16 ? 1 : M <= 32 ? 2 : 4; }

template <int MT, int EPI>
int gemv_occupancy(int device, int* blocks_per_sm) {
  static int configured[64] = {0};
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  auto kern = gemv_kernel<MT, EPI>;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(gsmem_bytes<MT>())) != cudaSuccess)
      return KOPT_ERR_CUDA;
    configured[device] = 1;
  }
  if (blocks_per_sm &&
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kern, kGThreads,
                                                    gsmem_bytes<MT>()) != cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}
template <int MT>
int gemv_occupancy_epi(int device, int epi, int* blocks_per_sm) {
  switch (epi) {
    case GEMV_F32: return gemv_occupancy<MT, GEMV_F32>(device, blocks_per_sm);
    case GEMV_BF16: return gemv_occupancy<MT, GEMV_BF16>(device, blocks_per_sm);
    case GEMV_RESID: return gemv_occupancy<MT, GEMV_RESID>(device, blocks_per_sm);
    case GEMV_SWIGLU: return gemv_occupancy<MT, GEMV_SWIGLU>(device, blocks_per_sm);
    default: return gemv_occupancy<MT, GEMV_ARGMAX>(device, blocks_per_sm);
  }
}
int gemv_configure(int device, int M, int epi, int* blocks_per_sm) {
  const int mt = gemv_mt(M);
  return mt == 1 ? gemv_occupancy_epi<1>(device, epi, blocks_per_sm)
                 : mt == 2 ? gemv_occupancy_epi<2>(device, epi, blocks_per_sm)
                           : gemv_occupancy_epi<4>(device, epi, blocks_per_sm);
}

template <int MT, int EPI>
int gemv_launch_t(const kopt_gemv_plan* plan, GemvParams& p, void* stream) {
  int rc = gemv_occupancy<MT, EPI>(plan->device, nullptr);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  // the four RMSNorm warps exist only when the norm is fused
  cfg.blockDim = dim3(p.nw != nullptr ? kGThreads : kGThreads - kGNormThreads);
  cfg.dynamicSmemBytes = gsmem_bytes<MT>();
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (plan->flags & KOPT_GEMV_OVERLAP_PREV) ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, gemv_kernel<MT, EPI>, p) != cudaSuccess) {
    cudaGetLastError();
    return KOPT_ERR_CUDA;
  }
  return KOPT_OK;
}
template <int MT>
int gemv_launch_epi(const kopt_gemv_plan* plan, GemvParams& p, void* stream) {
  switch (plan->epi) {
    case GEMV_F32: return gemv_launch_t<MT, GEMV_F32>(plan, p, stream);
    case GEMV_BF16: return gemv_launch_t<MT, GEMV_BF16>(plan, p, stream);
    case GEMV_RESID: return gemv_launch_t<MT, GEMV_RESID>(plan, p, stream);
    case GEMV_SWIGLU: return gemv_launch_t<MT, GEMV_SWIGLU>(plan, p, stream);
    default: return gemv_launch_t<MT, GEMV_ARGMAX>(plan, p, stream);
  }
}

}  // namespace kopt

// =================================================================================== C ABI
using namespace kopt;

extern "C" {

int kopt_add_rms_norm(void* res, const void* delta, const void* weight, void* out, int M, int N,
                      float eps, void* stream) {
  if (res == nullptr || weight == nullptr || out == nullptr || M < 1 || N < 8 || N % 8 != 0 ||
      N > 8 * 4 * 1024 || !aligned16(res) || !aligned16(weight) || !aligned16(out) ||
      (delta != nullptr && !aligned16(delta)))
    return KOPT_ERR_ARG;
  const int nv = N / 8;
  // one vector per thread up to 1024 threads (all loads of a row in one round), at most 4
  int threads = (nv + 31) / 32 * 32;
  if (threads > 1024) threads = 1024;
  if (nv > 4 * threads) return KOPT_ERR_ARG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M);
  cfg.blockDim = dim3(threads);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, add_rms_norm_kernel, static_cast<bf16*>(res),
                         static_cast<const bf16*>(delta), static_cast<const bf16*>(weight),
                         static_cast<bf16*>(out), N, eps) != cudaSuccess) {
    cudaGetLastError();
    return KOPT_ERR_CUDA;
  }
  return KOPT_OK;
}

int kopt_row_sumsq(const void* x, int M, int K, float* out, void* stream) {
  if (x == nullptr || out == nullptr || M < 1 || K < 8 || K % 8 != 0 || !aligned16(x))
    return KOPT_ERR_ARG;
  row_sumsq_kernel<<<M, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const bf16*>(x), K, out);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

int kopt_silu_mul(const void* gate_up, void* out, int M, int I, void* stream) {
  if (gate_up == nullptr || out == nullptr || M < 1 || I < 8 || I % 8 != 0 || M > 65535 ||
      !aligned16(gate_up) || !aligned16(out))
    return KOPT_ERR_ARG;
  const int nv = I / 8;
  const dim3 grid((nv + 255) / 256, M);
  silu_mul_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const bf16*>(gate_up), static_cast<bf16*>(out), I);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

int kopt_gemv_plan_make(int device, int M, int N, int K, int epi, int target_ctas,
                        kopt_gemv_plan* plan) {
  if (plan == nullptr || M < 1 || M > 64 || K < 8 || K % 8 != 0 || N < 1 || epi < GEMV_F32 ||
      epi > GEMV_ARGMAX || target_ctas < 0)
    return KOPT_ERR_ARG;
  if (N % (epi == GEMV_SWIGLU ? 64 : 16) != 0) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  int occ = 0, sms = 0;
  rc = gemv_configure(device, M, epi, &occ);
  if (rc) return rc;
  if (occ < 1) return KOPT_ERR_CUDA;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    return KOPT_ERR_CUDA;
  const int tiles = epi == GEMV_SWIGLU ? N / 64 : (N + kGRows - 1) / kGRows;
  const int nchunks = (K + kGBK - 1) / kGBK;
  const long long units = static_cast<long long>(tiles) * nchunks;
  // one resident wave: every CTA streams one equal run of units
  long long ctas = target_ctas > 0 ? target_ctas : static_cast<long long>(sms) * occ;
  if (ctas > units) ctas = units;
  const long long per = (units + ctas - 1) / ctas;
  const long long grid = (units + per - 1) / per;
  if (per > 0x7fffffffLL || grid > 0x7fffffffLL) return KOPT_ERR_ARG;
  *plan = kopt_gemv_plan{};
  plan->device = device;
  plan->M = M;
  plan->N = N;
  plan->K = K;
  plan->epi = epi;
  plan->units_per_cta = static_cast<int32_t>(per);
  plan->tiles = tiles;
  plan->grid = static_cast<int32_t>(grid);
  plan->ctas_per_sm = occ;
  plan->flags = 0;
  plan->ws_bytes = gemv_ws_layout(M, tiles, plan->grid).total;
  return KOPT_OK;
}

int kopt_gemv_fused(const kopt_gemv_plan* plan, const void* x, const void* w, void* y, void* ws,
                    const kopt_gemv_fuse* fuse, void* stream) {
  if (plan == nullptr || x == nullptr || w == nullptr || y == nullptr || ws == nullptr)
    return KOPT_ERR_ARG;
  if (fuse != nullptr) {
    if ((fuse->norm_weight != nullptr && !aligned16(fuse->norm_weight)) ||
        (fuse->ss_in != nullptr && (fuse->norm_weight == nullptr || fuse->ss_tiles < 1)) ||
        (fuse->ss_out != nullptr && plan->epi != GEMV_RESID))
      return KOPT_ERR_ARG;
  }
  if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return KOPT_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0) return KOPT_ERR_WORKSPACE;
  int rc = set_device(plan->device);
  if (rc) return rc;
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return KOPT_ERR_CUDA;
  const int mt = gemv_mt(plan->M);
  const bool glu = plan->epi == GEMV_SWIGLU;
  GemvParams p{};
  const cuuint32_t elem[2] = {1, 1};
  const cuuint64_t wdims[2] = {static_cast<cuuint64_t>(plan->K),
                               static_cast<cuuint64_t>(plan->N) * (glu ? 2 : 1)};
  const cuuint64_t xdims[2] = {static_cast<cuuint64_t>(plan->K), static_cast<cuuint64_t>(plan->M)};
  const cuuint64_t stride[1] = {static_cast<cuuint64_t>(plan->K) * 2};
  const cuuint32_t wbox[2] = {kGBK, glu ? 64u : static_cast<cuuint32_t>(kGRows)};
  const cuuint32_t xbox[2] = {kGBK, static_cast<cuuint32_t>(16 * mt)};
  if (enc(&p.tmw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), wdims, stride, wbox,
          elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return KOPT_ERR_ARG;
  if (enc(&p.tmx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims, stride, xbox,
          elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return KOPT_ERR_ARG;
  const int nchunks = (plan->K + kGBK - 1) / kGBK;
  const long long units = static_cast<long long>(plan->tiles) * nchunks;
  if (plan->units_per_cta < 1 || plan->grid != (units + plan->units_per_cta - 1) / plan->units_per_cta)
    return KOPT_ERR_ARG;
  const GemvWs lay = gemv_ws_layout(plan->M, plan->tiles, plan->grid);
  if (lay.total != plan->ws_bytes) return KOPT_ERR_WORKSPACE;
  char* base = static_cast<char*>(ws);
  p.y = y;
  p.xg = static_cast<const bf16*>(x);
  if (fuse != nullptr) {
    p.nw = static_cast<const bf16*>(fuse->norm_weight);
    p.ss_in = fuse->ss_in;
    p.ss_tiles = fuse->ss_tiles;
    p.ss_out = fuse->ss_out;
    p.eps = fuse->eps;
  }
  p.err = reinterpret_cast<int*>(base);
  p.cnt = reinterpret_cast<int*>(base + lay.cnt);
  p.part = reinterpret_cast<float*>(base + lay.part);
  p.keys = reinterpret_cast<unsigned long long*>(base + lay.keys);
  p.units = units;
  p.M = plan->M;
  p.N = plan->N;
  p.K = plan->K;
  p.nchunks = nchunks;
  p.tiles = plan->tiles;
  p.per = plan->units_per_cta;
  return mt == 1 ? gemv_launch_epi<1>(plan, p, stream)
                 : mt == 2 ? gemv_launch_epi<2>(plan, p, stream) : gemv_launch_epi<4>(plan, p, stream);
}

int kopt_gemv(const kopt_gemv_plan* plan, const void* x, const void* w, void* y, void* ws,
              void* stream) {
  return kopt_gemv_fused(plan, x, w, y, ws, nullptr, stream);
}

int kopt_gemv_read_error(const kopt_gemv_plan* plan, void* ws, int* err_out, void* stream) {
  if (plan == nullptr || ws == nullptr || err_out == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(plan->device);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int host = 0;
  if (cudaMemcpyAsync(&host, ws, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return KOPT_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return KOPT_ERR_CUDA;
  *err_out = host;
  if (host != 0 &&   // a timed-out launch may leave counters and keys behind: clear them too
      cudaMemsetAsync(ws, 0,
                      static_cast<size_t>(gemv_ws_layout(plan->M, plan->tiles, plan->grid).part),
                      st) != cudaSuccess)
    return KOPT_ERR_CUDA;
  return KOPT_OK;
}

}  // extern "C"
