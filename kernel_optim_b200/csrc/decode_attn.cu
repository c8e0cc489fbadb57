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
//   * One persistent-style grid of (co-resident CTAs) = slots_per_head * nkv CTAs. Every CTA plans
//     the call on the device from the live lengths pos[b] + 1 (no empty splits, unlike the
//     reference's capacity-sized NSPLIT, fused.py:211-214): if one balanced wave fits, each
//     (sequence, kv head) gets floor(L_b * P / sum L) splits of equal length; otherwise units of a
//     fixed chunk ~ sum L / (P * waves) are dealt round-robin to the CTAs.
//   * Warp 4 is a producer: it streams 64-token K and V tiles (four 16-token pages, 4 KiB each)
//     with cp.async.bulk global->shared copies into a 3-stage ring guarded by mbarriers (no TMA
//     multicast anywhere). Warps 0-3 consume one 16-token page each per tile.
//   * Consumers keep the 4 query rows of the group in registers (16 dims x 4 rows per lane), compute
//     q.k with packed fp32 FMA (fma.rn.f32x2, Blackwell), reduce over 8 lanes with a shuffle
//     reduce-scatter, run an fp32 online softmax (exp2 domain) and accumulate p.v with packed FMA.
//   * The fused variant computes the QK-norm/RoPE prologue in the CTA, appends the new token's K/V
//     to the cache from the CTA that owns position pos[b] and injects that token from shared memory.
//   * Splits of one (sequence, kv head) are merged by the last CTA to finish (atomic counter, no
//     waiting on other CTAs), so the reference's separate combine launch disappears.
//   * Every mbarrier wait is bounded in time; on expiry the kernel records KOPT_DEV_ERR_TIMEOUT,
//     stops issuing copies, waits (bounded) for copies in flight and runs to completion.

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "kopt.h"

namespace kopt {

constexpr int kD = 128;                 // head dim
constexpr int kGroup = 4;               // query heads per kv head
constexpr int kPage = 16;               // tokens per page (and per consumer warp per tile)
constexpr int kNW = 4;                  // consumer warps
constexpr int kTile = kPage * kNW;      // tokens per pipeline stage
constexpr int kStages = 3;
constexpr int kThreads = (kNW + 1) * 32;
constexpr int kMaxB = 256;
constexpr int kDefaultWaves = 4;
constexpr unsigned long long kTimeoutNs = 1000000000ull;  // 1 s per mbarrier wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1.0e30f;     // running-max seed (finite, as fused.py:164)

typedef __nv_bfloat16 bf16;

struct Params {
  const bf16* q;         // [B*T, q_stride] (unfused)
  const bf16* qkv;       // [B, (nq + 2 nkv) * 128] (fused)
  const bf16* qw;        // q_norm weight [128]
  const bf16* kw;        // k_norm weight [128]
  const bf16* cos;       // [rope_len, 128]
  const bf16* sin;
  bf16* q_out;           // optional roped q [B, nq*128]
  bf16* kc;              // cache K (layer base or page pool)
  bf16* vc;
  long long sb, sh;      // contiguous strides (elements)
  const int* bt;         // block table or nullptr
  const int* pos;        // [B]
  bf16* out;             // [B*T, nq*128]
  float* ws_o;           // [max_units, 4, 128]
  float2* ws_ml;         // [max_units, 4]
  int* ws_cnt;           // [B * nkv]
  int* ws_err;
  int bt_stride, num_pages, cap, rope_len;
  int B, T, nkv;
  int slots_per_head, waves;
  float scale_log2, eps;
};

struct __align__(128) Smem {
  bf16 k[kStages][kTile * kD];          // 3 x 16 KiB
  bf16 v[kStages][kTile * kD];          // 3 x 16 KiB
  union {
    float q[kGroup][kD];                // unit prologue: scaled q rows
    float o[kNW][kGroup][kD];           // unit epilogue: per-warp partial outputs
  } u;
  float red_m[kNW][kGroup];
  float red_l[kNW][kGroup];
  float p[kNW][kPage][kGroup];
  float alpha[kNW][kGroup];
  bf16 knew[kD];
  bf16 vnew[kD];
  int prefix[kMaxB + 1];
  int chunk[kMaxB];
  int lens[kMaxB];
  unsigned long long full[kStages];
  unsigned long long empty[kStages];
  int total_units;
  int last_flag;
  volatile int abort;
};

// ------------------------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait. With use_abort, returns false at once when another thread already gave up.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, Smem& s, int* err,
                                          bool use_abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (use_abort && s.abort) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      s.abort = 1;
      atomicOr(err, KOPT_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}
// 1-D bulk copy global -> shared, completion counted on an mbarrier (no multicast).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, "
      "[%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// bf16x2 word -> (low element, high element) as fp32; exact.
__device__ __forceinline__ float2 bf2f(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ float bf16r(float x) {  // round to bf16 (RNE) and back
  return __bfloat162float(__float2bfloat16_rn(x));
}

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
  __nv_bfloat162 a = __floats2bfloat162_rn(y[0], y[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(y[2], y[3]);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(dst) = u;
}

// ---------------------------------------------------------------------------- device plan
__device__ __forceinline__ int ceil_div_i(int a, int b) { return (a + b - 1) / b; }
__device__ __forceinline__ int round16(int a) { return (a + 15) & ~15; }

// Warp 0 fills s.lens / s.chunk / s.prefix / s.total_units from pos[].
__device__ void compute_plan(const Params& p, Smem& s, int lane) {
  long long tot = 0;
  int err = 0;
  for (int b = lane; b < p.B; b += 32) {
    int L = p.pos[b] + p.T;
    if (L < 1 || L > p.cap) {
      err |= KOPT_DEV_ERR_LEN;
      L = L < 1 ? 1 : p.cap;
    }
    s.lens[b] = L;
    tot += L;
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
  if (err && blockIdx.x == 0) atomicOr(p.ws_err, err);
  const int P = p.slots_per_head;
  // Candidate 1: one balanced wave.
  int sum1 = 0, maxc = 0;
  for (int b = lane; b < p.B; b += 32) {
    const int L = s.lens[b];
    int n = static_cast<int>((static_cast<long long>(L) * P) / tot);
    n = n < 1 ? 1 : n;
    const int c = round16(ceil_div_i(L, n));
    n = ceil_div_i(L, c);
    s.chunk[b] = c;
    s.prefix[b + 1] = n;
    sum1 += n;
    maxc = maxc > c ? maxc : c;
  }
  sum1 = __reduce_add_sync(0xffffffffu, sum1);
  maxc = __reduce_max_sync(0xffffffffu, maxc);
  const bool one_wave =
      sum1 <= P && static_cast<long long>(maxc) * sum1 * 4 <= tot * 5 + 64ll * sum1;
  if (!one_wave) {
    const long long per = static_cast<long long>(P) * p.waves;
    long long C = (tot + per - 1) / per;
    if (C > p.cap) C = p.cap;
    const int c = round16(static_cast<int>(C));
    for (int b = lane; b < p.B; b += 32) {
      s.chunk[b] = c;
      s.prefix[b + 1] = ceil_div_i(s.lens[b], c);
    }
  }
  __syncwarp();
  int carry = 0;
  for (int base = 0; base < p.B; base += 32) {
    const int b = base + lane;
    const int n = b < p.B ? s.prefix[b + 1] : 0;
    int incl = n;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += t;
    }
    if (b < p.B) s.prefix[b + 1] = carry + incl;
    carry += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    s.prefix[0] = 0;
    s.total_units = carry * p.nkv;
  }
}

struct Unit {
  int b, kvh, j, n, t0, t1, L;
};

__device__ __forceinline__ Unit unit_of(int u, const Params& p, const Smem& s) {
  Unit r;
  r.kvh = u % p.nkv;
  const int v = u / p.nkv;
  int lo = 0, hi = p.B;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (s.prefix[mid] <= v) lo = mid; else hi = mid;
  }
  r.b = lo;
  r.j = v - s.prefix[lo];
  r.n = s.prefix[lo + 1] - s.prefix[lo];
  r.L = s.lens[lo];
  const int c = s.chunk[lo];
  r.t0 = r.j * c;
  r.t1 = min(r.L, r.t0 + c);
  return r;
}

// Address (elements) of token t's row for (b, kvh); -1 when the page id is out of range.
template <bool PAGED>
__device__ __forceinline__ long long row_offset(const Params& p, int b, int kvh, int t) {
  if (PAGED) {
    const int pid = p.bt[static_cast<long long>(b) * p.bt_stride + t / kPage];
    if (pid < 0 || pid >= p.num_pages) return -1;
    return ((static_cast<long long>(pid) * p.nkv + kvh) * kPage + (t % kPage)) * kD;
  } else {
    return static_cast<long long>(b) * p.sb + static_cast<long long>(kvh) * p.sh +
           static_cast<long long>(t) * kD;
  }
}

// ------------------------------------------------------------------- consumer: one 16-token slab
// ks/vs: up to 16 rows of 128 bf16 in shared memory. Lane layout for q.k: ts = lane/8 picks the
// token within a group of 4, ds = lane%8 the 16 dims {8ds..8ds+7, 64+8ds..64+8ds+7}. For p.v the
// lane owns dims 4*lane..4*lane+3 of all 4 rows.
__device__ __forceinline__ void slab(const bf16* __restrict__ ks, const bf16* __restrict__ vs, int ntok,
                                     const float2 (&qa)[kGroup][4], const float2 (&qb)[kGroup][4],
                                     float& m_row, float& l_part, float2 (&o2)[kGroup][2],
                                     float* __restrict__ p_s, float* __restrict__ alpha_s, int lane) {
  const int ts = lane >> 3, ds = lane & 7;
  const bool hi4 = (ds & 4) != 0, hi2 = (ds & 2) != 0;
  float sc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int t = ts + 4 * k;
    uint4 ka = make_uint4(0, 0, 0, 0), kb = make_uint4(0, 0, 0, 0);
    if (t < ntok) {
      ka = *reinterpret_cast<const uint4*>(ks + t * kD + ds * 8);
      kb = *reinterpret_cast<const uint4*>(ks + t * kD + 64 + ds * 8);
    }
    const uint32_t kw[8] = {ka.x, ka.y, ka.z, ka.w, kb.x, kb.y, kb.z, kb.w};
    float2 acc[kGroup];
#pragma unroll
    for (int r = 0; r < kGroup; ++r) acc[r] = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 kf = bf2f(kw[i]);
#pragma unroll
      for (int r = 0; r < kGroup; ++r) acc[r] = __ffma2_rn(qa[r][i], kf, acc[r]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 kf = bf2f(kw[4 + i]);
#pragma unroll
      for (int r = 0; r < kGroup; ++r) acc[r] = __ffma2_rn(qb[r][i], kf, acc[r]);
    }
    float a[kGroup];
#pragma unroll
    for (int r = 0; r < kGroup; ++r) a[r] = acc[r].x + acc[r].y;
    // reduce-scatter over the 8 ds lanes: rows {0,1}|{2,3} by bit 2, then one row by bit 1
    float keep0 = hi4 ? a[2] : a[0], keep1 = hi4 ? a[3] : a[1];
    const float send0 = hi4 ? a[0] : a[2], send1 = hi4 ? a[1] : a[3];
    keep0 += __shfl_xor_sync(0xffffffffu, send0, 4);
    keep1 += __shfl_xor_sync(0xffffffffu, send1, 4);
    float keep = hi2 ? keep1 : keep0;
    const float send = hi2 ? keep0 : keep1;
    keep += __shfl_xor_sync(0xffffffffu, send, 2);
    keep += __shfl_xor_sync(0xffffffffu, keep, 1);
    sc[k] = t < ntok ? keep : -INFINITY;  // row ds>>1, token ts + 4k
  }
  // online softmax for this lane's row over the slab (16 tokens live in the 4 ts lane groups)
  float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
  const float m_new = fmaxf(m_row, mx);
  const float alpha = exp2f(m_row - m_new);
  float pr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) pr[k] = exp2f(sc[k] - m_new);
  l_part = l_part * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
  m_row = m_new;
  if ((ds & 1) == 0) {
    const int row = ds >> 1;
#pragma unroll
    for (int k = 0; k < 4; ++k) p_s[(ts + 4 * k) * kGroup + row] = pr[k];
    if (ts == 0) alpha_s[row] = alpha;
  }
  __syncwarp();
  const float4 al = *reinterpret_cast<const float4*>(alpha_s);
  const float alv[4] = {al.x, al.y, al.z, al.w};
#pragma unroll
  for (int r = 0; r < kGroup; ++r) {
    const float2 a2 = make_float2(alv[r], alv[r]);
    o2[r][0] = __fmul2_rn(o2[r][0], a2);
    o2[r][1] = __fmul2_rn(o2[r][1], a2);
  }
  auto pv = [&](int t) {
    const float4 pp = *reinterpret_cast<const float4*>(p_s + t * kGroup);
    const uint2 vw = *reinterpret_cast<const uint2*>(vs + t * kD + lane * 4);
    const float2 v01 = bf2f(vw.x), v23 = bf2f(vw.y);
    const float pv4[4] = {pp.x, pp.y, pp.z, pp.w};
#pragma unroll
    for (int r = 0; r < kGroup; ++r) {
      const float2 p2 = make_float2(pv4[r], pv4[r]);
      o2[r][0] = __ffma2_rn(p2, v01, o2[r][0]);
      o2[r][1] = __ffma2_rn(p2, v23, o2[r][1]);
    }
  };
  if (ntok == kPage) {
#pragma unroll
    for (int t = 0; t < kPage; ++t) pv(t);
  } else {
    for (int t = 0; t < ntok; ++t) pv(t);
  }
  __syncwarp();
}

// ------------------------------------------------------------------------------- main kernel
template <bool PAGED, bool FUSED>
__global__ void __launch_bounds__(kThreads, 2) decode_attn_kernel(const Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nq = p.nkv * kGroup;

  if (warp == 0) compute_plan(p, s, lane);
  if (threadIdx.x == 32) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(smem_u32(&s.full[i]), 1);
      mbar_init(smem_u32(&s.empty[i]), kNW);
    }
    s.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int total_units = s.total_units;

  if (warp == kNW) {
    // ------------------------------------------------------------------ producer warp
    const uint64_t pol = evict_first_policy();
    int it = 0;
    bool stop = false;
    for (int u = blockIdx.x; u < total_units && !stop; u += gridDim.x) {
      const Unit U = unit_of(u, p, s);
      const bool inject = FUSED && U.t1 == U.L;
      const int se = inject ? U.L - 1 : U.t1;  // end of the keys streamed from the cache
      const int ntiles = ceil_div_i(se - U.t0, kTile);
      for (int i = 0; i < ntiles; ++i, ++it) {
        const int stage = it % kStages;
        const uint32_t ph = (it / kStages) & 1;
        const int tq = U.t0 + i * kTile + lane * kPage;
        int nt = lane < kNW ? min(max(se - tq, 0), kPage) : 0;
        long long off = 0;
        if (nt > 0) {
          off = row_offset<PAGED>(p, U.b, U.kvh, tq);
          if (off < 0) {
            atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
            nt = 0;
          }
        }
        const uint32_t bytes = static_cast<uint32_t>(nt) * kD * 2;
        const uint32_t total = __reduce_add_sync(0xffffffffu, bytes) * 2;
        int ok = 1;
        if (lane == 0) {
          ok = mbar_wait(smem_u32(&s.empty[stage]), ph ^ 1, s, p.ws_err, true);
          if (ok) mbar_arrive_expect_tx(smem_u32(&s.full[stage]), total);
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          stop = true;
          break;
        }
        if (nt > 0) {
          const uint32_t fb = smem_u32(&s.full[stage]);
          bulk_g2s(smem_u32(&s.k[stage][lane * kPage * kD]), p.kc + off, bytes, fb, pol);
          bulk_g2s(smem_u32(&s.v[stage][lane * kPage * kD]), p.vc + off, bytes, fb, pol);
        }
      }
    }
    // Drain: wait (bounded, ignoring abort) for the copies still in flight into this CTA.
    if (lane == 0) {
      for (int k = 1; k <= kStages && k <= it; ++k) {
        const int i2 = it - k;
        mbar_wait(smem_u32(&s.full[i2 % kStages]), (i2 / kStages) & 1, s, p.ws_err, false);
      }
    }
    return;
  }

  // -------------------------------------------------------------------- consumer warps
  const int ctid = threadIdx.x;  // 0..127
  int it = 0;
  float* p_s = &s.p[warp][0][0];
  float* alpha_s = &s.alpha[warp][0];
  for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
    const Unit U = unit_of(u, p, s);
    const bool inject = FUSED && U.t1 == U.L;
    const int se = inject ? U.L - 1 : U.t1;
    const int ntiles = ceil_div_i(se - U.t0, kTile);
    const int qh = U.kvh * kGroup + warp;  // this warp's query head in the prologue

    // ---- prologue: q rows (and the new K/V for the CTA owning position L-1)
    if (FUSED) {
      const int row = (nq + 2 * p.nkv) * kD;
      const bf16* src = p.qkv + static_cast<long long>(U.b) * row;
      int rp = U.L - 1;
      if (rp >= p.rope_len) {
        if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_ROPE);
        rp = p.rope_len - 1;
      }
      const bf16* cs = p.cos + static_cast<long long>(rp) * kD;
      const bf16* sn = p.sin + static_cast<long long>(rp) * kD;
      float y[4];
      norm_rope_head(src + qh * kD, p.qw, cs, sn, p.eps, lane, y);
#pragma unroll
      for (int j = 0; j < 4; ++j) s.u.q[warp][4 * lane + j] = y[j] * p.scale_log2;
      if (p.q_out != nullptr && U.j == 0)
        store4_bf16(p.q_out + static_cast<long long>(U.b) * nq * kD + qh * kD + 4 * lane, y);
      if (inject && warp < 2) {
        const long long off = row_offset<PAGED>(p, U.b, U.kvh, U.L - 1);
        if (warp == 0) {
          norm_rope_head(src + (nq + U.kvh) * kD, p.kw, cs, sn, p.eps, lane, y);
          store4_bf16(&s.knew[4 * lane], y);
          if (off >= 0) store4_bf16(p.kc + off + 4 * lane, y);
        } else {
          const uint2 raw =
              *reinterpret_cast<const uint2*>(src + (nq + p.nkv + U.kvh) * kD + 4 * lane);
          *reinterpret_cast<uint2*>(&s.vnew[4 * lane]) = raw;
          if (off >= 0) *reinterpret_cast<uint2*>(p.vc + off + 4 * lane) = raw;
        }
        if (off < 0 && lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
      }
    } else {
      const bf16* src = p.q + static_cast<long long>(U.b) * p.T * nq * kD + qh * kD;
      const uint2 raw = *reinterpret_cast<const uint2*>(src + 4 * lane);
      const float2 a = bf2f(raw.x), b = bf2f(raw.y);
      s.u.q[warp][4 * lane + 0] = a.x * p.scale_log2;
      s.u.q[warp][4 * lane + 1] = a.y * p.scale_log2;
      s.u.q[warp][4 * lane + 2] = b.x * p.scale_log2;
      s.u.q[warp][4 * lane + 3] = b.y * p.scale_log2;
    }
    named_bar(1, kNW * 32);
    float2 qa[kGroup][4], qb[kGroup][4];
    {
      const int ds = lane & 7;
#pragma unroll
      for (int r = 0; r < kGroup; ++r) {
        const float4 a0 = *reinterpret_cast<const float4*>(&s.u.q[r][ds * 8]);
        const float4 a1 = *reinterpret_cast<const float4*>(&s.u.q[r][ds * 8 + 4]);
        const float4 b0 = *reinterpret_cast<const float4*>(&s.u.q[r][64 + ds * 8]);
        const float4 b1 = *reinterpret_cast<const float4*>(&s.u.q[r][64 + ds * 8 + 4]);
        qa[r][0] = make_float2(a0.x, a0.y); qa[r][1] = make_float2(a0.z, a0.w);
        qa[r][2] = make_float2(a1.x, a1.y); qa[r][3] = make_float2(a1.z, a1.w);
        qb[r][0] = make_float2(b0.x, b0.y); qb[r][1] = make_float2(b0.z, b0.w);
        qb[r][2] = make_float2(b1.x, b1.y); qb[r][3] = make_float2(b1.z, b1.w);
      }
    }
    named_bar(1, kNW * 32);

    float m_row = kNegBig, l_part = 0.f;
    float2 o2[kGroup][2];
#pragma unroll
    for (int r = 0; r < kGroup; ++r) o2[r][0] = o2[r][1] = make_float2(0.f, 0.f);

    for (int i = 0; i < ntiles; ++i, ++it) {
      const int stage = it % kStages;
      const uint32_t ph = (it / kStages) & 1;
      mbar_wait(smem_u32(&s.full[stage]), ph, s, p.ws_err, true);
      const int tv = min(se - (U.t0 + i * kTile), kTile);
      const int ntok = min(max(tv - warp * kPage, 0), kPage);
      if (ntok > 0)
        slab(&s.k[stage][warp * kPage * kD], &s.v[stage][warp * kPage * kD], ntok, qa, qb, m_row,
             l_part, o2, p_s, alpha_s, lane);
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&s.empty[stage]));
    }
    if (inject && warp == 0)
      slab(s.knew, s.vnew, 1, qa, qb, m_row, l_part, o2, p_s, alpha_s, lane);

    // ---- epilogue: merge the 4 warps, then the splits of this (b, kvh)
    float l = l_part;
    l += __shfl_xor_sync(0xffffffffu, l, 8);
    l += __shfl_xor_sync(0xffffffffu, l, 16);
#pragma unroll
    for (int r = 0; r < kGroup; ++r)
      *reinterpret_cast<float4*>(&s.u.o[warp][r][4 * lane]) =
          make_float4(o2[r][0].x, o2[r][0].y, o2[r][1].x, o2[r][1].y);
    if (lane < 8 && (lane & 1) == 0) {
      s.red_m[warp][lane >> 1] = m_row;
      s.red_l[warp][lane >> 1] = l;
    }
    named_bar(1, kNW * 32);
    const int r = warp;  // output row handled by this thread: query head kvh*4 + r
    float M = kNegBig;
#pragma unroll
    for (int w = 0; w < kNW; ++w) M = fmaxf(M, s.red_m[w][r]);
    float Lsum = 0.f;
    float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float f = exp2f(s.red_m[w][r] - M);
      Lsum += f * s.red_l[w][r];
      const float4 ow = *reinterpret_cast<const float4*>(&s.u.o[w][r][4 * lane]);
      O.x += f * ow.x; O.y += f * ow.y; O.z += f * ow.z; O.w += f * ow.w;
    }
    bf16* dst = p.out + static_cast<long long>(U.b) * p.T * nq * kD + (U.kvh * kGroup + r) * kD +
                4 * lane;
    if (U.n == 1) {
      const float inv = 1.0f / Lsum;
      const float y[4] = {O.x * inv, O.y * inv, O.z * inv, O.w * inv};
      store4_bf16(dst, y);
    } else {
      *reinterpret_cast<float4*>(&p.ws_o[(static_cast<long long>(u) * kGroup + r) * kD + 4 * lane]) = O;
      if (lane == 0) p.ws_ml[static_cast<long long>(u) * kGroup + r] = make_float2(M, Lsum);
      __threadfence();
      named_bar(1, kNW * 32);
      if (ctid == 0) {
        const int prev = atomicAdd(&p.ws_cnt[U.b * p.nkv + U.kvh], 1);
        s.last_flag = prev == U.n - 1;
      }
      named_bar(1, kNW * 32);
      if (s.last_flag) {
        __threadfence();
        const int base = s.prefix[U.b];
        float Mt = kNegBig;
        for (int jj = 0; jj < U.n; ++jj) {
          const int slot = (base + jj) * p.nkv + U.kvh;
          Mt = fmaxf(Mt, __ldcg(&p.ws_ml[static_cast<long long>(slot) * kGroup + r]).x);
        }
        float Lt = 0.f;
        float4 Ot = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int jj = 0; jj < U.n; ++jj) {
          const int slot = (base + jj) * p.nkv + U.kvh;
          const float2 ml = __ldcg(&p.ws_ml[static_cast<long long>(slot) * kGroup + r]);
          const float f = exp2f(ml.x - Mt);
          Lt += f * ml.y;
          const float4 oj =
              __ldcg(reinterpret_cast<const float4*>(&p.ws_o[(static_cast<long long>(slot) * kGroup + r) * kD + 4 * lane]));
          Ot.x += f * oj.x; Ot.y += f * oj.y; Ot.z += f * oj.z; Ot.w += f * oj.w;
        }
        const float inv = 1.0f / Lt;
        const float y[4] = {Ot.x * inv, Ot.y * inv, Ot.z * inv, Ot.w * inv};
        store4_bf16(dst, y);
        if (ctid == 0) atomicExch(&p.ws_cnt[U.b * p.nkv + U.kvh], 0);
      }
    }
    named_bar(1, kNW * 32);
  }
}

// ------------------------------------------------------------- standalone QK-norm/RoPE/append
// Grid (B*T, ceil((nq + 2 nkv) / 4)), 4 warps, one (token, head) per warp: fused.py:54-96.
template <bool PAGED>
__global__ void __launch_bounds__(128) qk_norm_rope_kernel(const Params p, int nheads) {
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
      const long long off = row_offset<PAGED>(p, b, h - nq, ps);
      if (off >= 0) store4_bf16(p.kc + off + 4 * lane, y);
      else if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
    }
  } else {
    const long long off = row_offset<PAGED>(p, b, h - nq - p.nkv, ps);
    if (off >= 0)
      *reinterpret_cast<uint2*>(p.vc + off + 4 * lane) = *reinterpret_cast<const uint2*>(src + 4 * lane);
    else if (lane == 0) atomicOr(p.ws_err, KOPT_DEV_ERR_PAGE);
  }
}

// ------------------------------------------------------------------------------ host side
constexpr int64_t kHeaderBytes = 256;
inline int64_t align256(int64_t x) { return (x + 255) & ~static_cast<int64_t>(255); }

struct WsLayout {
  int64_t err, cnt, ml, o, total;
};
inline WsLayout ws_layout(int B, int nkv, int max_units) {
  WsLayout w;
  w.err = 0;
  w.cnt = kHeaderBytes;
  w.ml = w.cnt + align256(static_cast<int64_t>(B) * nkv * 4);
  w.o = w.ml + align256(static_cast<int64_t>(max_units) * kGroup * 8);
  w.total = w.o + static_cast<int64_t>(max_units) * kGroup * kD * 4;
  return w;
}

template <bool PAGED, bool FUSED>
int attn_occupancy(int device, int* blocks_per_sm) {
  static int configured[64] = {0};
  if (device < 0 || device >= 64) return KOPT_ERR_ARG;
  auto kern = decode_attn_kernel<PAGED, FUSED>;
  if (!configured[device]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(Smem))) != cudaSuccess)
      return KOPT_ERR_CUDA;
    configured[device] = 1;
  }
  if (blocks_per_sm) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, kern, kThreads, sizeof(Smem)) !=
        cudaSuccess)
      return KOPT_ERR_CUDA;
  }
  return KOPT_OK;
}

inline int set_device(int device) {
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return KOPT_ERR_CUDA;
  if (cur != device && cudaSetDevice(device) != cudaSuccess) return KOPT_ERR_CUDA;
  return KOPT_OK;
}

inline bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }

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

int fill_ws(Params& p, const kopt_plan* plan, void* ws) {
  if (ws == nullptr || (reinterpret_cast<uintptr_t>(ws) & 255) != 0) return KOPT_ERR_WORKSPACE;
  const WsLayout w = ws_layout(plan->B, plan->nkv, plan->max_units);
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
  decode_attn_kernel<PAGED, FUSED><<<plan->grid, kThreads, sizeof(Smem),
                                     static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

}  // namespace kopt

// =================================================================================== C ABI
using namespace kopt;

extern "C" {

int kopt_abi_version(void) { return 1; }

const char* kopt_strerror(int status) {
  switch (status) {
    case KOPT_OK: return "ok";
    case KOPT_ERR_ARG: return "invalid argument (shape, head_dim, group, alignment or pointer)";
    case KOPT_ERR_CUDA: return "CUDA runtime call failed";
    case KOPT_ERR_WORKSPACE: return "workspace missing, misaligned or sized for another plan";
    default: return "unknown kopt status";
  }
}

int kopt_decode_attn_plan(int device, int B, int T, int nq, int nkv, int d, int target_ctas,
                          kopt_plan* plan) {
  if (plan == nullptr) return KOPT_ERR_ARG;
  if (d != kD || nkv < 1 || nq != nkv * kGroup || B < 1 || B > kMaxB || T != 1) return KOPT_ERR_ARG;
  int rc = set_device(device);
  if (rc) return rc;
  int slots = target_ctas;
  if (slots <= 0) {
    int sms = 0, occ = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      return KOPT_ERR_CUDA;
    rc = attn_occupancy<true, true>(device, &occ);
    if (rc) return rc;
    // the four instantiations share block size and shared memory, so one occupancy serves all
    rc = attn_occupancy<true, false>(device, nullptr);
    if (rc) return rc;
    rc = attn_occupancy<false, true>(device, nullptr);
    if (rc) return rc;
    rc = attn_occupancy<false, false>(device, nullptr);
    if (rc) return rc;
    slots = sms * (occ > 0 ? occ : 1);
  }
  const int P = slots / nkv > 0 ? slots / nkv : 1;
  plan->B = B;
  plan->T = T;
  plan->nkv = nkv;
  plan->slots_per_head = P;
  plan->grid = P * nkv;
  plan->waves = kDefaultWaves;
  plan->max_units = nkv * (P * kDefaultWaves + B);
  plan->device = device;
  plan->ws_bytes = ws_layout(B, nkv, plan->max_units).total;
  return KOPT_OK;
}

int kopt_workspace_init(const kopt_plan* plan, void* ws, void* stream) {
  if (plan == nullptr || ws == nullptr) return KOPT_ERR_ARG;
  int rc = set_device(plan->device);
  if (rc) return rc;
  const WsLayout w = ws_layout(plan->B, plan->nkv, plan->max_units);
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
    const WsLayout w = ws_layout(plan->B, plan->nkv, plan->max_units);
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
  rc = fill_ws(p, plan, ws);
  if (rc) return rc;
  p.q = static_cast<const bf16*>(q);
  p.pos = pos;
  p.out = static_cast<bf16*>(out);
  p.B = plan->B;
  p.T = plan->T;
  p.nkv = plan->nkv;
  p.slots_per_head = plan->slots_per_head;
  p.waves = plan->waves;
  p.scale_log2 = scale * kLog2e;
  return p.bt ? launch_attn<true, false>(plan, p, stream) : launch_attn<false, false>(plan, p, stream);
}

int kopt_decode_attn_fused(const kopt_plan* plan, const void* qkv, const void* q_norm_w,
                           const void* k_norm_w, const void* cos, const void* sin, int rope_len,
                           const kopt_kv_cache* cache, const int32_t* pos, void* out, void* q_out,
                           void* ws, float scale, float eps, void* stream) {
  if (plan == nullptr || qkv == nullptr || q_norm_w == nullptr || k_norm_w == nullptr ||
      cos == nullptr || sin == nullptr || pos == nullptr || out == nullptr || rope_len < 1)
    return KOPT_ERR_ARG;
  if (!aligned16(qkv) || !aligned16(out) || (q_out && !aligned16(q_out)) || !aligned16(cos) ||
      !aligned16(sin) || (reinterpret_cast<uintptr_t>(q_norm_w) & 7) ||
      (reinterpret_cast<uintptr_t>(k_norm_w) & 7))
    return KOPT_ERR_ARG;
  Params p{};
  int rc = fill_cache(p, cache);
  if (rc) return rc;
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
  p.out = static_cast<bf16*>(out);
  p.B = plan->B;
  p.T = plan->T;
  p.nkv = plan->nkv;
  p.slots_per_head = plan->slots_per_head;
  p.waves = plan->waves;
  p.scale_log2 = scale * kLog2e;
  p.eps = eps;
  return p.bt ? launch_attn<true, true>(plan, p, stream) : launch_attn<false, true>(plan, p, stream);
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
  if (p.bt)
    qk_norm_rope_kernel<true><<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p, nheads);
  else
    qk_norm_rope_kernel<false><<<grid, 128, 0, static_cast<cudaStream_t>(stream)>>>(p, nheads);
  return cudaGetLastError() == cudaSuccess ? KOPT_OK : KOPT_ERR_CUDA;
}

}  // extern "C"
