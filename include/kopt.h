/*
 * kopt.h -- C ABI of the B200 (sm_100a) decode-attention path for the Qwen3-4B engine.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream (as void*), launches
 * asynchronously on that stream, allocates nothing and returns an int status (KOPT_OK == 0).
 * All tensors are bf16 unless stated; head_dim is 128 and the GQA group is 4 (nq == 4 * nkv).
 *
 * Reference interfaces replaced (GodRishUniverse/kernel_optim, paths inside that project):
 *   kopt_decode_attn_plan  <- DecodeAttention.__init__      engine/kernels/fused.py:209-219
 *   kopt_decode_attn       <- DecodeAttention.__call__      engine/kernels/fused.py:221-234
 *                             (_decode_attn_kernel fused.py:138-185 + _decode_combine_kernel
 *                              fused.py:188-201 in one launch)
 *   kopt_qk_norm_rope      <- qk_norm_rope                  engine/kernels/fused.py:99-106
 *                             (_qk_norm_rope_kernel fused.py:54-96)
 *   kopt_decode_attn_fused <- qk_norm_rope + DecodeAttention.__call__ as called back to back in
 *                             Engine._layers, engine/engine.py:328-330 (and engine.py:283-286)
 */
#ifndef KOPT_H_
#define KOPT_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KOPT_API __attribute__((visibility("default")))
#else
#define KOPT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ---------------------------------------------------------------------- */
#define KOPT_OK 0
#define KOPT_ERR_ARG 1         /* bad shape, unsupported head_dim/group, bad pointer alignment */
#define KOPT_ERR_CUDA 2        /* a CUDA runtime call failed (launch, attribute, device query) */
#define KOPT_ERR_WORKSPACE 3   /* workspace too small for the plan */
#define KOPT_ERR_SCRATCH 4     /* plan needs more scratch than kopt_decode_attn_fused_noalloc has */

/* Bits of the device-side error word (read back with kopt_read_error). The kernels never trap:
 * a bad page id or length is recorded here and the access is skipped or clamped. */
#define KOPT_DEV_ERR_PAGE 1    /* block-table entry outside [0, num_pages) */
#define KOPT_DEV_ERR_LEN 2     /* pos[b] + T outside [1, cap] (clamped) */
#define KOPT_DEV_ERR_TIMEOUT 4 /* an mbarrier wait or the gather's flag wait ran past its limit */
#define KOPT_DEV_ERR_ROPE 8    /* pos[b] + t outside the RoPE table (clamped) */
#define KOPT_DEV_ERR_PLAN 16   /* internal work-split invariant violated (work skipped) */

/* ---- KV cache descriptor ---------------------------------------------------------------- *
 * Contiguous (block_table == NULL): one layer's cache [B, nkv, cap, 128] bf16 with arbitrary
 *   batch/head strides (elements, multiples of 8) and token stride 128, as engine/engine.py:186
 *   allocates it and as DecodeAttention receives k_cache[i] (engine.py:395).
 * Paged (block_table != NULL): one layer's page pool [num_pages, nkv, 16, 128] bf16; token t of
 *   sequence b lives in page block_table[b * bt_stride + t / 16], row t % 16. cap is the largest
 *   sequence length the table can address (bt_stride * 16). */
typedef struct kopt_kv_cache {
  void* k;
  void* v;
  int64_t stride_b;          /* contiguous only: elements between sequences */
  int64_t stride_h;          /* contiguous only: elements between kv heads */
  int32_t cap;               /* max tokens per sequence */
  int32_t num_pages;         /* paged only */
  const int32_t* block_table;/* paged only: [B, bt_stride] int32, device */
  int32_t bt_stride;
  int32_t page_size;         /* must be 16 */
} kopt_kv_cache;

/* ---- launch plan -------------------------------------------------------------------------- *
 * Filled by kopt_decode_attn_plan for a fixed (B, T, nkv, max_len) and reused by every call, so the
 * grid and workspace stay fixed across CUDA-graph replays. How the keys are split between CTAs is
 * decided on the device at every call from the live lengths (pos[b] + T): the pages of all
 * (sequence, kv head) pairs are laid end to end; static_pct percent of that line is split into one
 * static piece per CTA and the rest into chunks of chunk_tokens keys that CTAs claim from a
 * counter in the workspace once their piece is done, so SMs served faster take more. */
typedef struct kopt_plan {
  int32_t B;
  int32_t T;
  int32_t nkv;
  int32_t grid;              /* CTAs launched: one wave, SM count x resident CTAs per SM */
  int32_t ctas_per_sm;       /* resident CTAs per SM reported by the occupancy query */
  int32_t tile_tokens;       /* keys per pipeline stage */
  int32_t max_units;         /* partial-result slots in the workspace */
  int32_t device;
  int32_t max_len;           /* largest cache capacity (keys per sequence) a call may pass */
  int32_t chunk_tokens;      /* keys per dynamically scheduled chunk */
  int32_t static_pct;        /* share of the page line split statically, one piece per CTA
                                (environment KOPT_STATIC_PCT overrides the default at plan time) */
  int32_t flags;             /* KOPT_PLAN_* bits: 0 from kopt_decode_attn_plan, set by the caller */
  int64_t ws_bytes;          /* workspace bytes the caller must provide (zeroed once) */
} kopt_plan;

/* plan->flags bit: launch the attention kernel with programmatic dependent launch, so that its
 * CTAs take the SMs that the kernel before it on the stream leaves, and lay out the work split and
 * issue the first K/V page copies before waiting for that kernel to complete. Set it only when the
 * kernel right before the call on its stream writes none of pos, the block table and the cache
 * rows [0, pos[b]) of this call (the fused entry points, and kopt_decode_attn for T > 4; the
 * unfused T = 1 kernel waits before reading anything, and T = 2 .. 4 launches without it): e.g.
 * the QKV projection GEMM of a decode step, the kopt_qk_norm_rope before a verify step, or another
 * decode-attention call for a different layer. q / qkv, the norm weights, the RoPE tables, the rows
 * from pos[b] on, the workspace and the outputs are only touched after the wait. */
#define KOPT_PLAN_OVERLAP_PREV 1

/* Plan a decode-attention launch: B sequences of at most max_len keys, T query tokens each
 * (1 .. 8; T > 1 is the verify step, query t of a sequence seeing keys 0 .. pos + t, and only
 * kopt_decode_attn runs it), nq = 4 * nkv query heads of dim d == 128. target_ctas <= 0 launches
 * one CTA per resident slot (SM count x resident CTAs per SM); a positive value fixes the grid
 * (T = 1) or the number of CTAs the key splits may use (T > 1) instead.
 * Replaces DecodeAttention.__init__ (engine/kernels/fused.py:209-219), which also sizes its
 * scratch from the capacity. */
KOPT_API int kopt_decode_attn_plan(int device, int B, int T, int nq, int nkv, int d, int max_len,
                                   int target_ctas, kopt_plan* plan);

/* Zero a workspace of plan->ws_bytes bytes (split counters and the error word). Call once after
 * allocating it, and again after kopt_read_error reported a timeout. */
KOPT_API int kopt_workspace_init(const kopt_plan* plan, void* ws, void* stream);

/* Copy the device error word (KOPT_DEV_ERR_* bits) to *err_out and clear it. Synchronises the
 * stream. */
KOPT_API int kopt_read_error(const kopt_plan* plan, void* ws, int* err_out, void* stream);

/* Split-K GQA decode attention over a cache whose new K/V are already written at pos[b] (and,
 * for T > 1, at pos[b] + 1 .. pos[b] + T - 1): row b*T + t of out, head h =
 * softmax(q_(b*T+t),h . K[b, h/4, 0..pos[b]+t]^T * scale) V[b, h/4, 0..pos[b]+t].
 * q, out: [B*T, nq*128] bf16 contiguous; pos: [B] int32 device. Writes out and the workspace.
 * Replaces DecodeAttention.__call__(q, k_cache, v_cache, pos, out) (engine/kernels/fused.py:221). */
KOPT_API int kopt_decode_attn(const kopt_plan* plan, const void* q, const kopt_kv_cache* cache,
                     const int32_t* pos, void* out, void* ws, float scale, void* stream);

/* ---- decode-step epilogues (the ops around the projections of a layer) -------------------- */
/* res <- bf16(res + delta) when delta is not NULL; out = bf16(w * bf16(res * rsqrt(mean(res^2)
 * + eps))) per row, fp32 arithmetic. res, delta, out: [M, N] bf16, w: [N]; N a multiple of 8.
 * Launched with programmatic dependent launch: the kernel waits for its predecessor on the stream
 * before touching memory, so ordering is the plain stream order, while the next kernel (a
 * projection launched with KOPT_GEMV_OVERLAP_PREV) may start streaming its weights meanwhile.
 * Replaces add_rms_norm(res, delta, weight, out, eps) (engine/kernels/fused.py:39-46). */
KOPT_API int kopt_add_rms_norm(void* res, const void* delta, const void* weight, void* out, int M,
                               int N, float eps, void* stream);
/* out[m, i] = bf16(bf16(silu(gu[m, i])) * gu[m, I + i]): gate and up side by side in
 * gate_up [M, 2 I], out [M, I] bf16; I a multiple of 8.
 * Replaces silu_mul(gu, out) (engine/kernels/fused.py:123-127). */
KOPT_API int kopt_silu_mul(const void* gate_up, void* out, int M, int I, void* stream);

/* Per-head QK-RMSNorm + RoPE + KV append (no attention), reference cast order:
 * qkv [B*T, (nq + 2 nkv) * 128]; q heads -> q_out [B*T, nq*128]; k heads -> cache k at
 * pos[b] + t; v heads copied to cache v at pos[b] + t. cos/sin: [rope_len, 128] bf16.
 * Replaces qk_norm_rope(qkv, q_w, k_w, cos, sin, pos, q_out, k_cache, v_cache, T, eps, nq, nkv, d)
 * (engine/kernels/fused.py:99-106). */
KOPT_API int kopt_qk_norm_rope(const void* qkv, const void* q_norm_w, const void* k_norm_w,
                      const void* cos, const void* sin, int rope_len, const int32_t* pos,
                      void* q_out, const kopt_kv_cache* cache, int B, int T, int nq, int nkv,
                      int d, float eps, int* dev_err, int device, void* stream);

/* The engine's decode attention step in one launch: the QK-norm/RoPE prologue of the 4 query
 * heads of each group, the new token's K (normed, roped) and V appended to the cache at pos[b]
 * by the CTA that owns that position, and split-K attention over keys 0..pos[b] with the
 * cross-split LSE combine done by the last CTA of each (sequence, kv head).
 * qkv [B, (nq + 2 nkv) * 128] (T == 1); out [B, nq*128]; q_out optional (NULL) receives the
 * roped q. Replaces engine/engine.py:328-330: qk_norm_rope (fused.py:99) then attn1
 * (fused.py:221). */
KOPT_API int kopt_decode_attn_fused(const kopt_plan* plan, const void* qkv, const void* q_norm_w,
                           const void* k_norm_w, const void* cos, const void* sin, int rope_len,
                           const kopt_kv_cache* cache, const int32_t* pos, void* out, void* q_out,
                           void* ws, float scale, float eps, void* stream);

/* ---- multi-GPU: KV-head sharding with the all-gather fused into the attention kernel --------
 * Rank r of G (one GPU each, one node) owns kv heads [r*nkv/G, (r+1)*nkv/G) and runs
 * kopt_decode_attn_fused_gather with a plan for its nkv/G heads. Its CTAs store each finished
 * output row straight into every rank's gathered buffer (plain stores over NVLink through CUDA IPC
 * mappings), at column offset r * nq_local * 128. When all its CTAs are done, the last one raises
 * flags[w][r] = epoch + 1 on every rank w, then waits until every rank's flag in its own array has
 * reached epoch + 1 (bounded by wait_ns, 1 s by default; KOPT_DEV_ERR_TIMEOUT in the workspace
 * error word on expiry, after which the call still completes and its own rows are in place; while
 * that bit stays unread in the error word, later calls through the same workspace raise their
 * flags but do not wait) and
 * advances the epoch: once the call completes on a stream, the gathered rows of all ranks are in
 * this rank's buffer. Every rank must make the same calls in the same order. This takes the place
 * of a separate all-gather (NCCL) of the head outputs between attention and o_proj, which the
 * reference does not have (it runs on one GPU); the attention itself is fused.py:209-219 as for
 * kopt_decode_attn_fused. */
#define KOPT_IPC_HANDLE_BYTES 64
#define KOPT_MAX_RANKS 8
typedef struct kopt_gather {
  void* out[KOPT_MAX_RANKS];   /* out[w]: rank w's gathered buffer [B, row_elems] bf16 */
  int* flags[KOPT_MAX_RANKS];  /* flags[w]: rank w's flag array [world] int32, zeroed once */
  int* epoch;                  /* this rank's call counter (device int32, zeroed once) */
  int32_t rank;
  int32_t world;               /* 1 .. KOPT_MAX_RANKS */
  int64_t row_elems;           /* elements per gathered row: nq_total * 128 */
  int64_t wait_ns;             /* bound of the last CTA's wait for the peers' flags, in ns:
                                  0 = the default 1 s; at most 10 s (KOPT_ERR_ARG above) */
} kopt_gather;

/* kopt_decode_attn_fused whose output goes to every rank's gathered buffer (see above); plan->T 1. */
KOPT_API int kopt_decode_attn_fused_gather(const kopt_plan* plan, const void* qkv,
                                           const void* q_norm_w, const void* k_norm_w,
                                           const void* cos, const void* sin, int rope_len,
                                           const kopt_kv_cache* cache, const int32_t* pos,
                                           const kopt_gather* gather, void* q_out, void* ws,
                                           float scale, float eps, void* stream);

/* Device buffers shared between the ranks' processes (CUDA IPC). alloc zero-fills. */
KOPT_API int kopt_ipc_alloc(int device, int64_t bytes, void** ptr);
KOPT_API int kopt_ipc_free(int device, void* ptr);
KOPT_API int kopt_ipc_get_handle(const void* ptr, void* handle /* KOPT_IPC_HANDLE_BYTES */);
KOPT_API int kopt_ipc_open(int device, const void* handle, void** peer_ptr);
KOPT_API int kopt_ipc_close(int device, void* peer_ptr);

/* ---- prefill: causal GQA attention over the prompt --------------------------------------- *
 * out[b*S + s, h] = softmax over keys 0 .. s of (q[b*S + s, h] . K[b, h/4, key] * scale), times
 * V[b, h/4, key], for B prompts of S tokens each. q, out: [B*S, nq*128] bf16 row-major, 16-byte
 * aligned; q as kopt_qk_norm_rope writes it (normed, roped). The prompt's K/V are read from
 * positions 0 .. S-1 of `cache` (paged or contiguous), where kopt_qk_norm_rope writes them when
 * called with pos = 0 and T = S. dev_err: device int, KOPT_DEV_ERR_* bits OR-ed in (a bad page id
 * is recorded and page 0 read instead; a wait that runs out records KOPT_DEV_ERR_TIMEOUT). On the
 * tcgen05 tensor cores: S = Q K^T and O += P V in tensor memory, K/V tiles fed by TMA, fp32 online
 * softmax. Allocates nothing; not for use while another launch holds this GPU's tensor memory.
 * Replaces F.scaled_dot_product_attention(q, k, v, is_causal=True) with GQA in Engine._prefill
 * (engine/engine.py:376-377). */
KOPT_API int kopt_prefill_attn(const void* q, const kopt_kv_cache* cache, void* out, int B, int S,
                               int nq, int nkv, int d, float scale, int* dev_err, int device,
                               void* stream);

/* kopt_decode_attn_fused without a workspace argument, for callers that cannot allocate device
 * memory for it (an engine that owns the whole memory budget and hands out only fixed buffers, a
 * process whose allocator must not grow after start-up, a plugin host without a device allocator
 * at the call site). This entry point has no counterpart in the reference, which always allocates
 * its scratch (DecodeAttention.__init__). It allocates nothing: the split scratch is an 8 MiB
 * buffer built into this library, present on every GPU that loads it until the process exits.
 *   - Plans whose ws_bytes exceed 8 MiB are rejected with KOPT_ERR_SCRATCH (for example B = 16
 *     sequences of up to 4097 keys need 2.7 MiB; 4 sequences of 131072 keys do not fit).
 *   - The first call on a device resolves the buffer's device address (cudaGetSymbolAddress) with
 *     that device current; make that first call before any stream capture.
 *   - Every call clears the buffer's error word and split counters on `stream` before the launch.
 *     All calls share the one buffer, so calls whose executions overlap on the GPU (other streams,
 *     other threads) race and corrupt each other's results: serialise them.
 *   - dev_err (device int, may be NULL) receives the KOPT_DEV_ERR_* bits of this call. */
KOPT_API int kopt_decode_attn_fused_noalloc(const kopt_plan* plan, const void* qkv,
                                            const void* q_norm_w, const void* k_norm_w,
                                            const void* cos, const void* sin, int rope_len,
                                            const kopt_kv_cache* cache, const int32_t* pos,
                                            void* out, void* q_out, float scale, float eps,
                                            int* dev_err, void* stream);

/* ---- decode-step projections (skinny GEMM) ------------------------------------------------ *
 * y[M, N] = x[M, K] . W[N, K]^T for the rows of a decode batch (M <= 64), bf16 x and W, fp32 sums,
 * each weight read once for all rows, on the tcgen05 tensor cores (weight rows as the MMA's M = 128,
 * decode rows as its N, fp32 accumulators in tensor memory). Replaces Gemv
 * (engine/kernels/gemv.py:109-150) and the
 * epilogues of its kernel (gemv.py:29-106), with its NORM prologue (kopt_gemv_fused). */
#define KOPT_GEMV_F32 0     /* y: float [M, N], the fp32 sums */
#define KOPT_GEMV_BF16 1    /* y: bf16 [M, N] = bf16(sum) */
#define KOPT_GEMV_RESID 2   /* y: the residual h, bf16 [M, N], updated in place: h = bf16(h + bf16(sum)) */
#define KOPT_GEMV_SWIGLU 3  /* W: [gate; up] rows, [2N, K]; y: bf16 [M, N] =
                               bf16(bf16(silu(bf16(gate sum))) * bf16(up sum)) */
#define KOPT_GEMV_ARGMAX 4  /* y: int64 [M], per row the index of the largest bf16(sum), the
                               smallest index among equal values: greedy decoding over the LM
                               head (engine/engine.py:263 logits, then argmax) without writing
                               the [M, N] logits */
typedef struct kopt_gemv_plan {
  int32_t device;
  int32_t M, N, K;
  int32_t epi;               /* KOPT_GEMV_* */
  int32_t units_per_cta;     /* (weight tile, 64-wide K chunk) units per CTA: each CTA streams one
                                contiguous run of them, tile-major; a tile whose units fall to
                                several CTAs is summed from their fp32 partials in CTA order, so
                                results never depend on timing */
  int32_t tiles;             /* weight tiles: ceil(N / 128) (SWIGLU: N / 64 gate rows with their up
                                rows) */
  int32_t grid;              /* CTAs: ceil(tiles * ceil(K / 64) / units_per_cta) */
  int32_t ctas_per_sm;       /* resident CTAs per SM reported by the occupancy query */
  int32_t flags;             /* KOPT_GEMV_* bits below: 0 from kopt_gemv_plan_make */
  int64_t ws_bytes;          /* workspace bytes: error word, counters, partials (zeroed once) */
} kopt_gemv_plan;

/* plan->flags bit: launch with programmatic dependent launch. The CTAs start while the kernel
 * before them on the stream drains and stream their first weight tiles before waiting for it;
 * x, y (h) and the workspace are touched only after the wait, so any predecessor is safe. */
#define KOPT_GEMV_OVERLAP_PREV 1

/* Plan a projection of M rows (1 .. 64), N outputs (a multiple of 16; of 64 for SWIGLU) and K
 * inputs (a multiple of 8). target_ctas = 0 launches one resident wave (one CTA per SM); a
 * positive value asks for that many CTAs instead (at most one per unit). */
KOPT_API int kopt_gemv_plan_make(int device, int M, int N, int K, int epi, int target_ctas,
                                 kopt_gemv_plan* plan);
/* y = epilogue(x . W^T) on `stream`. x: [M, K] bf16 row-major; W: [N, K] (SWIGLU [2N, K]) bf16
 * row-major; all 16-byte aligned; ws: plan->ws_bytes, 256-byte aligned, zero before first use. */
KOPT_API int kopt_gemv(const kopt_gemv_plan* plan, const void* x, const void* w, void* y, void* ws,
                       void* stream);
/* Fusions around a projection (gemv.py:1-20, 66-79, 95-98): the RMSNorm of x applied in shared
 * memory as the x tiles arrive, bf16(norm_weight * bf16(x * rstd)) with rstd = rsqrt(ss / K + eps),
 * and, for KOPT_GEMV_RESID, the row sums of squares of the new residual that the next projection's
 * norm needs. Sums of squares travel as per-tile partials, added in tile order by the consumer, so
 * results never depend on timing (the reference adds them with atomics). */
typedef struct kopt_gemv_fuse {
  const void* norm_weight;   /* bf16 [K], 16-byte aligned; NULL: no norm (x used as it is) */
  const float* ss_in;        /* fp32 [ss_tiles][M] row sums of squares of x (a RESID projection's
                                ss_out, or kopt_row_sumsq); NULL: every CTA sums the x rows
                                itself (correct, but a latency-bound pass of several µs) */
  int32_t ss_tiles;
  float eps;
  float* ss_out;             /* KOPT_GEMV_RESID only: fp32 [plan->tiles][M]; NULL: not written */
} kopt_gemv_fuse;
/* out[m] = sum over k of x[m][k]^2 (x bf16 [M, K] row-major, 16-byte aligned, K a multiple of 8;
 * out fp32 [M]), one CTA per row, sums in a fixed order: the ss_in of a fused RMSNorm when no
 * residual projection wrote it (the reference's embed_ss, engine/kernels/gemv.py:202-217). */
KOPT_API int kopt_row_sumsq(const void* x, int M, int K, float* out, void* stream);
/* kopt_gemv with the fusions above (fuse may be NULL). Replaces Gemv.__call__ with norm=True and
 * the ss / ss_out hand-off of engine/kernels/gemv.py:140-150. */
KOPT_API int kopt_gemv_fused(const kopt_gemv_plan* plan, const void* x, const void* w, void* y,
                             void* ws, const kopt_gemv_fuse* fuse, void* stream);
/* Copy the workspace error word (KOPT_DEV_ERR_TIMEOUT) to *err_out and clear it. Synchronises. */
KOPT_API int kopt_gemv_read_error(const kopt_gemv_plan* plan, void* ws, int* err_out, void* stream);

/* Human-readable text for a KOPT_* status. */
KOPT_API const char* kopt_strerror(int status);

/* ABI version of this library (bumped on any signature change). */
KOPT_API int kopt_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KOPT_H_ */
