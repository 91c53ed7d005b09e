/* ork_npu.h -- resident-weight matmul engine, B200 (sm_100a) implementation.
 *
 * Drop-in for the hot path of ork-driver's C API (ork-driver include/ork_npu.h and its parts
 * include/ork/{context,weights,run}.h): pack a weight B[K,N] once into HBM-resident storage, then run
 * C = A.B many times, and persist / reload int4 weights in the compact 'O4N1' blob. Same symbol names,
 * argument meanings, return conventions and blob bytes as the reference; the device behind them is a
 * CUDA GPU instead of an RK35xx NPU, so the NPU-specific surface (IOMMU domains, orkd, SDP LUTs, core
 * budgets, regcmd probes) is not part of this library.
 *
 *   int8   C[M,N] int32 = A[M,K] int8  x B[K,N] int8   (raw sums; caller applies scales)
 *   w4a8   C[M,N] int32 = A[M,K] int8  x int4-quantized B (uniform grid or NF4 codebook, nibbles in HBM)
 *   W4A4   C[M,N] int32 = A[M,K] int4-in-int8 x B[K,N] int4-in-int8
 *   fp16   C[M,N] fp32  = A[M,K] fp16  x B[K,N] fp16
 *
 * A and C are row-major; run calls are synchronous: when a run returns 0, C is complete. A and C may be
 * host pointers (copied through the context's CUDA stream) or device pointers (used in place).
 * Threading: one context per process and per GPU; calls on one context are not thread-safe, exactly as
 * in the reference (ork-driver include/ork_npu.h:20, include/ork/context.h:60-68).
 */
#ifndef ORK_NPU_H
#define ORK_NPU_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ork-driver include/ork_npu.h:19-21. The fp16 element type is the compiler's IEEE binary16; compilers
 * without _Float16 may define ORK_F16_AS_U16 to see the same bits as uint16_t (identical ABI). */
#ifdef ORK_F16_AS_U16
typedef uint16_t ork_f16;
#else
typedef _Float16 ork_f16;
#endif
typedef struct ork_npu ork_npu; /* device context (one per process per GPU) */
typedef struct ork_w ork_w;     /* resident packed weights for one B[K,N] */

/* ork-driver include/ork_npu.h:30 and :37. */
#define ORK_NPU_VERSION "1.0.190"
#define ORK_PACK_FORMAT_VERSION 1u

/* ork-driver include/ork/weights.h:115: int4 weight-store codebook kind. */
enum { ORK_QK_UNIFORM = 0, ORK_QK_CODEBOOK_NF4 = 1 };

/* ork-driver include/ork/run.h:27. Never returned here: every shape inside the API's dimension rules
 * has a verified path on the GPU. Defined so callers that test for it still compile. */
#define ORK_RC_WEDGE_PRONE (-501)

/* ---- context (ork-driver include/ork/context.h) ------------------------------------------------ */

/* include/ork/context.h:14. "1.0.190+b200". */
const char *ork_npu_version(void);
/* include/ork/context.h:37. The O4N1 blob version this build reads and writes (1). */
uint32_t ork_pack_format_version(void);
/* include/ork/context.h:73. Opens the calling thread's current CUDA device (cudaSetDevice first to pick
 * another), creates the context's stream. NULL when no CUDA device is present or usable. */
ork_npu *ork_npu_init(void);
/* include/ork/context.h:83. Frees the context. Weights packed on it must be freed first (ork_mm_free). */
void ork_npu_free(ork_npu *ctx);

/* ---- pack / load / dump (ork-driver include/ork/weights.h) -------------------------------------- */

/* include/ork/weights.h:39. B row-major fp16 [K][N]; K%32==0, N%16==0, else NULL. */
ork_w *ork_f16_mm_pack(ork_npu *ctx, int K, int N, const ork_f16 *B);
/* include/ork/weights.h:47. B row-major int8 [K][N]; K%32==0, N%32==0, else NULL. */
ork_w *ork_i8_mm_pack(ork_npu *ctx, int K, int N, const int8_t *B);
/* include/ork/weights.h:92. f32 given n-major [N][K]; per-output-channel symmetric int8:
 * bscale[n] = max(1e-9,max|w|)/127, code = clamp(rint(w*(127/max)), +-127). Writes bscale_out[N] when
 * non-NULL; the weight itself keeps no scale (ork_w_bscale returns NULL), as in the reference. */
ork_w *ork_i8_mm_pack_f32(ork_npu *ctx, int K, int N, const float *f32, float *bscale_out);
/* include/ork/weights.h:116. w4a8: f32 n-major [N][K] quantized per output channel to int4, kept as
 * nibbles in HBM. Uniform grid (scale = max/7, codes in [-7,7]) unless env ORK_NF4 is set (NF4 codebook,
 * bscale = max/127, quant_kind = ORK_QK_CODEBOOK_NF4). Env ORK_SR selects stochastic rounding. The weight
 * runs through ork_i8_mm_run. K%32, N%32. */
ork_w *ork_i4a8_mm_pack(ork_npu *ctx, int K, int N, const float *f32, float *bscale_out);
/* include/ork/weights.h:124. As above with an optional importance matrix imatrix[K] selecting each
 * channel's clip scale from the grid {1,.92,.85,.78,.70,.62,.55}; NULL is byte-identical to the above. */
ork_w *ork_i4a8_mm_pack_im(ork_npu *ctx, int K, int N, const float *f32, const float *imatrix, float *bscale_out);
/* include/ork/weights.h:125. W4A4: B row-major int8 [K][N] holding int4 values [-8,7] (the low nibble
 * is kept). K%32, N%64. Runs through ork_i4_mm_run. */
ork_w *ork_i4_mm_pack(ork_npu *ctx, int K, int N, const int8_t *B);

/* include/ork/weights.h:230. Compact int4 persist of an ork_i4a8_mm_pack(_im)/ork_i4a8_mm_load weight:
 * {u32 0x4F344E31 'O4N1', u32 version 1, i32 K, i32 N, u32 quant_kind} + bscale[N] f32 + nibbles[N][K/2]
 * (low nibble = even k). out == NULL returns the size; returns 0 if cap is short or w has no int4 store. */
size_t ork_i4a8_w_dump(const ork_w *w, void *out, size_t cap);
/* include/ork/weights.h:255. Reload an O4N1 blob; NULL unless the size is exact and magic, version, K,
 * N and quant_kind all check. The loaded weight runs via ork_i8_mm_run and re-dumps byte-identically. */
ork_w *ork_i4a8_mm_load(ork_npu *ctx, int K, int N, const void *blob, size_t n);
/* include/ork/weights.h:288 and :294. CPU-only O4N1 writer: the exact bytes ork_i4a8_mm_pack_im +
 * ork_i4a8_w_dump would produce (nf4 chosen by the argument, not ORK_NF4), with no device involved; the
 * _qerr form also reports sqrt(sum imp*(w-q)^2 / sum imp*w^2). ctx may be NULL. out == NULL -> size. */
size_t ork_i4a8_pack_cpu_blob(ork_npu *ctx, int K, int N, const float *f32, const float *imatrix, int nf4,
                              void *out, size_t cap);
size_t ork_i4a8_pack_cpu_blob_qerr(ork_npu *ctx, int K, int N, const float *f32, const float *imatrix,
                                   int nf4, void *out, size_t cap, float *qerr_out);

/* ---- persisted tiled weights (.orkpack entries; ork-driver include/ork/weights.h:159-269) --------
 * Every blob from ork_w_dump / ork_*_w_dump_cpu starts with this one-page header and every
 * ork_*_mm_load* refuses a blob whose stamp disagrees with this build (src/npu/core/packhdr.c). The
 * header layout, magic, refusal order and codes are the reference's; `capid` identifies THIS build's
 * caps (B200, K-major resident rows) and `soc` reads "b200", so a blob tiled for an RK35xx NPU is
 * refused with ORK_PACKERR_CAPS here and a B200 blob is refused the same way by an NPU build. After the
 * header the payload is the weight's resident layout: int8 [N][K] (int4 stores inflated to their int8
 * codes), fp16 [N][K], or W4A4 nibbles [N][K/2] with the low nibble holding the even k. */
#define ORK_PACK_MAGIC 0x4b50414fu /* "OAPK" */
#define ORK_PACK_HDR_BYTES 4096u
typedef struct {
  uint32_t magic;     /* ORK_PACK_MAGIC */
  uint32_t fmt;       /* ork_pack_format_version() at dump time */
  uint32_t capid;     /* resolved-caps identity of the dumping build */
  uint32_t dtype;     /* 0 fp16, 1 int8, 2 int4 (ork-driver include/ork/run.h:42) */
  int32_t K, N;
  uint32_t hdr_bytes; /* == ORK_PACK_HDR_BYTES */
  uint32_t flags;     /* reserved, 0 */
  char soc[16];       /* device id at dump time, for the diagnostic */
} ork_pack_hdr;       /* zero-padded to ORK_PACK_HDR_BYTES */
#define ORK_PACKERR_SHORT (-1)
#define ORK_PACKERR_UNSTAMPED (-2)
#define ORK_PACKERR_FORMAT (-3)
#define ORK_PACKERR_CAPS (-4)
#define ORK_PACKERR_SHAPE (-5)
/* include/ork/weights.h:199. == ORK_PACK_HDR_BYTES. */
size_t ork_pack_hdr_bytes(void);
/* include/ork/weights.h:203. Header + the weight's resident bytes; out == NULL returns the size, 0 on a
 * short cap or a NULL weight. An int4-store weight (ork_i4a8_*) dumps as int8 (its inflated codes), as
 * the reference's resident int8 tiles do, and reloads with ork_i8_mm_load. */
size_t ork_w_dump(const ork_w *w, void *out, size_t cap);
/* include/ork/weights.h:210. The exact bytes ork_i8_mm_pack(B) + ork_w_dump would give, computed on the
 * host with no device (ctx may be NULL). B row-major int8 [K][N]; K%32, N%32. out == NULL -> size. */
size_t ork_i8_w_dump_cpu(ork_npu *ctx, int K, int N, const int8_t *B, void *out, size_t cap);
/* include/ork/weights.h:213. The NPU's full-K companion tiling has no counterpart in the K-major B200
 * layout (every weight is already full-K): always 0, the reference's "no companion" answer. */
size_t ork_i8_w_dump_bf_cpu(ork_npu *ctx, int K, int N, const int8_t *B, void *out, size_t cap);
/* include/ork/weights.h:219. The exact bytes ork_i4_mm_pack(B) + ork_w_dump would give (W4A4, dtype 2),
 * host only (ctx may be NULL). K%32, N%64. out == NULL -> size. */
size_t ork_i4_w_dump_cpu(ork_npu *ctx, int K, int N, const int8_t *B, void *out, size_t cap);
/* include/ork/weights.h:226, :229, :265. Reload a stamped blob of that dtype and (K,N); NULL on any header
 * refusal (the cause is printed once) or a size that is not header + payload exactly. */
ork_w *ork_f16_mm_load(ork_npu *ctx, int K, int N, const void *blob, size_t n);
ork_w *ork_i8_mm_load(ork_npu *ctx, int K, int N, const void *blob, size_t n);
ork_w *ork_i4_mm_load(ork_npu *ctx, int K, int N, const void *blob, size_t n);
/* include/ork/weights.h:243. Load a W4A4 blob (ork_i4_w_dump_cpu / ork_w_dump of an int4 weight) as an
 * int8-compute weight: the int4 values are its int8 codes (sign-extended), it runs with ork_i8_mm_run,
 * and with G > 0 dividing K it is tagged for ork_i8_mm_run_grouped. Carries no scales. */
ork_w *ork_i4a8_mm_load_tiled(ork_npu *ctx, int K, int N, const void *blob, size_t n, int G);

/* ---- per-group scales (ork-driver include/ork/weights.h:126-132, include/ork/run.h:121-125) ------- */

/* include/ork/weights.h:128. W4A4 weight with K split into groups of G: G%32, K%G, G <= 10752, plus the
 * ork_i4_mm_pack rules (K%32, N%64). Runs with ork_i4_mm_run_grouped (and ork_i4_mm_run). */
ork_w *ork_i4_mm_pack_grouped(ork_npu *ctx, int K, int N, const int8_t *B, int G);
/* include/ork/weights.h:132 (src/npu.c:1191). Tag an int4 or int8 weight with group size G (0 clears);
 * -1 for fp16 / NULL weights or a G that does not divide K. */
int ork_w_set_group(ork_w *w, int G);
/* include/ork/run.h:121 and include/ork/weights.h:253. C fp32 [M][N] = sum over K-groups g (ascending)
 * of ((float)dot_g(A[m], B[:,n]) * aScale[m*(K/G)+g]) * bScale[g*N+n], the int32 group dot exact and
 * every fp32 multiply and add rounded separately -- bit-identical to ork-driver's CPU accumulate
 * (src/npu/core/buf.c:501-520). _i4_: W4A4 weight, A int4 values in int8; _i8_: any int8-compute weight
 * (int8, int4 store or tiled-loaded) with a group size, A int8. Group sizes: G%16 for int8 weights,
 * G%32 for int4 weights. 0 ok; -1 on bad arguments, an ungrouped weight, overlapping A/C, or a device
 * error. */
int ork_i4_mm_run_grouped(ork_npu *ctx, ork_w *w, int M, const int8_t *A, const float *aScale,
                          const float *bScale, float *C);
int ork_i8_mm_run_grouped(ork_npu *ctx, ork_w *w, int M, const int8_t *A, const float *aScale,
                          const float *bScale, float *C);

/* ---- batches of independent matmuls (ork-driver include/ork/dynamic.h:14-30, include/ork/chain.h:
 * 110-120, include/ork/run.h:119-120) --------------------------------------------------------------- */

/* include/ork/dynamic.h:14-28. One matmul of a batch: C = A . w with the run rules of ork_i8_mm_run /
 * ork_i4_mm_run; cstride (int8 tasks) is C's row stride in elements, 0 = w's N. */
typedef struct {
  ork_w *w;
  int M;
  const int8_t *A;
  int32_t *C;
  int cstride;
} ork_mm_task_i8;
typedef struct {
  ork_w *w;
  int M;
  const int8_t *A;
  int32_t *C;
} ork_mm_task_i4;
/* include/ork/dynamic.h:30, include/ork/chain.h:120 (stream), :110 (int4 chain), include/ork/dynamic.h:33
 * (experts; nc, the NPU core count, is ignored). Run S independent matmuls as one batch: decode-sized
 * tasks (M <= 8) of one weight format share ONE kernel launch, larger tasks follow on the same stream;
 * synchronous, every C complete on return. 0 ok; -1 on bad arguments (a NULL or wrong-dtype weight,
 * M < 1, NULL A/C, cstride < N, A/C overlap) or a device error. S = 0 is a no-op. */
int ork_i8_mm_run_chain(ork_npu *ctx, int S, const ork_mm_task_i8 *tasks);
int ork_i8_mm_run_stream(ork_npu *ctx, int S, const ork_mm_task_i8 *tasks);
int ork_i4_mm_run_chain(ork_npu *ctx, int S, const ork_mm_task_i4 *tasks);
int ork_i4_mm_run_experts(ork_npu *ctx, const ork_mm_task_i4 *ex, int ntask, int nc);
/* include/ork/run.h:119-120. Asynchronous submit of one matmul (any weight dtype; A int8/int4 or fp16 as
 * the weight's run function takes, copied at submit) into a ring of 8 in-flight slots; returns a ticket
 * >= 0, or -1 when the arguments are bad or all slots are in flight (collect first). ork_mm_collect waits
 * for that ticket's matmul, writes C (int32 or fp32 [M][N]) and frees the slot: 0 ok, -1 for an unknown or
 * already collected ticket or a device error. */
int ork_mm_submit(ork_npu *ctx, ork_w *w, int M, const void *A);
int ork_mm_collect(ork_npu *ctx, int ticket, void *C);
/* include/ork/chain.h:123. The int4 (W4A4) batch, twin of ork_i8_mm_run_stream: same meaning and return
 * codes as ork_i4_mm_run_chain (the reference deals the tasks over its NPU cores; the GPU serves the
 * whole batch). */
int ork_i4_mm_run_stream(ork_npu *ctx, int S, const ork_mm_task_i4 *tasks);

/* include/ork/chain.h:124-143. Runs that return at once, joined by ork_async_wait. Same buffers, checks,
 * numerics and results as the synchronous call of the same name without _async (host or device
 * buffers). The whole job is queued on the context's stream -- A in (through pinned staging when A is
 * pageable host memory), the kernels, C out (to pinned staging when C is pageable) -- and the call
 * returns; ork_async_wait waits for it, copies staged results into C, and returns the job's status
 * (0 ok, -1 on any error the synchronous call would report) and frees the handle. No thread is
 * created. A launcher returns NULL for a NULL context or weight, M < 1, an int8 run on a weight of
 * another kind, an empty or NULL task list (the reference's refusals), or when a job is already in
 * flight on the context; ork_async_wait(NULL) returns -1. Contract (the reference's, enforced here):
 * one job in flight per context; until its wait every other run on the context returns -1; A, C and
 * the task arrays stay valid until the wait. */
typedef struct ork_async ork_async;
ork_async *ork_mm_run_async(ork_npu *ctx, ork_w *w, int M, const ork_f16 *A, float *C);
ork_async *ork_i8_mm_run_async(ork_npu *ctx, ork_w *w, int M, const int8_t *A, int32_t *C);
ork_async *ork_i4_mm_run_async(ork_npu *ctx, ork_w *w, int M, const int8_t *A, int32_t *C);
ork_async *ork_i8_mm_run_chain_async(ork_npu *ctx, int S, const ork_mm_task_i8 *tasks);
ork_async *ork_i4_mm_run_chain_async(ork_npu *ctx, int S, const ork_mm_task_i4 *tasks);
ork_async *ork_i8_mm_run_stream_async(ork_npu *ctx, int S, const ork_mm_task_i8 *tasks);
ork_async *ork_i4_mm_run_stream_async(ork_npu *ctx, int S, const ork_mm_task_i4 *tasks);
int ork_async_wait(ork_async *h);
/* include/ork/chain.h:146. The CPU (sched_getcpu) of the thread that queued the context's latest
 * ork_async job, -1 if none (the reference records its worker thread's CPU). */
int ork_npu_last_async_cpu(ork_npu *ctx);

/* include/ork/chain.h:105-110. One decode token through a Llama/Qwen-style layer: x fp32 [D] ->
 * RMSNorm(attn_norm) -> per-tensor int8 -> q, k, v projections -> per head: RMSNorm(q_norm), RoPE NeoX at
 * `pos` (base rope_base), attention over the nkv cached keys/values (Kc, Vc fp32 [Hkv][nkv][dk], grouped
 * query heads) -> int8 -> o projection -> residual -> RMSNorm(ffn_norm) -> int8 -> gate, up -> SwiGLU ->
 * int8 -> down -> residual = x_out [D]. The arithmetic of src/npu/i8/chain.c:106-122 with the glue of
 * src/spine_kernels.h; the k and v projections are computed as in the reference but the caches are only
 * read (see ork_b200_i8_mm_layer_async in ork_b200.h for the appending form). Weights: int8-compute weights
 * (wq D x H*dk, wk / wv D x Hkv*dk, wo H*dk x D, wg / wu D x Nff, wd Nff x D). dv must equal dk. Host or
 * device pointers; synchronous. 0 ok, -3 on bad arguments or shapes, -1 on a device error. */
struct ork_layer_dims {
  uint32_t D, H, Hkv, dk, dv, Nff, nkv, pos;
  double attn_scale, rope_base;
};
int ork_i8_mm_layer(ork_npu *ctx, const struct ork_layer_dims *d, ork_w *wq, ork_w *wk, ork_w *wv, ork_w *wo,
                    ork_w *wg, ork_w *wu, ork_w *wd, const float *attn_norm, const float *q_norm,
                    const float *ffn_norm, const float *x, const float *Kc, const float *Vc, float *x_out);

/* include/ork/weights.h:141. Frees a weight's host bookkeeping. Unlike the reference (which leaves the
 * NPU window to teardown), device memory is released here as well: HBM has no IOVA window to protect. */
void ork_w_free(ork_w *w);
/* include/ork/weights.h:149. Frees a weight and its device memory. */
void ork_mm_free(ork_npu *ctx, ork_w *w);
/* include/ork/weights.h:150. Resident device bytes of the packed weight. */
size_t ork_w_bytes(const ork_w *w);
/* include/ork/weights.h:154. (K,N) of the weight; NULL w yields 0,0. */
void ork_w_dims(const ork_w *w, int *K, int *N);
/* include/ork/weights.h:155. ORK_QK_* of an int4 weight store; 0 for other weights, -1 for NULL. */
int ork_w_quant_kind(const ork_w *w);
/* include/ork/weights.h:158. Per-output-channel scale[N] of an int4-packed/loaded weight, else NULL. */
const float *ork_w_bscale(const ork_w *w);

/* ---- run (ork-driver include/ork/run.h, include/ork/weights.h:345) ------------------------------- */

/* include/ork/weights.h:345. C fp32 [M][N] = A fp16 [M][K] x B. 0 ok; -1 on bad args, a weight of
 * another dtype, overlapping A/C, or a device error. */
int ork_f16_mm_run(ork_npu *ctx, ork_w *w, int M, const ork_f16 *A, float *C);
/* include/ork/run.h:21. C int32 [M][N] = A int8 [M][K] x B, exact. Accepts int8 packs (ork_i8_mm_pack,
 * ork_i8_mm_pack_f32) and int4 stores (ork_i4a8_mm_pack(_im), ork_i4a8_mm_load). Errors as above. */
int ork_i8_mm_run(ork_npu *ctx, ork_w *w, int M, const int8_t *A, int32_t *C);
/* include/ork/run.h:111. W4A4: C int32 = A (int4 values in int8) x B; exact int32 accumulation. */
int ork_i4_mm_run(ork_npu *ctx, ork_w *w, int M, const int8_t *A, int32_t *C);

/* Fused output stages (include/ork/run.h:48-108). The int8 matmul's int32 sum requantized in the output
 * stage: out = clamp(rne(acc * mult / 2^shift)) with rne = round half to even (the reference's own model
 * of its NPU stage, examples/test_mm_i8_out8.c:24-33), clamped to int8 (out8) or int16 (out16); ewmul
 * multiplies by G (int8 [M][N], e.g. silu(gate)) first: C = clamp_i8(rne(acc * G * mult / 2^shift)), the
 * up projection of a fused SwiGLU. Weights: int8-compute (ork_i8_mm_pack(_f32), int4 stores). Returns 0;
 * -2 for another weight kind, K not a multiple of 512 or above 4096, N not a multiple of 32 (the
 * reference's limits, kept for identical refusals), or a negative mult / shift; -1 on NULL or overlapping
 * buffers or a device error. M <= 0 does nothing and returns 0. Host or device buffers. */
int ork_i8_mm_run_out8(ork_npu *ctx, ork_w *w, int M, const int8_t *A, int8_t *C, int mult, int shift);
int ork_i8_mm_run_out16(ork_npu *ctx, ork_w *w, int M, const int8_t *A, short *C, int mult, int shift);
int ork_i8_mm_run_ewmul(ork_npu *ctx, ork_w *w, int M, const int8_t *A, const int8_t *G, int8_t *C, int mult,
                        int shift);
/* include/ork/sdp.h:45-52. Standalone element-wise multiply: out[m][n] = clamp_i8(rne(up * silu * mult /
 * 2^shift)). -2 outside M 1..8176, N 16..8192 (multiple of 16), mult 0..0x7fff, shift 0..31; -1 on NULL
 * or overlapping buffers. us (may be NULL) receives the kernel's device time in microseconds. */
int ork_i8_npu_ewmul(ork_npu *ctx, const int8_t *up, const int8_t *silu, int M, int N, int mult, int shift,
                     int8_t *out, double *us);

/* include/ork/run.h:132. The API's explicit CPU int8 matmul (B row-major raw codes). It exists for
 * callers who want to time the CPU side of a routing decision; no run function above ever calls it. */
void ork_i8_mm_run_cpu(int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C);

#ifdef __cplusplus
}
#endif
#endif /* ORK_NPU_H */
