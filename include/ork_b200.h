/* ork_b200.h -- B200-specific additions to the ork_npu.h API.
 *
 * Every name here starts with ork_b200_ (except ork_i8_mm_run_noalloc, which the reference does not
 * have either) so that none collides with a name of ork-driver's own API: where the reference has a
 * function of the same purpose, ork_npu.h declares it with the reference's name and prototype, and the
 * B200 form here carries the prefix (the reference's ork_i8_mm_run_async, for instance, takes host
 * buffers and returns an ork_async handle; ork_b200_i8_mm_run_async takes device buffers and is
 * stream-ordered).
 *
 * The reference's run calls are synchronous over host buffers; on a GPU the same matmuls are most
 * useful stream-ordered over device buffers, so they can be queued back to back (or captured in a CUDA
 * graph) without a host round trip per call. These entry points expose that, plus the little a caller
 * needs to integrate the context with its own CUDA stream. Entry points documented as taking device
 * pointers check, before anything is queued, that each one is memory of the context's GPU (or managed
 * memory), and return -1 (-3 for the layer calls) with a message when one is not. Include after
 * ork_npu.h.
 */
#ifndef ORK_B200_H
#define ORK_B200_H
#include "ork_npu.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Asynchronous device-pointer runs: A and C must be device memory of the context's GPU; the matmul is
 * enqueued on the context's stream and the call returns without waiting. Same argument rules and return
 * codes as the synchronous runs; launch errors are reported here, execution errors by ork_b200_sync. The
 * host-buffer forms with an ork_async handle are ork_npu.h's ork_*_mm_run_async. */
int ork_b200_i8_mm_run_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, int32_t *dC);
int ork_b200_i4_mm_run_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, int32_t *dC);
int ork_b200_f16_mm_run_async(ork_npu *ctx, ork_w *w, int M, const ork_f16 *dA, float *dC);

/* No counterpart in ork-driver. ork_i8_mm_run for callers that cannot let a library allocate device
 * memory at run time (an engine that reserved nearly all HBM for its own pool at start-up, a process
 * under a hard device-memory cap, or code that must not trigger the device-wide synchronisation
 * cudaMalloc / cudaFree can cause). Same arguments, checks and result as ork_i8_mm_run: device-resident
 * A and C are used in place, and host A and C are staged through a fixed 4 MiB scratch area built into
 * the library (held on every GPU that loads it) instead of buffers the context allocates; the call
 * allocates nothing. Limit: the host buffers' share -- M*K rounded up to 256 for a host A, 4*M*N for a
 * host C -- must fit in 4 MiB, else -1 with a message. The first call on a device looks up the scratch
 * address (make it before any stream capture). One scratch array per GPU serves every call, so calls on
 * one device must not overlap (they would race on it). */
int ork_i8_mm_run_noalloc(ork_npu *ctx, ork_w *w, int M, const int8_t *A, int32_t *C);

/* Grouped runs over device pointers (A, aScale, bScale, C on the context's GPU), enqueued like the
 * async runs above; same arguments and checks as ork_i4_mm_run_grouped / ork_i8_mm_run_grouped. */
int ork_b200_i4_mm_run_grouped_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, const float *daScale,
                                const float *dbScale, float *dC);
int ork_b200_i8_mm_run_grouped_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, const float *daScale,
                                const float *dbScale, float *dC);

/* ork_i8_mm_run_chain over device pointers (every A and C on the context's GPU), enqueued without waiting:
 * the batch's decode-sized tasks go into one launch, as in the synchronous form. A task with a C row
 * stride other than N must be decode-sized (M <= 8). Capturable in a CUDA graph. */
int ork_b200_i8_mm_run_chain_async(ork_npu *ctx, int S, const ork_mm_task_i8 *tasks);

/* The fused output stages (ork_i8_mm_run_out8 / _out16 / _ewmul) over device pointers, enqueued without
 * waiting. Decode-sized runs (M <= 8) requantize inside the matmul kernel; larger M use a context scratch
 * for the int32 sums (allocated on first use: make one call before capturing a CUDA graph). */
int ork_b200_i8_mm_run_out8_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, int8_t *dC, int mult, int shift);
int ork_b200_i8_mm_run_out16_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, short *dC, int mult, int shift);
int ork_b200_i8_mm_run_ewmul_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, const int8_t *dG, int8_t *dC,
                              int mult, int shift);

/* ork_i8_mm_layer over device pointers, enqueued without waiting (the first layer call on a context
 * allocates its workspace: make one before capturing a CUDA graph), with an optional decode extension:
 *   k_norm   RMSNorm gain applied to the token's k per head (Qwen3's k-norm; NULL: none);
 *   append   non-zero: the token's k (dequantized, k-normed, rotated at pos) and v are written into Kc / Vc
 *            at slot nkv of each kv head, and attention covers nkv + 1 keys (the token attends to itself);
 *   hstride  kv-head stride of the caches in tokens (their capacity; 0 = nkv, allowed only without append
 *            and dpos);
 *   dpos     non-NULL: pos and nkv are both read from this device int when the kernels run (cached tokens
 *            = position of the token), so a captured CUDA graph replays across decode steps. A position
 *            whose keys do not fit hstride skips attention and is reported as an execution error.
 * kv = NULL is ork_i8_mm_layer's behaviour. Same return codes. */
typedef struct ork_b200_layer_kv {
  const float *k_norm;
  int append;
  int hstride;
  const int *dpos;
} ork_b200_layer_kv;
int ork_b200_i8_mm_layer_async(ork_npu *ctx, const struct ork_layer_dims *d, ork_w *wq, ork_w *wk, ork_w *wv, ork_w *wo,
                          ork_w *wg, ork_w *wu, ork_w *wd, const float *attn_norm, const float *q_norm,
                          const float *ffn_norm, const float *x, float *Kc, float *Vc, float *x_out,
                          const ork_b200_layer_kv *kv);

/* Several consecutive decode layers in one call: layer l's output is layer l+1's input, x feeds the first
 * and x_out receives the last. Same dims (d) and one int8-compute weight format for all layers; kv's
 * append / hstride / dpos apply to every layer, each layer's k-norm is its own (k_norm, may be NULL; kv's
 * k_norm is not used). When the layers fit the persistent kernel the whole stack is ONE launch whose
 * weight stream runs across layer boundaries; otherwise the multi-launch form runs layer by layer. The
 * first call with a given list of layers uploads its pointer table (make it before capturing a CUDA graph).
 * Returns as ork_b200_i8_mm_layer_async. */
typedef struct ork_b200_layer_w {
  ork_w *wq, *wk, *wv, *wo, *wg, *wu, *wd;
  const float *attn_norm, *q_norm, *ffn_norm, *k_norm;
  float *Kc, *Vc;
} ork_b200_layer_w;
int ork_b200_i8_mm_layers_async(ork_npu *ctx, const struct ork_layer_dims *d, int nlayers, const ork_b200_layer_w *layers,
                           const float *x, float *x_out, const ork_b200_layer_kv *kv);

/* Decode glue around the LM head (device pointers, on the context stream; 0, or -1 on bad arguments).
 * ork_b200_rmsnorm_q8_async: RMSNorm of the row x[n] with gain g (NULL: none; eps 1e-6) and its per-tensor
 *   int8 quantization, the decode layer's formulas (ork-driver src/spine_kernels.h spine_rmsnorm +
 *   spine_quant): y = (x / sqrt(mean(x^2) + 1e-6)) * g, s = 127 / max(1e-6, max|y|), q8 = clamp(rint(y*s),
 *   +-127); *scale = s when scale is not NULL. n <= 8192.
 * ork_b200_argmax_scaled_async: the first j with the largest C[j] * bs[j] over an int32 matmul row C[n]
 *   (bs: the weight's per-channel scales), written as int64 to *idx: the greedy pick over the LM head. */
int ork_b200_rmsnorm_q8_async(ork_npu *ctx, const float *x, const float *g, int n, int8_t *q8, float *scale);
/* The same glue over a block of rows (a prefill), one launch each, device pointers, 0 or -1:
 * ork_b200_rows_q8_async: each row of x [rows][n] (n <= 8192) RMSNorm-ed with gain g when norm != 0 (g NULL:
 *   none), then quantized with its own scale: q8 [rows][n], scales[rows] (may be NULL).
 * ork_b200_rows_swiglu_q8_async: h = silu(Cg / s) * (Cu / s) per element of the gate / up results
 *   [rows][n] (int32; s = scales_in[row], the scales their input rows were quantized with), each row of h
 *   quantized: q8 [rows][n], scales[rows]. n <= 8192.
 * ork_b200_rows_dequant_async: out[m][j] = res[m][j] + C[m][j] / scales[m] * bs[j] (bs, res may be NULL;
 *   out may be res). */
int ork_b200_rows_q8_async(ork_npu *ctx, const float *x, const float *g, int rows, int n, int norm, int8_t *q8,
                           float *scales);
int ork_b200_rows_swiglu_q8_async(ork_npu *ctx, const int32_t *Cg, const int32_t *Cu, int rows, int n,
                                  const float *scales_in, int8_t *q8, float *scales);
int ork_b200_rows_dequant_async(ork_npu *ctx, const int32_t *C, int rows, int n, const float *scales, const float *bs,
                                const float *res, float *out);
/* ork_b200_rows_qk_rope_async: rows t = 0..T-1 of the q [T][H*dk], k and v [T][Hkv*dk] projections at positions
 *   pos0 + t: each q and k head RMSNorm-ed (gains q_norm / k_norm [dk], may be NULL; eps 1e-6) and rotated
 *   (RoPE NeoX at angle pos * base^(-2i/dk), ork-driver src/spine_kernels.h spine_rope_neox); q_out
 *   [H][T][dk]; k and v written into the caches Kc / Vc [Hkv][hstride][dk] at row pos0 + t
 *   (pos0 + T <= hstride). dk 64, 128 or 256. */
int ork_b200_rows_qk_rope_async(ork_npu *ctx, const float *q, const float *k, const float *v, int T, int H, int Hkv,
                                int dk, const float *q_norm, const float *k_norm, int pos0, float base, float *q_out,
                                float *Kc, float *Vc, int hstride);
int ork_b200_argmax_scaled_async(ork_npu *ctx, const int32_t *C, const float *bs, int n, long long *idx);

/* Column-sharded runs with the gather fused into the matmul (one process per GPU, NVLink peer memory).
 * Rank g of R holds output channels [col0, col0 + ncols) of a weight; its run writes those columns of C
 * into EVERY rank's C buffer ([M][ldc] int32) and signals every rank once per run; a rank that needs C
 * waits with ork_b200_peers_wait_async (bounded: an expired wait reports an error at the next sync).
 * Buffers come from ork_b200_sym_alloc (device memory + its CUDA IPC handle, ORK_B200_IPC_HANDLE_BYTES
 * bytes, exchanged by the caller over any transport) and ork_b200_sym_open (a peer's buffer mapped here).
 * flags[r] is rank r's signal block (at least 4 * R bytes of a symmetric buffer, zero at allocation).
 * A run is the local matmul plus one push kernel (its programmatic dependent) that stores the shard into
 * every rank's C and signals. ork_b200_{i8,i4}_mm_run_gather_async is a run whose push kernel also
 * waits (bounded) for every rank's signal of the run: C is complete on this rank once the stream passes
 * it, with no separate wait (one launch fewer per matmul); each run is consumed by exactly one wait,
 * its own or an ork_b200_peers_wait_async, in order. Every rank issues the same runs (same M) on a table
 * in the same order. Reuse rule: a run stores into every rank's C as soon as it starts on any rank, so
 * every rank must be done reading a table's C before any rank issues the next run on that table: e.g.
 * read C before issuing the next peer run (on any table) and alternate between at least two tables, or
 * pass a barrier after reading.
 * Returns 0 / NULL-free on success, -1 (NULL) on bad arguments or CUDA errors. No counterpart in
 * ork-driver, which gathers its cores' column slices on the host (src/npu.c:1356-1398). */
#define ORK_B200_IPC_HANDLE_BYTES 64
typedef struct ork_b200_peers ork_b200_peers;
void *ork_b200_sym_alloc(ork_npu *ctx, size_t bytes, void *handle_out);
int ork_b200_sym_free(ork_npu *ctx, void *p);
void *ork_b200_sym_open(ork_npu *ctx, const void *handle);
int ork_b200_sym_close(ork_npu *ctx, void *peer);
ork_b200_peers *ork_b200_peers_create(ork_npu *ctx, int nranks, int rank, void *const *C, void *const *flags, int ldc,
                                      int col0, int ncols);
void ork_b200_peers_destroy(ork_b200_peers *p);
int ork_b200_i8_mm_run_peers_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p);
int ork_b200_i4_mm_run_peers_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p);
int ork_b200_peers_wait_async(ork_npu *ctx, ork_b200_peers *p);
int ork_b200_i8_mm_run_gather_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p);
int ork_b200_i4_mm_run_gather_async(ork_npu *ctx, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p);
/* Landing buffers for a faster run + gather of up to `rows` rows: land[r] is rank r's symmetric buffer of
 * rows * ldc 8-byte words (zero at allocation, 16-byte aligned; every rank attaches the same set). A
 * run + gather of M <= rows then stores each value with the run's tag into every peer's landing buffer
 * (an 8-byte word: single-copy atomic) and unpacks the other ranks' tagged words into C once they carry
 * the tag -- no signal and no system-scope fence (shard widths and ldc multiples of 4; else, and for
 * larger M, the signalled push). Same reuse rule. 0, or -1 on bad arguments. */
int ork_b200_peers_land(ork_b200_peers *p, void *const *land, int rows);
/* Copy `bytes` between any two host / device addresses, ordered after the context's queued work, and wait
 * for it (for callers without a CUDA binding of their own, e.g. to read a symmetric buffer). 0 or -1. */
int ork_b200_copy(ork_npu *ctx, void *dst, const void *src, size_t bytes);

/* The load-time header check of the .orkpack loaders, callable without a device: 0 when `blob` is a
 * stamped blob of this build for (dtype, K, N), else ORK_PACKERR_SHORT / _UNSTAMPED / _FORMAT / _CAPS /
 * _SHAPE, checked in that order (ork-driver src/npu/core/packhdr.c). And the caps id this build stamps. */
int ork_b200_pack_check(const void *blob, size_t n, int dtype, int K, int N);
uint32_t ork_b200_pack_capid(void);

/* Wait for everything queued on the context's stream; 0 ok, -1 if the GPU reported an error. */
int ork_b200_sync(ork_npu *ctx);
/* The cudaStream_t the context queues on, and a way to substitute the caller's own stream (NULL restores
 * the context's private stream). The caller keeps ownership of a stream it passes in. */
void *ork_b200_stream(ork_npu *ctx);
int ork_b200_set_stream(ork_npu *ctx, void *cuda_stream);
/* CUDA device ordinal of the context. */
int ork_b200_device(const ork_npu *ctx);
/* Programmatic dependent launch for the async runs (default on): a queued matmul starts streaming its
 * weights while the previous kernel on the stream drains, and waits for that kernel before reading A. */
int ork_b200_set_pdl(ork_npu *ctx, int on);
/* Device bytes of run-time staging the context holds (host-buffer runs, grouped scales, decode-layer
 * workspace, ork_async pinned staging), all allocated on first use and grown on demand: 0 for a context
 * that has made no such call. For tests and tooling (e.g. that ork_i8_mm_run_noalloc allocated nothing). */
size_t ork_b200_staging_bytes(const ork_npu *ctx);
/* Number of kernels this context has launched (all kernels are this library's own). */
uint64_t ork_b200_launches(const ork_npu *ctx);
/* Device address and byte size of a weight's resident storage (read-only for callers). */
const void *ork_b200_weight_ptr(const ork_w *w);
/* Copy a weight's resident bytes (the K-major resident format: int8 [N][K], fp16 [N][K], or nibbles
 * [N][K/2] with the low nibble holding the even k) to host memory. Returns the bytes copied, or the
 * size needed when out is NULL, 0 on error or a short cap. For tests and tooling. */
size_t ork_b200_weight_read(const ork_w *w, void *out, size_t cap);
/* Which kernel path a run of M rows would take: 0 = CUDA-core decode GEMV, 1 = tcgen05 tensor-core
 * GEMM. Exposed for tests and benchmarks. */
int ork_b200_route(const ork_w *w, int M);
/* Force a route for subsequent runs on this context: -1 automatic (default), 0 GEMV, 1 tensor core. */
int ork_b200_force_route(ork_npu *ctx, int route);
/* The kernel choice's tuning variables (ORKB_TC_TN, _NA, _STAGES, _PAIR, _SK, ORKB_GEMV_KIND, _CPW, _TR,
 * ORKB_LAYER_FUSED) are read from the environment once per context, when it is created; this re-reads
 * them into the context (for tuning sweeps and tests that change them). 0, or -1 for a NULL context. */
int ork_b200_reload_tuning(ork_npu *ctx);
/* The tensor-core kernel's tile choice for a run of M rows on a K x N weight of format fmt (0 fp16,
 * 1 int8, 2 uniform int4 -- w4a8 uniform and W4A4 --, 3 NF4), as the router makes it (tuning variables
 * ORKB_TC_* as the environment holds them at this call): out[0] operands swapped (the weight on the 128-row MMA side),
 * out[1] tile width on the other side, out[2] K split (CTAs per cluster), out[3] stage ring depth
 * (0 = the variant's default), out[4] CTA-pair tile. Host-only: needs no device. Returns 0, or -1 on a
 * bad argument. For tests and tooling. */
int ork_b200_tc_choice(int fmt, int M, int K, int N, int *out);
/* The decode GEMV's kernel choice for a block of M <= 8 rows (format codes as above): out[0] 1 = direct-load kernel (a warp per channel group, any K), 0 = staged
 * kernel (a CTA stages whole rows in shared memory); out[1] channels per warp of the direct kernel
 * (0 for staged); out[2] channels per CTA of the staged kernel (0 for direct); out[3] activation rows
 * per pass (1, 2, 4 or 8). Tuning variables ORKB_GEMV_* as the environment holds them at this call.
 * Host-only; returns 0, or -1 on a bad argument. For tests and tooling. */
int ork_b200_gemv_choice(int fmt, int M, int K, int N, int *out);

#ifdef __cplusplus
}
#endif
#endif /* ORK_B200_H */
