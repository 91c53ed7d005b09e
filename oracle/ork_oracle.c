/* ork_oracle.c -- CPU restatement of ork-driver's resident-weight matmul path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the B200 library is compared against; it is
 * never linked into, loaded by, or called from the product library (ork-driver_b200/). Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs load it.
 *
 * Every function restates one piece of the reference (paths are relative to the ork-driver project) in
 * plain scalar C. Build flags: -O2 -ffp-contract=off, so the float quantizers round exactly like the
 * reference's x86 scalar build (no FMA contraction; lrintf = round-half-even in the default FP mode).
 *
 * Parity pin: the integer GEMM reproduces the reference's own fnv64 goldens (examples/quant.c:72-81,
 * examples/test_matmul.c:84-86, :611-612, :639-641) and the quantizers/O4N1 writer are compared byte for
 * byte against the reference's compiled CPU code (oracle/_ref, built by oracle/Makefile) by
 * tests/golden/make_fixtures.py and tests/test_oracle.py.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------------------------------------------
 * Fused output stages (include/ork/run.h:48-108 ork_i8_mm_run_out8 / _out16 / _ewmul, include/ork/sdp.h:45-52
 * ork_i8_npu_ewmul). The reference's model of the NPU's requant stage, which its own test compares the
 * silicon against bit for bit (examples/test_mm_i8_out8.c:24-33 requant_i8): v = acc * mult in 64 bits,
 * q = v >> shift (arithmetic floor), +1 when the remainder exceeds half or equals half with q odd (round
 * half to even), then clamp. ewmul multiplies by the second operand before the stage; the standalone
 * element-wise multiply is the same stage on up * silu (the operands of sdp.h:45). shift 0 keeps v. */
static int64_t orc_rne_shift(int64_t v, int shift)
{
    if (shift <= 0) return v;
    const int64_t q = v >> shift, rem = v - (q << shift), half = (int64_t)1 << (shift - 1);
    return (rem > half || (rem == half && (q & 1))) ? q + 1 : q;
}

/* out[i] = clamp(rne((in[i] * (g ? g[i] : 1)) * mult / 2^shift)) for i < n; bits 8 -> int8, 16 -> int16 */
ORC_API void orc_requant(size_t n, const int32_t *in, const int8_t *g, int mult, int shift, int bits, void *out)
{
    const int64_t hi = bits == 16 ? 32767 : 127, lo = -hi - 1;
    for (size_t i = 0; i < n; i++) {
        int64_t v = (int64_t)in[i] * mult;
        if (g) v *= g[i];
        int64_t q = orc_rne_shift(v, shift);
        q = q > hi ? hi : q < lo ? lo : q;
        if (bits == 16) ((int16_t *)out)[i] = (int16_t)q;
        else ((int8_t *)out)[i] = (int8_t)q;
    }
}

/* ---------------------------------------------------------------------------------------------------
 * Grouped (per-K-group scaled) GEMM. src/npu/core/buf.c:501-520 (orki_cpu_gemm_grouped), shared by
 * ork_i4_mm_run_grouped and ork_i8_mm_run_grouped offline: Sk = K/G; for each row m the fp32 row starts
 * at 0 and, for g ascending, gains ((float)acc * aScale[m*Sk+g]) * bScale[g*N+n] where acc is the exact
 * int32 dot of A[m][gG..gG+G) with B[gG..gG+G)[n] (B row-major [K][N]). Every multiply and add is a
 * separately rounded fp32 operation (-ffp-contract=off). Returns -1 on bad arguments, as the reference. */
ORC_API int orc_gemm_grouped(int M, int K, int N, int G, const int8_t *A, const int8_t *B, const float *aScale,
                             const float *bScale, float *C)
{
    if (M < 1 || K < 1 || N < 1 || G < 1 || (K % G) || !A || !B || !aScale || !bScale || !C) return -1;
    const int Sk = K / G;
#pragma omp parallel for schedule(static) if (M > 1)
    for (int m = 0; m < M; m++) {
        float *crow = C + (size_t)m * N;
        int32_t *acc = malloc((size_t)N * sizeof *acc);
        for (int n = 0; n < N; n++) crow[n] = 0.0f;
        if (!acc) continue;
        for (int g = 0; g < Sk; g++) {
            const float as = aScale[(size_t)m * Sk + g];
            const float *bs = bScale + (size_t)g * N;
            for (int n = 0; n < N; n++) acc[n] = 0;
            for (int k = g * G; k < (g + 1) * G; k++) {
                const int32_t a = A[(size_t)m * K + k];
                if (!a) continue;
                const int8_t *brow = B + (size_t)k * N;
                for (int n = 0; n < N; n++) acc[n] += a * (int32_t)brow[n];
            }
            for (int n = 0; n < N; n++) {
                const float t = (float)acc[n] * as;
                crow[n] += t * bs[n];
            }
        }
        free(acc);
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------------------
 * Integer GEMM. src/npu/core/buf.c:428-477 (orki_cpu_gemm_i32): C[M][N] int32 = A[M][K] int8 x B[K][N]
 * int8 (B row-major), k-outer AXPY into a zeroed C row, exact int32 accumulation. Parallel over M. */
ORC_API void orc_gemm_i32(int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C)
{
#pragma omp parallel for schedule(static) if (M > 1)
    for (int m = 0; m < M; m++) {
        const int8_t *arow = A + (size_t)m * K;
        int32_t *crow = C + (size_t)m * N;
        for (int n = 0; n < N; n++) crow[n] = 0;
        for (int k = 0; k < K; k++) {
            const int32_t a = arow[k];
            if (!a) continue;
            const int8_t *brow = B + (size_t)k * N;
            for (int n = 0; n < N; n++) crow[n] += a * (int32_t)brow[n];
        }
    }
}

/* Same arithmetic with B given n-major (Bt[N][K]), which is how the quantizers emit codes. */
ORC_API void orc_gemm_i32_nk(int M, int K, int N, const int8_t *A, const int8_t *Bt, int32_t *C)
{
#pragma omp parallel for schedule(static) collapse(2) if (M * N > 64)
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            const int8_t *a = A + (size_t)m * K, *b = Bt + (size_t)n * K;
            int32_t s = 0;
            for (int k = 0; k < K; k++) s += (int32_t)a[k] * (int32_t)b[k];
            C[(size_t)m * N + n] = s;
        }
}

/* ---------------------------------------------------------------------------------------------------
 * fp16 reference. examples/test_matmul.c:37 and examples/layer.c:43: C[m][n] = sequential f32 sum over k
 * of (float)A[m][k] * (float)B[k][n]; A [M][K], B [K][N] row-major IEEE half bit patterns. */
static float orc_h2f(uint16_t h)
{
    uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1f, f = h & 0x3ff, u;
    if (e == 0) {
        if (f == 0) u = s;
        else { /* subnormal: renormalise */
            int sh = 0;
            while (!(f & 0x400)) { f <<= 1; sh++; }
            f &= 0x3ff;
            u = s | ((uint32_t)(113 - sh) << 23) | (f << 13);
        }
    } else if (e == 31) u = s | 0x7f800000u | (f << 13);
    else u = s | ((e + 112) << 23) | (f << 13);
    float r;
    memcpy(&r, &u, 4);
    return r;
}

ORC_API void orc_gemm_f16(int M, int K, int N, const uint16_t *A, const uint16_t *B, float *C)
{
    float *bt = (float *)malloc((size_t)K * N * sizeof(float));
    if (!bt) return;
    for (size_t i = 0; i < (size_t)K * N; i++) bt[i] = orc_h2f(B[i]);
#pragma omp parallel for schedule(static) if (M > 1)
    for (int m = 0; m < M; m++) {
        float *acc = C + (size_t)m * N;
        for (int n = 0; n < N; n++) acc[n] = 0.0f;
        for (int k = 0; k < K; k++) { /* k-outer keeps the per-(m,n) sum sequential in k */
            const float a = orc_h2f(A[(size_t)m * K + k]);
            const float *brow = bt + (size_t)k * N;
            for (int n = 0; n < N; n++) acc[n] += a * brow[n];
        }
    }
    free(bt);
}

/* ---------------------------------------------------------------------------------------------------
 * Per-output-channel int8 quantization of f32[N][K] (n-major).
 * src/npu.c:854-865 (orki_chan_scales_f32): mx = max(1e-9, max|w|), inv = 127/mx, bscale = mx/127;
 * src/npu/i8/pack.c:450-452 (quant32_f32_i8, scalar branch): q = lrintf(w*inv) clamped to [-127,127].
 * codes_nk is [N][K]; bscale may be NULL. */
ORC_API void orc_i8_quant_f32(int K, int N, const float *f32, int8_t *codes_nk, float *bscale)
{
    for (int n = 0; n < N; n++) {
        const float *fr = f32 + (size_t)n * K;
        float mx = 1e-9f;
        for (int k = 0; k < K; k++) { float v = fabsf(fr[k]); if (v > mx) mx = v; }
        const float inv = 127.0f / mx;
        if (bscale) bscale[n] = mx / 127.0f;
        int8_t *dst = codes_nk + (size_t)n * K;
        for (int k = 0; k < K; k++) {
            int q = (int)lrintf(fr[k] * inv);
            dst[k] = (int8_t)(q > 127 ? 127 : q < -127 ? -127 : q);
        }
    }
}

/* ---------------------------------------------------------------------------------------------------
 * int4 / NF4 quantizers. */

/* src/npu.c:888-892 (ORKI_NF4_LEVELS): the 16 normalised NF4 levels. */
static const float ORC_NF4[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

/* src/npu/i4/quant.c:26 (ORK_IM_CLIP_GRID): clip ratios tried by the imatrix scale search. */
static const float ORC_CLIP[7] = {1.0f, 0.92f, 0.85f, 0.78f, 0.70f, 0.62f, 0.55f};

/* src/npu/internal.h:589 (ork_xs32): the xorshift32 used for stochastic rounding. */
static uint32_t orc_xs32(uint32_t *s) { uint32_t x = *s; x ^= x << 13; x ^= x >> 17; x ^= x << 5; *s = x; return x; }

/* src/npu/i4/pack.c:128-131 et al.: the NF4 int8 LUT, lut[i] = (int8)lrintf(level[i]*127). */
ORC_API void orc_nf4_lut(int8_t lut[16])
{
    for (int i = 0; i < 16; i++) lut[i] = (int8_t)lrintf(ORC_NF4[i] * 127.0f);
}

/* NF4 nearest/stochastic index of one normalised weight. src/npu/i4/quant.c:73-86: clamp to [-1,1],
 * hi = first level >= wn, lo = hi-1 (or 0); ties (t >= 0.5) go to hi; SR picks hi when t > u. */
static int orc_nf4_index(float wn, int sr, uint32_t *seed)
{
    if (wn > 1.0f) wn = 1.0f; else if (wn < -1.0f) wn = -1.0f;
    int hi = 0;
    while (hi < 15 && ORC_NF4[hi] < wn) hi++;
    int lo = hi > 0 ? hi - 1 : 0;
    if (lo == hi) return hi;
    float t = (wn - ORC_NF4[lo]) / (ORC_NF4[hi] - ORC_NF4[lo]);
    if (sr) {
        float u = (float)(orc_xs32(seed) >> 8) * (1.0f / 16777216.0f);
        return (t > u) ? hi : lo;
    }
    return (t >= 0.5f) ? hi : lo;
}

/* Weighted reconstruction error of one channel at a candidate absmax. src/npu/i4/quant.c:130-151
 * (wq_err_chan): f32 sequential sum of im[k]*d*d (strict left-to-right, no contraction). */
static float orc_wq_err(const float *fr, int K, float absmax, int nf4, const float *im)
{
    float e = 0.0f;
    if (nf4) {
        float sc = absmax / 127.0f, inv = absmax > 0 ? 1.0f / absmax : 0.0f;
        for (int k = 0; k < K; k++) {
            int idx = orc_nf4_index(fr[k] * inv, 0, NULL);
            float dq = (float)((int8_t)lrintf(ORC_NF4[idx] * 127.0f)) * sc;
            float d = fr[k] - dq;
            e += (im ? im[k] : 1.0f) * d * d;
        }
    } else {
        float scale = absmax / 7.0f, inv = scale > 0 ? 1.0f / scale : 0.0f;
        for (int k = 0; k < K; k++) {
            int q = (int)lrintf(fr[k] * inv);
            if (q > 7) q = 7; else if (q < -7) q = -7;
            float dq = (float)q * scale;
            float d = fr[k] - dq;
            e += (im ? im[k] : 1.0f) * d * d;
        }
    }
    return e;
}

/* src/npu/i4/quant.c:153-161 (orki_wq_best_absmax): try each clip ratio, keep the strictly smaller error. */
static float orc_best_absmax(const float *fr, int K, float raw, int nf4, const float *im)
{
    float best_abs = raw, best_e = orc_wq_err(fr, K, raw, nf4, im);
    for (int g = 1; g < 7; g++) {
        float cand = raw * ORC_CLIP[g];
        float e = orc_wq_err(fr, K, cand, nf4, im);
        if (e < best_e) { best_e = e; best_abs = cand; }
    }
    return best_abs;
}

/* The compact O4N1 blob of ork_i4a8_mm_pack_im + ork_i4a8_w_dump, equivalently ork_i4a8_pack_cpu_blob.
 * src/npu/i4/pack.c:806-863 (ork_i4a8_pack_cpu_blob_qerr) with quant.c:28-40 (uniform) and :70-90 (NF4):
 *   header {u32 0x4F344E31, u32 version=1, i32 K, i32 N, u32 quant_kind} (src/npu/internal.h:584,597),
 *   bscale[N] f32, then Bi4[N][K/2] with the low nibble holding the even k.
 *   per channel: mx = max(1e-9, max|w|) -> optional imatrix clip search -> uniform: scale = mx/7,
 *   q = clamp(lrintf(w*(1/scale)), +-7) stored as q&0xf; NF4: bscale = mx/127, index of the nearest level.
 *   sr != 0 reproduces ORK_SR (one xorshift stream seeded 0x2545F491 for the whole call).
 * Returns the blob size (out == NULL queries the size), or 0 on bad dims / short cap. */
ORC_API size_t orc_i4a8_blob(int K, int N, const float *f32, const float *imatrix, int nf4, int sr,
                             void *out, size_t cap)
{
    if (K % 32 || N % 32 || !f32 || K <= 0 || N <= 0) return 0;
    const size_t hdr = 20, sc = (size_t)N * 4, nib = (size_t)K * N / 2, need = hdr + sc + nib;
    if (!out) return need;
    if (cap < need) return 0;
    nf4 = nf4 ? 1 : 0;
    uint32_t seed = 0x2545F491u;
    uint8_t *p = (uint8_t *)out;
    float *bscale = (float *)(p + hdr);
    uint8_t *bi4 = p + hdr + sc;
    for (int n = 0; n < N; n++) {
        const float *fr = f32 + (size_t)n * K;
        float mx = 1e-9f;
        for (int k = 0; k < K; k++) { float v = fabsf(fr[k]); if (v > mx) mx = v; }
        if (imatrix) mx = orc_best_absmax(fr, K, mx, nf4, imatrix);
        uint8_t *nb = bi4 + (size_t)n * (K / 2);
        if (nf4) {
            bscale[n] = mx / 127.0f;
            float inv = mx > 0 ? 1.0f / mx : 0.0f;
            for (int k = 0; k < K; k++) {
                uint8_t v = (uint8_t)(orc_nf4_index(fr[k] * inv, sr, &seed) & 0xf);
                if (k & 1) nb[k >> 1] |= (uint8_t)(v << 4); else nb[k >> 1] = v;
            }
        } else {
            float scale = mx / 7.0f;
            bscale[n] = scale;
            float inv = scale > 0 ? 1.0f / scale : 0.0f;
            for (int k = 0; k < K; k++) {
                int q;
                if (sr) {
                    float u = (float)(orc_xs32(&seed) >> 8) * (1.0f / 16777216.0f);
                    q = (int)floorf(fr[k] * inv + u);
                } else q = (int)lrintf(fr[k] * inv);
                if (q > 7) q = 7; else if (q < -7) q = -7;
                uint8_t v = (uint8_t)(q & 0xf);
                if (k & 1) nb[k >> 1] |= (uint8_t)(v << 4); else nb[k >> 1] = v;
            }
        }
    }
    uint32_t h[5] = {0x4F344E31u, 1u, (uint32_t)K, (uint32_t)N, (uint32_t)(nf4 ? 1 : 0)};
    memcpy(p, h, hdr);
    return need;
}

/* Decode an O4N1 blob to int8 codes exactly as the offline loader does. src/npu/i4/pack.c:115-150
 * (ork_i4a8_mm_load): exact size, magic, version 1, K, N and kind checks; uniform nibbles sign-extend,
 * NF4 nibbles map through lut[]. codes_kn is [K][N] (the reference's cpu_codes orientation). Returns 0 on
 * success, -1 on a refused blob. */
ORC_API int orc_i4a8_blob_codes(int K, int N, const void *blob, size_t n, int8_t *codes_kn, float *bscale, int *qk)
{
    if (K % 32 || N % 32 || K <= 0 || N <= 0 || !blob) return -1;
    const size_t hdr = 20, sc = (size_t)N * 4, nib = (size_t)K * N / 2;
    if (n != hdr + sc + nib) return -1;
    uint32_t h[5];
    memcpy(h, blob, hdr);
    if (h[0] != 0x4F344E31u || h[1] != 1u || (int32_t)h[2] != K || (int32_t)h[3] != N) return -1;
    if (h[4] != 0 && h[4] != 1) return -1;
    const uint8_t *p = (const uint8_t *)blob;
    if (bscale) memcpy(bscale, p + hdr, sc);
    if (qk) *qk = (int)h[4];
    int8_t lut[16];
    orc_nf4_lut(lut);
    const uint8_t *nibs = p + hdr + sc;
    for (int nn = 0; nn < N; nn++) {
        const uint8_t *nb = nibs + (size_t)nn * (K / 2);
        for (int k = 0; k < K; k++) {
            uint8_t ix = (k & 1) ? (nb[k >> 1] >> 4) : (nb[k >> 1] & 0xf);
            codes_kn[(size_t)k * N + nn] = h[4] ? lut[ix] : (int8_t)(ix >= 8 ? (int)ix - 16 : (int)ix);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------------------------------
 * Fixed-seed input generators of the reference's example tests (restated so golden checksums can be
 * reproduced on identical inputs), and the FNV-1a checksum they hash the int32 output with. */

/* examples/quant.c:18 (frand): sd = sd*1103515245 + 12345; ((int)((sd>>9)&0x3fff) - 8192)/16384.0f. */
ORC_API void orc_gen_frand(uint32_t *sd, float *out, size_t n)
{
    uint32_t s = *sd;
    for (size_t i = 0; i < n; i++) {
        s = s * 1103515245u + 12345u;
        out[i] = ((int)((s >> 9) & 0x3fff) - 8192) / 16384.0f;
    }
    *sd = s;
}

/* examples/test_matmul.c:11 (rnd): sd = sd*1103515245 + 12345; (sd>>16)%4; the int8 tests use rnd()-1. */
ORC_API void orc_gen_rnd_i8(uint32_t *sd, int8_t *out, size_t n, int offset)
{
    uint32_t s = *sd;
    for (size_t i = 0; i < n; i++) {
        s = s * 1103515245u + 12345u;
        out[i] = (int8_t)((int)((s >> 16) % 4) - offset);
    }
    *sd = s;
}

/* The same stream as IEEE half bit patterns of the small integers 0..3 (examples/test_matmul.c:23-24). */
ORC_API void orc_gen_rnd_f16(uint32_t *sd, uint16_t *out, size_t n)
{
    static const uint16_t h[4] = {0x0000, 0x3c00, 0x4000, 0x4200}; /* 0.0, 1.0, 2.0, 3.0 */
    uint32_t s = *sd;
    for (size_t i = 0; i < n; i++) {
        s = s * 1103515245u + 12345u;
        out[i] = h[(s >> 16) % 4];
    }
    *sd = s;
}

/* Advance the LCG by n steps in O(log n) (affine-map squaring). */
ORC_API uint32_t orc_lcg_skip(uint32_t sd, uint64_t n)
{
    uint32_t a = 1103515245u, c = 12345u, ra = 1u, rc = 0u;
    while (n) {
        if (n & 1) { ra = ra * a; rc = rc * a + c; }
        c = c * a + c;
        a = a * a;
        n >>= 1;
    }
    return ra * sd + rc;
}

/* FNV-1a 64 chained over a buffer (examples/quant.c:22-23, examples/test_matmul.c:15-17). */
ORC_API uint64_t orc_fnv64(uint64_t h, const void *p, size_t n)
{
    const uint8_t *b = (const uint8_t *)p;
    for (size_t i = 0; i < n; i++) { h ^= b[i]; h *= 1099511628211ULL; }
    return h;
}

ORC_API int orc_threads(void)
{
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Sets the OpenMP team size of the parallel regions the calling thread starts next, in this library and
 * in oracle/_ref (one OpenMP runtime per process): the CPU baselines use every host core even where the
 * launcher exported OMP_NUM_THREADS=1 (torchrun does). Returns the new team size. */
ORC_API int orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* ---------------------------------------------------------------------------------------------------
 * Whole decode layer. src/npu/i8/chain.c:106-122 (ork_i8_mm_layer, direct path) over the glue kernels of
 * src/spine_kernels.h:19-38, restated: RMSNorm y = x * (1/sqrtf(sum(x^2)/D + eps)) * g (sum sequential);
 * per-tensor int8 quantization s = 127 / max(1e-6, max|x|), q = clamp(lrintf(x*s), +-127), dequant int32/s;
 * RoPE NeoX on pairs (i, i+D/2), theta = pos * powf(base, -2i/D); M = 1 attention with a running max,
 * exp-sum and sequential weighted sum; SwiGLU silu(g) * u with silu(g) = g / (1 + expf(-g)). The k and v
 * projections are computed as in the reference; kv_ext (this library's decode extension) additionally
 * normalises + rotates the token's k (k_norm may be NULL), writes k and v at slot nkv of the caches
 * (head stride `hstride` tokens) and attends over nkv + 1 keys. dims = {D, H, Hkv, dk, dv, Nff, nkv, pos}.
 * Weights are int8 codes B [K][N] row-major. */
static void orc_rms(const float *x, const float *g, int n, float *y)
{
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    const float r = 1.0f / sqrtf(ss / n + 1e-6f);
    for (int i = 0; i < n; i++) y[i] = x[i] * r * g[i];
}

static float orc_q8(const float *x, int n, int8_t *q)
{
    float mx = 1e-6f;
    for (int i = 0; i < n; i++) {
        const float a = fabsf(x[i]);
        if (a > mx) mx = a;
    }
    const float s = 127.0f / mx;
    for (int i = 0; i < n; i++) {
        const int v = (int)lrintf(x[i] * s);
        q[i] = (int8_t)(v > 127 ? 127 : (v < -127 ? -127 : v));
    }
    return s;
}

/* The decode glue in front of the LM head: RMSNorm of one row (gain g, NULL = none) and its per-tensor int8
 * quantization, as orc_rms + orc_q8 (src/spine_kernels.h spine_rmsnorm + spine_quant); returns s. */
ORC_API float orc_rms_q8(const float *x, const float *g, int n, int8_t *q)
{
    float *y = malloc((size_t)n * sizeof *y), *one = NULL;
    if (!g) {
        one = malloc((size_t)n * sizeof *one);
        for (int i = 0; i < n; i++) one[i] = 1.0f;
    }
    orc_rms(x, g ? g : one, n, y);
    const float s = orc_q8(y, n, q);
    free(y);
    free(one);
    return s;
}

/* The FFN epilogue of the decode layer over one row: SwiGLU of the dequantized gate / up results
 * (g = cg / s, u = cu / s, h = g / (1 + expf(-g)) * u; src/spine_kernels.h spine_silu_glu) and the
 * per-tensor int8 quantization of h (spine_quant); returns the new scale. */
ORC_API float orc_swiglu_q8(const int32_t *cg, const int32_t *cu, int n, float s, int8_t *q)
{
    float *h = malloc((size_t)n * sizeof *h);
    for (int i = 0; i < n; i++) {
        const float gi = cg[i] / s, ui = cu[i] / s;
        h[i] = (gi / (1.0f + expf(-gi))) * ui;
    }
    const float sh = orc_q8(h, n, q);
    free(h);
    return sh;
}

static void orc_rope(float *x, int n, int pos, float base)
{
    const int h = n / 2;
    for (int i = 0; i < h; i++) {
        const float th = pos * powf(base, -2.0f * i / n), c = cosf(th), s = sinf(th);
        const float a = x[i], b = x[i + h];
        x[i] = a * c - b * s;
        x[i + h] = a * s + b * c;
    }
}

static void orc_attn1(const float *q, const float *Kh, const float *Vh, int nk, int dk, int dv, float scale, float *o)
{
    float *s = malloc((size_t)nk * sizeof *s);
    float mx = -1e30f;
    for (int j = 0; j < nk; j++) {
        float a = 0.0f;
        for (int d = 0; d < dk; d++) a += q[d] * Kh[(size_t)j * dk + d];
        s[j] = a * scale;
        if (s[j] > mx) mx = s[j];
    }
    float z = 0.0f;
    for (int j = 0; j < nk; j++) {
        s[j] = expf(s[j] - mx);
        z += s[j];
    }
    for (int d = 0; d < dv; d++) {
        float acc = 0.0f;
        for (int j = 0; j < nk; j++) acc += s[j] * Vh[(size_t)j * dv + d];
        o[d] = acc / z;
    }
    free(s);
}

static void orc_gemv1(int K, int N, const int8_t *a, const int8_t *B, int32_t *c) { orc_gemm_i32(1, K, N, a, B, c); }

ORC_API int orc_layer_i8(const uint32_t *dm, double attn_scale, double rope_base, const int8_t *Bq, const int8_t *Bk,
                         const int8_t *Bv, const int8_t *Bo, const int8_t *Bg, const int8_t *Bu, const int8_t *Bd,
                         const float *attn_norm, const float *q_norm, const float *ffn_norm, const float *x,
                         float *Kc, float *Vc, float *x_out, int kv_ext, const float *k_norm, int hstride)
{
    const int D = (int)dm[0], H = (int)dm[1], Hkv = (int)dm[2], dk = (int)dm[3], dv = (int)dm[4], F = (int)dm[5],
              nkv = (int)dm[6], pos = (int)dm[7];
    if (dk != dv || Hkv < 1 || H % Hkv) return -3;
    const int Nq = H * dk, Nk = Hkv * dk, grp = H / Hkv, hs = kv_ext ? hstride : nkv;
    int32_t *cq = malloc((size_t)Nq * 4), *ck = malloc((size_t)Nk * 4), *cv = malloc((size_t)Nk * 4),
            *co = malloc((size_t)D * 4), *cg = malloc((size_t)F * 4), *cu = malloc((size_t)F * 4),
            *cd = malloc((size_t)D * 4);
    int8_t *a8 = malloc((size_t)(Nq > F ? (Nq > D ? Nq : D) : (F > D ? F : D)));
    float *t = malloc((size_t)D * 4), *qf = malloc((size_t)Nq * 4), *ao = malloc((size_t)Nq * 4),
          *x1 = malloc((size_t)D * 4), *g = malloc((size_t)F * 4), *u = malloc((size_t)F * 4),
          *kf = malloc((size_t)dk * 4);
    int rc = -1;
    if (cq && ck && cv && co && cg && cu && cd && a8 && t && qf && ao && x1 && g && u && kf) {
        orc_rms(x, attn_norm, D, t);
        const float sx = orc_q8(t, D, a8);
        orc_gemv1(D, Nq, a8, Bq, cq);
        orc_gemv1(D, Nk, a8, Bk, ck);
        orc_gemv1(D, Nk, a8, Bv, cv);
        if (kv_ext) {  /* the token's own k (normed, rotated) and v join the caches at slot nkv */
            for (int hk = 0; hk < Hkv; hk++) {
                for (int d = 0; d < dk; d++) kf[d] = ck[hk * dk + d] / sx;
                if (k_norm) orc_rms(kf, k_norm, dk, kf);
                orc_rope(kf, dk, pos, (float)rope_base);
                for (int d = 0; d < dk; d++) {
                    Kc[((size_t)hk * hs + nkv) * dk + d] = kf[d];
                    Vc[((size_t)hk * hs + nkv) * dv + d] = cv[hk * dk + d] / sx;
                }
            }
        }
        const int nk = kv_ext ? nkv + 1 : nkv;
        for (int i = 0; i < Nq; i++) qf[i] = cq[i] / sx;
        for (int h = 0; h < H; h++) {
            float *qh = qf + (size_t)h * dk;
            orc_rms(qh, q_norm, dk, qh);
            orc_rope(qh, dk, pos, (float)rope_base);
            orc_attn1(qh, Kc + (size_t)(h / grp) * hs * dk, Vc + (size_t)(h / grp) * hs * dv, nk, dk, dv,
                      (float)attn_scale, ao + (size_t)h * dv);
        }
        const float sa = orc_q8(ao, Nq, a8);
        orc_gemv1(Nq, D, a8, Bo, co);
        for (int i = 0; i < D; i++) x1[i] = x[i] + co[i] / sa;
        orc_rms(x1, ffn_norm, D, t);
        const float sf = orc_q8(t, D, a8);
        orc_gemv1(D, F, a8, Bg, cg);
        orc_gemv1(D, F, a8, Bu, cu);
        for (int i = 0; i < F; i++) {
            const float gi = cg[i] / sf, ui = cu[i] / sf;
            g[i] = (gi / (1.0f + expf(-gi))) * ui;
        }
        const float sg = orc_q8(g, F, a8);
        orc_gemv1(F, D, a8, Bd, cd);
        for (int i = 0; i < D; i++) x_out[i] = x1[i] + cd[i] / sg;
        rc = 0;
    }
    free(cq); free(ck); free(cv); free(co); free(cg); free(cu); free(cd);
    free(a8); free(t); free(qf); free(ao); free(x1); free(g); free(u); free(kf);
    return rc;
}
