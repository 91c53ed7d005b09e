/* ref_layer.c -- test infrastructure only (built into oracle/_ref/libork_ref.so by `make -C oracle ref`).
 *
 * Runs the arithmetic of ork-driver's whole-decode-layer entry point, ork_i8_mm_layer's direct path
 * (src/npu/i8/chain.c:106-122), on the host: the reference's own glue kernels (src/spine_kernels.h, compiled
 * from where they lie) around its exact int32 GEMM (orki_cpu_gemm_i32, src/npu/core/buf.c:428), in the
 * reference's order. chain.c itself does not build on x86 (NEON), so this shim is the compiled reference
 * that the restated layer in ork_oracle.c is checked against. Weights are raw int8 codes B [K][N].
 */
#include <stdint.h>
#include <stdlib.h>

#include "spine_kernels.h"

void orki_cpu_gemm_i32(int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C);

__attribute__((visibility("default"))) int ref_layer_i8(const uint32_t *dm, double attn_scale, double rope_base,
                                                        const int8_t *Bq, const int8_t *Bk, const int8_t *Bv,
                                                        const int8_t *Bo, const int8_t *Bg, const int8_t *Bu,
                                                        const int8_t *Bd, const float *attn_norm, const float *q_norm,
                                                        const float *ffn_norm, const float *x, const float *Kc,
                                                        const float *Vc, float *x_out)
{
    int D = (int)dm[0], H = (int)dm[1], Hkv = (int)dm[2], dk = (int)dm[3], dv = (int)dm[4], Nff = (int)dm[5],
        nkv = (int)dm[6], pos = (int)dm[7];
    int Nq = H * dk, Nkv = Hkv * dk, rk2 = (Hkv > 0) ? H / Hkv : 1;
    int32_t *Cq = malloc((size_t)Nq * 4), *Ck = malloc((size_t)Nkv * 4), *Cv = malloc((size_t)Nkv * 4),
            *Co = malloc((size_t)D * 4), *Cg = malloc((size_t)Nff * 4), *Cu = malloc((size_t)Nff * 4),
            *Cd = malloc((size_t)D * 4);
    int8_t *xn8 = malloc(D), *ao8 = malloc(Nq), *xf8 = malloc(D), *ac8 = malloc(Nff);
    float *xo = malloc((size_t)D * 4), *qf = malloc((size_t)Nq * 4), *ao = malloc((size_t)Nq * 4),
          *x1 = malloc((size_t)D * 4), *xf = malloc((size_t)D * 4), *gf = malloc((size_t)Nff * 4),
          *uf = malloc((size_t)Nff * 4), *act = malloc((size_t)Nff * 4);
    int rc = -1;
    if (Cq && Ck && Cv && Co && Cg && Cu && Cd && xn8 && ao8 && xf8 && ac8 && xo && qf && ao && x1 && xf && gf && uf &&
        act) {
        float sx = (spine_rmsnorm(x, attn_norm, D, 1e-6f, xo), spine_quant(xo, D, xn8));
        orki_cpu_gemm_i32(1, D, Nq, xn8, Bq, Cq);
        orki_cpu_gemm_i32(1, D, Nkv, xn8, Bk, Ck);
        orki_cpu_gemm_i32(1, D, Nkv, xn8, Bv, Cv);
        for (int i = 0; i < Nq; i++) qf[i] = Cq[i] / sx;
        for (int h = 0; h < H; h++) {
            float *qh = qf + (size_t)h * dk;
            spine_rmsnorm(qh, q_norm, dk, 1e-6f, qh);
            spine_rope_neox(qh, dk, pos, (float)rope_base);
            spine_attn(qh, Kc + (size_t)(h / rk2) * nkv * dk, Vc + (size_t)(h / rk2) * nkv * dv, nkv, dk, dv,
                       (float)attn_scale, ao + (size_t)h * dv);
        }
        float sa = spine_quant(ao, Nq, ao8);
        orki_cpu_gemm_i32(1, Nq, D, ao8, Bo, Co);
        for (int i = 0; i < D; i++) x1[i] = x[i] + Co[i] / sa;
        float sf = (spine_rmsnorm(x1, ffn_norm, D, 1e-6f, xf), spine_quant(xf, D, xf8));
        orki_cpu_gemm_i32(1, D, Nff, xf8, Bg, Cg);
        orki_cpu_gemm_i32(1, D, Nff, xf8, Bu, Cu);
        for (int i = 0; i < Nff; i++) {
            gf[i] = Cg[i] / sf;
            uf[i] = Cu[i] / sf;
        }
        spine_silu_glu(gf, uf, Nff, act);
        float sac = spine_quant(act, Nff, ac8);
        orki_cpu_gemm_i32(1, Nff, D, ac8, Bd, Cd);
        for (int i = 0; i < D; i++) x_out[i] = x1[i] + Cd[i] / sac;
        rc = 0;
    }
    free(Cq); free(Ck); free(Cv); free(Co); free(Cg); free(Cu); free(Cd);
    free(xn8); free(ao8); free(xf8); free(ac8);
    free(xo); free(qf); free(ao); free(x1); free(xf); free(gf); free(uf); free(act);
    return rc;
}
