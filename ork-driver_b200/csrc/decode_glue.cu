// decode_glue.cu -- the glue around int8 matmuls outside the decode layer (the LM head of a decode step, and
// the rows of a prefill), one launch each:
//   ork_b200_rmsnorm_q8_async   RMSNorm (gain g) of one row and its per-tensor int8 quantization: the
//                               formulas of glue.cuh, i.e. the decode layer's own (ork-driver's CPU glue,
//                               src/spine_kernels.h spine_rmsnorm / spine_quant), in the same order:
//                               r = 1 / sqrt(sum(x^2) / n + 1e-6), y = (x * r) * g, s = 127 / max(1e-6,
//                               max|y|), q = clamp(rint(y * s), +-127);
//   ork_b200_rows_q8_async      the same for each row of a block (per-row scales), RMSNorm optional;
//   ork_b200_rows_swiglu_q8_async  SwiGLU of dequantized gate / up rows, then per-row quantization (the
//                               decode layer's FFN epilogue: h = silu(g / s) * (u / s));
//   ork_b200_rows_dequant_async out = res + C / s[row] * bs[col] (the decode layer's x1 = x + Co / sa);
//   ork_b200_rows_qk_rope_async per row and head: q / k RMSNorm + RoPE NeoX (the decode layer's head_vec),
//                               q out head-major, k and v into the caches at the row's position;
//   ork_b200_argmax_scaled_async the greedy pick over an int32 matmul row C[n] whose weight has per-channel
//                               scales bs[n]: the first j with the largest C[j] * bs[j] (the row's positive
//                               activation factor does not move it), as int64.
// The argmax reduces (value, index) keys in one 64-bit word with atomicMax; the grid's last CTA publishes
// the index and clears the word and the count for the next call (a 16-byte scratch made with the context).
// Compiled with -fmad=false, like the decode layer.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "glue.cuh"
#include "ork_internal.h"
#include "ork_structs.h"

namespace orkb {

namespace {

constexpr int kNormThreads = 1024;
constexpr int kNormPer = 8;  // row elements per thread: rows up to 8192
constexpr int kPickThreads = 512;

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();  // red may still be read by a previous reduction
  if (lane == 0) red[w] = v;
  __syncthreads();
  return warp_sum(lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f);
}
__device__ __forceinline__ float block_max(float v, float *red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  return warp_max(lane < (int)(blockDim.x >> 5) ? red[lane] : -3.0e38f);
}

// The per-tensor quantization of one row held in registers (y[u] = element t + u * blockDim.x): s =
// 127 / max(1e-6, max|y|) (the block's maximum), q = clamp(rint(y * s), +-127).
__device__ __forceinline__ void row_q8(const float (&y)[kNormPer], int n, int8_t *q8, float *scale, float *red) {
  const int t = threadIdx.x;
  float mx = 1e-6f;
#pragma unroll
  for (int u = 0; u < kNormPer; u++)
    if (t + u * (int)blockDim.x < n) mx = fmaxf(mx, fabsf(y[u]));
  mx = block_max(mx, red);
  const float s = glue::qscale(mx);
#pragma unroll
  for (int u = 0; u < kNormPer; u++) {
    const int i = t + u * (int)blockDim.x;
    if (i < n) q8[i] = glue::q8(y[u], s);
  }
  if (t == 0 && scale) *scale = s;
}

// Row blockIdx.x of x [rows][n]: optionally RMSNorm-ed (gain g, may be NULL), then quantized.
__global__ void __launch_bounds__(kNormThreads) rows_q8_kernel(const float *__restrict__ x,
                                                               const float *__restrict__ g, int n, int norm,
                                                               int8_t *__restrict__ q8, float *__restrict__ scale) {
  __shared__ float red[32];
  const int t = threadIdx.x;
  const float *xr = x + (size_t)blockIdx.x * n;
  float v[kNormPer];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kNormPer; u++) {
    const int i = t + u * kNormThreads;
    v[u] = i < n ? xr[i] : 0.0f;
    ss += v[u] * v[u];
  }
  if (norm) {
    const float r = glue::rms_recip(block_sum(ss, red), n);
#pragma unroll
    for (int u = 0; u < kNormPer; u++) {
      const int i = t + u * kNormThreads;
      v[u] = i < n ? v[u] * r * (g ? g[i] : 1.0f) : 0.0f;
    }
  }
  row_q8(v, n, q8 + (size_t)blockIdx.x * n, scale ? scale + blockIdx.x : nullptr, red);
}

// Row blockIdx.x of the gate / up matmul results [rows][n] (int32, activation scale s[row]): SwiGLU of
// the dequantized pair, then quantized -- the decode layer's FFN epilogue.
__global__ void __launch_bounds__(kNormThreads) rows_swiglu_q8_kernel(const int32_t *__restrict__ Cg,
                                                                      const int32_t *__restrict__ Cu, int n,
                                                                      const float *__restrict__ s_in,
                                                                      int8_t *__restrict__ q8, float *__restrict__ scale) {
  __shared__ float red[32];
  const int t = threadIdx.x;
  const size_t o = (size_t)blockIdx.x * n;
  const float sa = s_in[blockIdx.x];
  float h[kNormPer];
#pragma unroll
  for (int u = 0; u < kNormPer; u++) {
    const int i = t + u * kNormThreads;
    h[u] = i < n ? glue::silu_mul(Cg[o + i] / sa, Cu[o + i] / sa) : 0.0f;
  }
  row_q8(h, n, q8 + o, scale ? scale + blockIdx.x : nullptr, red);
}

// Row t (position pos0 + t) of the q / k / v projections [T][heads * dk]: each q and k head RMSNorm-ed
// (gains qg / kg, may be NULL) and rotated (RoPE NeoX, pair (i, i + dk/2) at angle pos * base^(-2i/dk)),
// the decode layer's head_vec arithmetic; q written head-major [H][T][dk], k and v into the caches at
// [Hkv][hstride][dk] row pos0 + t. One warp per (row, head); lane l holds elements l + 32 u.
template <int PER>
__global__ void __launch_bounds__(128) rows_qk_rope_kernel(const float *__restrict__ q, const float *__restrict__ k,
                                                           const float *__restrict__ v, int T, int H, int Hkv,
                                                           const float *__restrict__ qg, const float *__restrict__ kg,
                                                           int pos0, float base, float *__restrict__ qo,
                                                           float *__restrict__ Kc, float *__restrict__ Vc,
                                                           int hstride) {
  constexpr int dk = 32 * PER;
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // (t, head) of H + Hkv heads
  if (item >= T * (H + Hkv)) return;  // whole warps
  const int t = item / (H + Hkv), hh = item % (H + Hkv);
  const bool isq = hh < H;
  const int h = isq ? hh : hh - H;
  const float *src = isq ? q + ((size_t)t * H + h) * dk : k + ((size_t)t * Hkv + h) * dk;
  const float *g = isq ? qg : kg;
  float x[PER];
#pragma unroll
  for (int u = 0; u < PER; u++) x[u] = src[lane + 32 * u];
  if (g) {
    float sq = 0.0f;
#pragma unroll
    for (int u = 0; u < PER; u++) sq += x[u] * x[u];
    const float rr = glue::rms_recip(warp_sum(sq), dk);
#pragma unroll
    for (int u = 0; u < PER; u++) x[u] = x[u] * rr * g[lane + 32 * u];
  }
  const int pos = pos0 + t;
#pragma unroll
  for (int u = 0; u < PER / 2; u++) {
    const float th = glue::rope_angle(pos, base, lane + 32 * u, dk);
    const float c = cosf(th), s = sinf(th), x0 = x[u], x1 = x[u + PER / 2];
    x[u] = x0 * c - x1 * s;
    x[u + PER / 2] = x0 * s + x1 * c;
  }
  if (isq) {
#pragma unroll
    for (int u = 0; u < PER; u++) qo[((size_t)h * T + t) * dk + lane + 32 * u] = x[u];
  } else {
    const size_t o = ((size_t)h * hstride + pos) * dk;
    const float *vs = v + ((size_t)t * Hkv + h) * dk;
#pragma unroll
    for (int u = 0; u < PER; u++) {
      Kc[o + lane + 32 * u] = x[u];
      Vc[o + lane + 32 * u] = vs[lane + 32 * u];
    }
  }
}

// out[m][j] = res[m][j] + C[m][j] / s[m] * bs[j] (res, bs optional): the dequantization (and residual)
// after a matmul of quantized rows.
__global__ void rows_dequant_kernel(const int32_t *__restrict__ C, int rows, int n, const float *__restrict__ s,
                                    const float *__restrict__ bs, const float *__restrict__ res,
                                    float *__restrict__ out) {
  const size_t total = (size_t)rows * n;
  for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
    const int m = (int)(e / n), j = (int)(e % n);
    float v = C[e] / s[m];
    if (bs) v = v * bs[j];
    out[e] = res ? res[e] + v : v;
  }
}

// float -> unsigned key with the same order (larger float, larger key)
__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(kPickThreads) argmax_scaled_kernel(const int32_t *__restrict__ C,
                                                                     const float *__restrict__ bs, int n,
                                                                     unsigned long long *best, unsigned int *count,
                                                                     long long *idx) {
  __shared__ unsigned long long red[kPickThreads / 32];
  unsigned long long k = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float v = (float)C[i] * bs[i];
    const unsigned long long key = ((unsigned long long)ordered(v) << 32) | (0xffffffffu - (uint32_t)i);
    k = key > k ? key : k;  // ties: the smaller index has the larger low word
  }
  for (int o = 16; o; o >>= 1) {
    const unsigned long long p = __shfl_xor_sync(0xffffffffu, k, o);
    k = p > k ? p : k;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = k;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kPickThreads / 32; w++) k = red[w] > k ? red[w] : k;
    atomicMax(best, k);
    __threadfence();
    if (atomicAdd(count, 1u) == gridDim.x - 1u) {  // the last CTA
      __threadfence();
      const unsigned long long b = atomicAdd(best, 0ull);  // every CTA's maximum is in
      *idx = (long long)(0xffffffffu - (uint32_t)(b & 0xffffffffull));
      *best = 0ull;
      *count = 0u;
    }
  }
}

}  // namespace

}  // namespace orkb

using namespace orkb;

extern "C" {

static int glue_launched(ork_npu *c, const char *name) {
  c->launches += 1;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  return 0;
}

int ork_b200_rmsnorm_q8_async(ork_npu *c, const float *x, const float *g, int n, int8_t *q8, float *scale) {
  return ork_b200_rows_q8_async(c, x, g, 1, n, 1, q8, scale);
}

int ork_b200_rows_q8_async(ork_npu *c, const float *x, const float *g, int rows, int n, int norm, int8_t *q8,
                           float *scales) {
  if (!c || !x || !q8 || rows < 1 || n < 1 || n > kNormThreads * kNormPer) return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, "ork_b200_rows_q8_async", {x, g, q8, scales})) return -1;
  rows_q8_kernel<<<rows, kNormThreads, 0, c->stream>>>(x, g, n, norm, q8, scales);
  return glue_launched(c, "ork_b200_rows_q8_async");
}

int ork_b200_rows_swiglu_q8_async(ork_npu *c, const int32_t *Cg, const int32_t *Cu, int rows, int n,
                                  const float *scales_in, int8_t *q8, float *scales) {
  if (!c || !Cg || !Cu || !scales_in || !q8 || rows < 1 || n < 1 || n > kNormThreads * kNormPer) return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, "ork_b200_rows_swiglu_q8_async", {Cg, Cu, scales_in, q8, scales})) return -1;
  rows_swiglu_q8_kernel<<<rows, kNormThreads, 0, c->stream>>>(Cg, Cu, n, scales_in, q8, scales);
  return glue_launched(c, "ork_b200_rows_swiglu_q8_async");
}

int ork_b200_rows_dequant_async(ork_npu *c, const int32_t *C, int rows, int n, const float *scales, const float *bs,
                                const float *res, float *out) {
  if (!c || !C || !scales || !out || rows < 1 || n < 1) return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, "ork_b200_rows_dequant_async", {C, scales, bs, res, out})) return -1;
  const size_t total = (size_t)rows * n;
  const int blocks = (int)std::min<size_t>(148 * 8, (total + 255) / 256);
  rows_dequant_kernel<<<blocks, 256, 0, c->stream>>>(C, rows, n, scales, bs, res, out);
  return glue_launched(c, "ork_b200_rows_dequant_async");
}

int ork_b200_rows_qk_rope_async(ork_npu *c, const float *q, const float *k, const float *v, int T, int H, int Hkv,
                                int dk, const float *q_norm, const float *k_norm, int pos0, float base, float *q_out,
                                float *Kc, float *Vc, int hstride) {
  if (!c || !q || !k || !v || !q_out || !Kc || !Vc || T < 1 || H < 1 || Hkv < 1 || pos0 < 0 ||
      pos0 + T > hstride)
    return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, "ork_b200_rows_qk_rope_async", {q, k, v, q_norm, k_norm, q_out, Kc, Vc})) return -1;
  const int blocks = (T * (H + Hkv) + 3) / 4;
  if (dk == 64)
    rows_qk_rope_kernel<2><<<blocks, 128, 0, c->stream>>>(q, k, v, T, H, Hkv, q_norm, k_norm, pos0, base, q_out, Kc,
                                                          Vc, hstride);
  else if (dk == 128)
    rows_qk_rope_kernel<4><<<blocks, 128, 0, c->stream>>>(q, k, v, T, H, Hkv, q_norm, k_norm, pos0, base, q_out, Kc,
                                                          Vc, hstride);
  else if (dk == 256)
    rows_qk_rope_kernel<8><<<blocks, 128, 0, c->stream>>>(q, k, v, T, H, Hkv, q_norm, k_norm, pos0, base, q_out, Kc,
                                                          Vc, hstride);
  else
    return -1;
  return glue_launched(c, "ork_b200_rows_qk_rope_async");
}

int ork_b200_argmax_scaled_async(ork_npu *c, const int32_t *C, const float *bs, int n, long long *idx) {
  if (!c || !C || !bs || !idx || n < 1 || !c->dG) return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, "ork_b200_argmax_scaled_async", {C, bs, idx})) return -1;
  unsigned long long *best = reinterpret_cast<unsigned long long *>(c->dG);
  unsigned int *count = reinterpret_cast<unsigned int *>(best + 1);
  const int blocks = (int)std::min<long long>(296, ((long long)n + kPickThreads - 1) / kPickThreads);
  argmax_scaled_kernel<<<blocks, kPickThreads, 0, c->stream>>>(C, bs, n, best, count, idx);
  return glue_launched(c, "ork_b200_argmax_scaled_async");
}

}  // extern "C"
