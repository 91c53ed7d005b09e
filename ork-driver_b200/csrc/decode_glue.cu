// decode_glue.cu -- the decode step's glue around the LM head, as one launch each:
//   ork_b200_rmsnorm_q8_async   RMSNorm (gain g) of one row and its per-tensor int8 quantization: the
//                               formulas of glue.cuh, i.e. the decode layer's own (ork-driver's CPU glue,
//                               src/spine_kernels.h spine_rmsnorm / spine_quant), in the same order:
//                               r = 1 / sqrt(sum(x^2) / n + 1e-6), y = (x * r) * g, s = 127 / max(1e-6,
//                               max|y|), q = clamp(rint(y * s), +-127);
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

__global__ void __launch_bounds__(kNormThreads) rmsnorm_q8_kernel(const float *__restrict__ x,
                                                                  const float *__restrict__ g, int n,
                                                                  int8_t *__restrict__ q8, float *__restrict__ scale) {
  __shared__ float red[32];
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  float v[kNormPer], gg[kNormPer];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kNormPer; u++) {
    const int i = t + u * kNormThreads;
    v[u] = i < n ? x[i] : 0.0f;
    gg[u] = i < n ? (g ? g[i] : 1.0f) : 0.0f;
  }
#pragma unroll
  for (int u = 0; u < kNormPer; u++) ss += v[u] * v[u];
  ss = warp_sum(ss);
  if (lane == 0) red[w] = ss;
  __syncthreads();
  ss = warp_sum(lane < kNormThreads / 32 ? red[lane] : 0.0f);
  const float r = glue::rms_recip(ss, n);
  float mx = 1e-6f;
#pragma unroll
  for (int u = 0; u < kNormPer; u++)
    if (t + u * kNormThreads < n) mx = fmaxf(mx, fabsf(v[u] * r * gg[u]));
  mx = warp_max(mx);
  __syncthreads();  // red is reused
  if (lane == 0) red[w] = mx;
  __syncthreads();
  mx = warp_max(lane < kNormThreads / 32 ? red[lane] : -3.0e38f);
  const float s = glue::qscale(mx);
#pragma unroll
  for (int u = 0; u < kNormPer; u++) {
    const int i = t + u * kNormThreads;
    if (i < n) q8[i] = glue::q8(v[u] * r * gg[u], s);
  }
  if (t == 0 && scale) *scale = s;
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

int ork_b200_rmsnorm_q8_async(ork_npu *c, const float *x, const float *g, int n, int8_t *q8, float *scale) {
  if (!c || !x || !q8 || n < 1 || n > kNormThreads * kNormPer) return -1;
  DeviceGuard dg(c->device);
  rmsnorm_q8_kernel<<<1, kNormThreads, 0, c->stream>>>(x, g, n, q8, scale);
  c->launches += 1;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    log_err("ork_b200_rmsnorm_q8_async", e);
    return -1;
  }
  return 0;
}

int ork_b200_argmax_scaled_async(ork_npu *c, const int32_t *C, const float *bs, int n, long long *idx) {
  if (!c || !C || !bs || !idx || n < 1 || !c->dG) return -1;
  DeviceGuard dg(c->device);
  unsigned long long *best = reinterpret_cast<unsigned long long *>(c->dG);
  unsigned int *count = reinterpret_cast<unsigned int *>(best + 1);
  const int blocks = (int)std::min<long long>(296, ((long long)n + kPickThreads - 1) / kPickThreads);
  argmax_scaled_kernel<<<blocks, kPickThreads, 0, c->stream>>>(C, bs, n, best, count, idx);
  c->launches += 1;
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    log_err("ork_b200_argmax_scaled_async", e);
    return -1;
  }
  return 0;
}

}  // extern "C"
