// outstage.cu -- the reference's fused output stages on B200 (ork-driver include/ork/run.h:48-108,
// include/ork/sdp.h:45-52): an int8 matmul whose output is requantized to int8 / int16 (out8, out16), or
// multiplied element-wise by a second int8 tensor before the requant (ewmul: the up projection times
// silu(gate) of a SwiGLU), and the standalone int8 element-wise multiply.
//
// Arithmetic, per output element (the model the reference's own test checks its NPU against bit for
// bit, examples/test_mm_i8_out8.c:24-33): v = acc * mult (times G for ewmul) in 64-bit integers, then
// v / 2^shift rounded half to even, clamped to [-128, 127] (or [-32768, 32767]). Exact on every input.
//
// Decode-sized runs (M <= 8) requantize in the staged GEMV's store (gemv.cu store_out): the int32 sums
// never reach memory and the stage costs no launch. Larger M take the ordinary route to an int32
// scratch and one elementwise pass (requant_kernel).
//
// Validation and return codes follow the reference: -2 for a weight that is not int8-compute, K not a
// multiple of 512 or above 4096, N not a multiple of 32 (src/npu/i8/run.c:402-476 -- limits of the
// NPU's requant stage, kept so a caller sees the same refusals); for ork_i8_npu_ewmul -2 outside
// M 1..8176, N 16..8192 multiple of 16, mult 0..0x7fff, shift 0..31 (run.c:514-519). -3 (SoC without
// the fused stage) never occurs on B200. M <= 0 does nothing and returns 0, as the reference's loops.
#include <cuda_runtime.h>

#include <cstdio>

#include "ork_b200.h"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"
#include "requant.cuh"

namespace orkb {

namespace {

constexpr int kEwThreads = 256;

// 16 outputs per thread: int32 sums (and G) read as 16-byte vectors where the row allows
template <int MODE>
__global__ void __launch_bounds__(kEwThreads)
requant_kernel(const int32_t *__restrict__ C, const int8_t *__restrict__ G, size_t n, int mult, int shift,
               void *__restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (size_t i0 = ((size_t)blockIdx.x * kEwThreads + threadIdx.x) * 16; i0 < n;
       i0 += (size_t)gridDim.x * kEwThreads * 16) {
#pragma unroll 4
    for (int u = 0; u < 16; u++) {
      const size_t i = i0 + u;
      if (i >= n) break;
      int64_t v = (int64_t)C[i] * mult;
      if (MODE == OUT_EWMUL) v *= G[i];
      const int64_t q = requant_rne(v, shift);
      if (MODE == OUT_I16)
        reinterpret_cast<int16_t *>(out)[i] = (int16_t)(q > 32767 ? 32767 : q < -32768 ? -32768 : q);
      else
        reinterpret_cast<int8_t *>(out)[i] = (int8_t)(q > 127 ? 127 : q < -128 ? -128 : q);
    }
  }
}

__global__ void __launch_bounds__(kEwThreads)
ewmul_kernel(const int8_t *__restrict__ a, const int8_t *__restrict__ b, size_t n, int mult, int shift,
             int8_t *__restrict__ out) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (size_t i = (size_t)blockIdx.x * kEwThreads + threadIdx.x; i < n; i += (size_t)gridDim.x * kEwThreads) {
    const int64_t q = requant_rne((int64_t)a[i] * b[i] * mult, shift);
    out[i] = (int8_t)(q > 127 ? 127 : q < -128 ? -128 : q);
  }
}

unsigned int blocks_for(size_t n, size_t per_block) {
  const size_t b = (n + per_block - 1) / per_block;
  return (unsigned int)(b < 4096 ? (b ? b : 1) : 4096);
}

}  // namespace

cudaError_t launch_requant(const int32_t *C, size_t n, const OutStage &os, void *out, cudaStream_t s) {
  const unsigned int nb = blocks_for(n, (size_t)kEwThreads * 16);
  switch (os.mode) {
    case OUT_I8: requant_kernel<OUT_I8><<<nb, kEwThreads, 0, s>>>(C, os.G, n, os.mult, os.shift, out); break;
    case OUT_I16: requant_kernel<OUT_I16><<<nb, kEwThreads, 0, s>>>(C, os.G, n, os.mult, os.shift, out); break;
    case OUT_EWMUL: requant_kernel<OUT_EWMUL><<<nb, kEwThreads, 0, s>>>(C, os.G, n, os.mult, os.shift, out); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_ewmul_i8(const int8_t *a, const int8_t *b, size_t n, int mult, int shift, int8_t *out,
                            cudaStream_t s) {
  ewmul_kernel<<<blocks_for(n, kEwThreads), kEwThreads, 0, s>>>(a, b, n, mult, shift, out);
  return cudaGetLastError();
}

}  // namespace orkb

using namespace orkb;

namespace {

// The reference's shape and weight checks of the fused output stages (src/npu/i8/run.c:404-406).
int stage_check(const ork_w *w, int mult, int shift) {
  if (!w || w->dtype != DT_I8 || w->fmt == FMT_F16) return -2;
  if (w->K % 512 || w->K > 4096 || w->N % 32) return -2;
  if (mult < 0 || shift < 0 || shift > 62) return -2;  // negative gains / shifts have no meaning here
  return 0;
}

// Enqueue out = stage(A . W) on device pointers: the requant in the decode kernel's store for M <= 8,
// else int32 sums into the context's scratch and one elementwise pass.
int stage_enqueue(ork_npu *c, ork_w *w, int M, const int8_t *dA, const int8_t *dG, void *dOut, const OutStage &os0,
                  const char *name) {
  OutStage os = os0;
  os.G = dG;
  if (M <= 8 && batched_supports(w->fmt, M, w->K)) {
    ChainTask t{w->d, dA, dOut, M, w->K, w->N, w->N, w->fmt, os};
    int nl = 0;
    const cudaError_t e = launch_gemv_batched(&t, 1, c->stream, c->pdl, &nl);
    c->launches += (uint64_t)nl;
    if (e != cudaSuccess) {
      log_err(name, e);
      return -1;
    }
    return 0;
  }
  const size_t n = (size_t)M * w->N;
  if (!grow(&c->dC, &c->capC, n * 4)) return -1;
  if (launch(c, w, M, dA, c->dC)) return -1;
  const cudaError_t e = launch_requant((const int32_t *)c->dC, n, os, dOut, c->stream);
  c->launches += 1;
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  return 0;
}

// The synchronous form over host or device buffers.
int stage_sync(ork_npu *c, ork_w *w, int M, const int8_t *A, const int8_t *G, void *C, int mode, int mult, int shift,
               const char *name) {
  if (!c || !w || !A || !C || (mode == OUT_EWMUL && !G)) return -1;
  if (const int r = stage_check(w, mult, shift)) return r;
  if (M <= 0) return 0;
  if (async_in_flight(c, name)) return -1;
  const size_t K = w->K, N = w->N, esz = mode == OUT_I16 ? 2 : 1;
  const size_t abytes = (size_t)M * K, cbytes = (size_t)M * N * esz, gbytes = mode == OUT_EWMUL ? (size_t)M * N : 0;
  if (overlaps(A, abytes, C, cbytes) || (gbytes && overlaps(G, gbytes, C, cbytes))) {
    fprintf(stderr, "[ork] ERROR [%s]: memory overlap detected between an input and C.\n", name);
    return -1;
  }
  DeviceGuard dg(c->device);
  const bool a_dev = is_device_ptr(A, c->device) && (uintptr_t)A % 16 == 0;
  const bool g_dev = !gbytes || is_device_ptr(G, c->device);
  const bool c_dev = is_device_ptr(C, c->device) && (uintptr_t)C % esz == 0;
  const void *dA = A;
  if (!a_dev) {
    if (!grow(&c->dA, &c->capA, abytes)) return -1;
    if (cudaMemcpyAsync(c->dA, A, abytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess) return -1;
    dA = c->dA;
  }
  // G and the output are staged in the context's staging block: G first, the output 256 B further on
  const size_t goff = 0, ooff = (gbytes + 255) & ~(size_t)255;
  if ((!g_dev || !c_dev) && !grow(&c->dS, &c->capS, ooff + cbytes)) return -1;
  const int8_t *dG = G;
  if (!g_dev) {
    if (cudaMemcpyAsync((uint8_t *)c->dS + goff, G, gbytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
      return -1;
    dG = (const int8_t *)c->dS + goff;
  }
  void *dOut = c_dev ? C : (void *)((uint8_t *)c->dS + ooff);
  if (stage_enqueue(c, w, M, (const int8_t *)dA, dG, dOut, OutStage{mode, mult, shift, nullptr}, name)) return -1;
  if (!c_dev && cudaMemcpyAsync(C, dOut, cbytes, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
  const cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  if (device_error()) return -1;
  return 0;
}

int stage_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, const int8_t *dG, void *dC, int mode, int mult,
                int shift, const char *name) {
  if (!c || !w || !dA || !dC || (mode == OUT_EWMUL && !dG)) return -1;
  if (const int r = stage_check(w, mult, shift)) return r;
  if (M <= 0) return 0;
  const size_t esz = mode == OUT_I16 ? 2 : 1;
  if ((uintptr_t)dA % 16 || (uintptr_t)dC % esz) return -1;
  if (overlaps(dA, (size_t)M * w->K, dC, (size_t)M * w->N * esz)) return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, name, {dA, dG, dC})) return -1;
  return stage_enqueue(c, w, M, dA, dG, dC, OutStage{mode, mult, shift, nullptr}, name);
}

}  // namespace

extern "C" {

int ork_i8_mm_run_out8(ork_npu *c, ork_w *w, int M, const int8_t *A, int8_t *C, int mult, int shift) {
  return stage_sync(c, w, M, A, nullptr, C, OUT_I8, mult, shift, "ork_i8_mm_run_out8");
}

int ork_i8_mm_run_out16(ork_npu *c, ork_w *w, int M, const int8_t *A, short *C, int mult, int shift) {
  return stage_sync(c, w, M, A, nullptr, C, OUT_I16, mult, shift, "ork_i8_mm_run_out16");
}

int ork_i8_mm_run_ewmul(ork_npu *c, ork_w *w, int M, const int8_t *A, const int8_t *G, int8_t *C, int mult,
                        int shift) {
  return stage_sync(c, w, M, A, G, C, OUT_EWMUL, mult, shift, "ork_i8_mm_run_ewmul");
}

int ork_b200_i8_mm_run_out8_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, int8_t *dC, int mult, int shift) {
  return stage_async(c, w, M, dA, nullptr, dC, OUT_I8, mult, shift, "ork_b200_i8_mm_run_out8_async");
}

int ork_b200_i8_mm_run_out16_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, short *dC, int mult, int shift) {
  return stage_async(c, w, M, dA, nullptr, dC, OUT_I16, mult, shift, "ork_b200_i8_mm_run_out16_async");
}

int ork_b200_i8_mm_run_ewmul_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, const int8_t *dG, int8_t *dC, int mult,
                              int shift) {
  return stage_async(c, w, M, dA, dG, dC, OUT_EWMUL, mult, shift, "ork_b200_i8_mm_run_ewmul_async");
}

// out[m][n] = clamp_i8(rne(up[m][n] * silu[m][n] * mult / 2^shift)); us = the kernel's device time.
int ork_i8_npu_ewmul(ork_npu *c, const int8_t *up, const int8_t *silu, int M, int N, int mult, int shift,
                     int8_t *out, double *us) {
  if (us) *us = 0;
  if (!c || !up || !silu || !out) return -1;
  if (M < 1 || M > 8176 || N < 16 || N > 8192 || (N & 15)) return -2;  // src/npu/i8/run.c:518
  if (mult < 0 || mult > 0x7fff || shift < 0 || shift > 31) return -2;  // run.c:519
  const size_t n = (size_t)M * N, pad = (n + 255) & ~(size_t)255;
  if (overlaps(up, n, out, n) || overlaps(silu, n, out, n)) return -1;
  if (async_in_flight(c, "ork_i8_npu_ewmul")) return -1;
  DeviceGuard dg(c->device);
  const bool dev = is_device_ptr(up, c->device) && is_device_ptr(silu, c->device) && is_device_ptr(out, c->device);
  const int8_t *da = up, *db = silu;
  int8_t *dout = out;
  if (!dev) {
    if (!grow(&c->dS, &c->capS, 3 * pad)) return -1;
    int8_t *base = (int8_t *)c->dS;
    if (cudaMemcpyAsync(base, up, n, cudaMemcpyDefault, c->stream) != cudaSuccess ||
        cudaMemcpyAsync(base + pad, silu, n, cudaMemcpyDefault, c->stream) != cudaSuccess)
      return -1;
    da = base, db = base + pad, dout = base + 2 * pad;
  }
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  const bool timed = us && cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
  if (timed) cudaEventRecord(e0, c->stream);
  cudaError_t e = launch_ewmul_i8(da, db, n, mult, shift, dout, c->stream);
  c->launches += 1;
  if (timed) cudaEventRecord(e1, c->stream);
  if (e == cudaSuccess && !dev) e = cudaMemcpyAsync(out, dout, n, cudaMemcpyDefault, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (timed) {
    float ms = 0;
    if (e == cudaSuccess && cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess) *us = ms * 1e3;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  if (e != cudaSuccess) {
    log_err("ork_i8_npu_ewmul", e);
    return -1;
  }
  return 0;
}

}  // extern "C"
