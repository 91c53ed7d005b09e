// noalloc.cu -- ork_i8_mm_run_noalloc: the synchronous int8 run for callers that cannot allocate.
//
// ork_i8_mm_run copies host activations into, and results out of, device staging buffers that the
// context allocates (cudaMalloc) on first use and grows when a larger run arrives. Some callers cannot
// let a library allocate device memory at run time: an engine that has handed nearly all of the GPU's
// memory to its own pool at start-up (a KV cache reserved up front), a process under a hard device
// memory cap, or code that must not let a run call trigger the device-wide synchronisation that
// cudaMalloc / cudaFree can cause. This entry point runs the same kernels through a fixed scratch area
// that is part of the library image instead: a file-scope __device__ array of kScratchBytes, present on
// every GPU that loads the library until the process exits. It calls no allocating routine.
//
// Set-up: on its first call on a device (that device current) the entry point looks up the array's
// device address with cudaGetSymbolAddress -- the array's name is only a host-side stand-in, not a
// device pointer -- and reuses it for that device afterwards. Make that first call before any stream
// capture. Every call shares the one array and leaves its contents behind; nothing in it needs to start
// at zero (the kernels write every output element). Calls that overlap on the GPU -- from two threads,
// or two contexts on one device -- race on the array, so calls on one device must be serialised.
// Device-resident A and C (memory of the context's GPU) are used in place, as by ork_i8_mm_run; only
// host buffers go through the array.
#define ORK_F16_AS_U16
#include <cstdio>
#include <mutex>

#include "ork_b200.h"
#include "ork_structs.h"

namespace {

constexpr size_t kScratchBytes = (size_t)4 << 20;  // staged activations (rounded to 256 B) + int32 results

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_dev[orkb::kMaxDevices];  // device address of g_noalloc_scratch, per device

// Device address of the scratch array on `dev`, which must be the current device.
void *scratch_on(int dev) {
  if (dev < 0 || dev >= orkb::kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch_dev[dev]) {
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      fprintf(stderr, "[ork] ERROR ork_i8_mm_run_noalloc: scratch address lookup failed: %s\n",
              cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_dev[dev] = p;
  }
  return g_scratch_dev[dev];
}

}  // namespace

extern "C" int ork_i8_mm_run_noalloc(ork_npu *c, ork_w *w, int M, const int8_t *A, int32_t *C) {
  if (!c || !w || !A || !C || M < 1 || w->dtype != orkb::DT_I8) return -1;
  const size_t abytes = (size_t)M * w->K, cbytes = (size_t)M * w->N * 4;
  if (orkb::overlaps(A, abytes, C, cbytes)) {
    fprintf(stderr, "[ork] ERROR [ork_i8_mm_run_noalloc]: A and C overlap\n");
    return -1;
  }
  if (orkb::async_in_flight(c, "ork_i8_mm_run_noalloc")) return -1;
  orkb::DeviceGuard dg(c->device);
  // as in ork_i8_mm_run: device memory of the context's GPU is used in place; only host buffers are
  // staged, and only they count against the scratch
  const bool a_dev = orkb::is_device_ptr(A, c->device) && (uintptr_t)A % 16 == 0;
  const bool c_dev = orkb::is_device_ptr(C, c->device) && (uintptr_t)C % 4 == 0;
  const size_t aregion = a_dev ? 0 : (abytes + 255) & ~(size_t)255, cregion = c_dev ? 0 : cbytes;
  if (aregion + cregion > kScratchBytes) {
    fprintf(stderr,
            "[ork] ERROR ork_i8_mm_run_noalloc: M=%d K=%d N=%d needs %zu bytes of scratch for its host "
            "buffers (M*K rounded up to 256 for A, 4*M*N for C); the fixed scratch holds %zu\n",
            M, w->K, w->N, aregion + cregion, kScratchBytes);
    return -1;
  }
  uint8_t *base = nullptr;
  if (aregion + cregion) {
    base = (uint8_t *)scratch_on(c->device);
    if (!base) return -1;
  }
  const void *dA = a_dev ? (const void *)A : (const void *)base;
  void *dC = c_dev ? (void *)C : (void *)(base + aregion);
  if (!a_dev && cudaMemcpyAsync((void *)dA, A, abytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  const int route = orkb::route_for(c, w, M);
  if (route < 0) return -1;
  orkb::RunArgs args{w->d, dA, dC, M, w->K, w->N, w->fmt, &c->tune, c->tune.tc_flags ? c->dF : nullptr};
  int n = 0;
  const cudaError_t e = route == 1 ? orkb::launch_gemm_tc(args, c->stream, c->pdl, &n)
                                   : orkb::launch_gemv(args, c->stream, c->pdl, &n);
  c->launches += (uint64_t)n;
  if (e != cudaSuccess) {
    fprintf(stderr, "[ork] ERROR ork_i8_mm_run_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return -1;
  }
  if (!c_dev && cudaMemcpyAsync(C, dC, cbytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  const cudaError_t s = cudaStreamSynchronize(c->stream);
  if (s != cudaSuccess) {
    fprintf(stderr, "[ork] ERROR ork_i8_mm_run_noalloc: %s\n", cudaGetErrorString(s));
    return -1;
  }
  if (orkb::device_error()) {
    fprintf(stderr, "[ork] ERROR ork_i8_mm_run_noalloc: a kernel's bounded pipeline wait timed out\n");
    return -1;
  }
  return 0;
}
