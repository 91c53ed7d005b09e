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
// or two contexts on one device -- race on the array.
#define ORK_F16_AS_U16
#include <cstdio>
#include <mutex>

#include "ork_b200.h"
#include "ork_structs.h"

namespace {

constexpr size_t kScratchBytes = (size_t)4 << 20;  // activations (rounded to 256 B) + int32 results
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kScratchBytes];

std::mutex g_mu;
void *g_scratch_dev[kMaxDevices];  // device address of g_noalloc_scratch, per device

// Device address of the scratch array on `dev`, which must be the current device.
void *scratch_on(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
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

struct CurrentDevice {  // make `dev` current for the call, restore the caller's device afterwards
  int prev = -1;
  explicit CurrentDevice(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~CurrentDevice() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

}  // namespace

extern "C" int ork_i8_mm_run_noalloc(ork_npu *c, ork_w *w, int M, const int8_t *A, int32_t *C) {
  if (!c || !w || !A || !C || M < 1 || w->dtype != orkb::DT_I8) return -1;
  const size_t abytes = (size_t)M * w->K, cbytes = (size_t)M * w->N * 4;
  const uintptr_t a0 = (uintptr_t)A, c0 = (uintptr_t)C;
  if (a0 < c0 + cbytes && c0 < a0 + abytes) {
    fprintf(stderr, "[ork] ERROR [ork_i8_mm_run_noalloc]: A and C overlap\n");
    return -1;
  }
  const size_t aregion = (abytes + 255) & ~(size_t)255;
  if (aregion + cbytes > kScratchBytes) {
    fprintf(stderr,
            "[ork] ERROR ork_i8_mm_run_noalloc: M=%d K=%d N=%d needs %zu bytes of scratch "
            "(M*K rounded up to 256 + 4*M*N); the fixed scratch holds %zu\n",
            M, w->K, w->N, aregion + cbytes, kScratchBytes);
    return -1;
  }
  CurrentDevice cd(c->device);
  uint8_t *base = (uint8_t *)scratch_on(c->device);
  if (!base) return -1;
  void *dA = base, *dC = base + aregion;
  if (cudaMemcpyAsync(dA, A, abytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  const int route = orkb::route_for(c, w, M);
  if (route < 0) return -1;
  orkb::RunArgs args{w->d, dA, dC, M, w->K, w->N, w->fmt, &c->tune};
  int n = 0;
  const cudaError_t e = route == 1 ? orkb::launch_gemm_tc(args, c->stream, c->pdl, &n)
                                   : orkb::launch_gemv(args, c->stream, c->pdl, &n);
  c->launches += (uint64_t)n;
  if (e != cudaSuccess) {
    fprintf(stderr, "[ork] ERROR ork_i8_mm_run_noalloc: launch failed: %s\n", cudaGetErrorString(e));
    return -1;
  }
  if (cudaMemcpyAsync(C, dC, cbytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
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
