// api.cpp -- the C ABI of the B200 resident-weight matmul engine (include/ork_npu.h, include/ork_b200.h).
//
// The reference's context owns an NPU fd, DMA scratch and a worker pool (ork-driver
// src/npu/internal.h:40-144); here it owns a CUDA device ordinal, a stream, and two device staging
// buffers that host-pointer runs copy A into and C out of. A weight (src/npu/internal.h:145-159) is one
// cudaMalloc'd block in a K-major resident format plus, for int4 stores, the host copy of the
// per-channel scales that the O4N1 blob carries. Run calls validate their arguments exactly as the
// reference does (src/npu/i8/run.c:139-151, src/npu.c:1824-1832) and return 0 / -1.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

#include "ork_b200.h"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"
#include "pack.h"

using namespace orkb;

namespace orkb {

// 0 = CUDA-core GEMV, 1 = tcgen05 GEMM, -1 = no kernel for this weight / shape.
int route_for(const ork_npu *c, const ork_w *w, int M) {
  const bool tc = gemm_tc_supports(w->fmt, M, w->K, w->N), gv = gemv_supports(w->fmt, w->K);
  if (!tc && !gv) return -1;
  if (c && c->force_route == 0) return gv ? 0 : 1;
  if (c && c->force_route == 1) return tc ? 1 : 0;
  // measured crossover: the CUDA-core GEMV wins up to M = 4 everywhere and up to M = 8 on weights below
  // 4 Mi elements; the tensor-core kernel wins beyond (2048x2048 at M = 8: 2.9 us split 8 ways against
  // 3.3 us for the GEMV)
  if (M <= 4 || (M <= 8 && (size_t)w->K * w->N < ((size_t)4 << 20))) return gv ? 0 : 1;
  return tc ? 1 : 0;
}

cudaError_t smem_attr(const void *kernel, int bytes) {
  static std::mutex mu;
  static std::vector<std::pair<const void *, int>> done;  // (kernel, device) pairs already raised
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  for (auto &d : done)
    if (d.first == kernel && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.emplace_back(kernel, dev);
  return e;
}

// One error word per device in mapped, pinned host memory, set by any kernel that records an error
// (errword.cuh); the per-module device flags say which and are read (and cleared) only when it is set.
static unsigned int *g_err_host = nullptr;
static bool g_err_ready[kMaxDevices];
static std::mutex g_err_mu;

bool err_word_init(int dev) {
  if (dev < 0 || dev >= kMaxDevices) return false;
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (g_err_ready[dev]) return true;
  if (!g_err_host) {
    void *p = nullptr;
    if (cudaHostAlloc(&p, kMaxDevices * sizeof(unsigned int), cudaHostAllocPortable | cudaHostAllocMapped) !=
        cudaSuccess)
      return false;
    memset(p, 0, kMaxDevices * sizeof(unsigned int));
    g_err_host = (unsigned int *)p;
  }
  unsigned int *d = nullptr;
  if (cudaHostGetDevicePointer((void **)&d, g_err_host + dev, 0) != cudaSuccess) return false;
  cudaError_t (*set[])(unsigned int *) = {gemv_set_err_word, tc_set_err_word, layer_set_err_word,
                                          fused_set_err_word, peer_set_err_word};
  for (auto f : set)
    if (f(d) != cudaSuccess) return false;
  g_err_ready[dev] = true;
  return true;
}

// Sticky device-side errors of the current device (a bounded wait that expired, a decode position outside
// the caches): one read of the host-mapped word after a synchronisation; cleared when read.
bool device_error() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || !g_err_host) return false;
  volatile unsigned int *w = g_err_host + dev;
  if (!*w) return false;
  *w = 0u;
  tc_error_flag(true), gemv_error_flag(true), layer_error_flag(true), fused_error_flag(true), peer_error_flag(true);
  return true;
}

void log_err(const char *what, cudaError_t e) {
  fprintf(stderr, "[ork] ERROR %s: %s\n", what, cudaGetErrorString(e));
}

DeviceGuard::DeviceGuard(int dev) {
  if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
  if (prev != dev) cudaSetDevice(dev);
}
DeviceGuard::~DeviceGuard() {
  int cur = -1;
  if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
}

bool grow(void **p, size_t *cap, size_t need) {
  if (*cap >= need) return true;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  size_t sz = need < ((size_t)1 << 20) ? ((size_t)1 << 20) : need;
  if (cudaMalloc(p, sz) != cudaSuccess) {
    *p = nullptr;
    return false;
  }
  *cap = sz;
  return true;
}

bool overlaps(const void *a, size_t an, const void *b, size_t bn) {
  const uintptr_t a0 = (uintptr_t)a, a1 = a0 + an, b0 = (uintptr_t)b, b1 = b0 + bn;
  return a0 < b1 && b0 < a1;
}

// Device memory of the context's GPU (or managed memory) can be used in place.
bool is_device_ptr(const void *p, int device) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (at.type == cudaMemoryTypeManaged) return true;
  return at.type == cudaMemoryTypeDevice && at.device == device;
}

bool pinned_host_ptr(const void *p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

bool device_ptrs_ok(const ork_npu *c, const char *name, std::initializer_list<const void *> ps) {
  for (const void *p : ps)
    if (p && !is_device_ptr(p, c->device)) {
      fprintf(stderr, "[ork] ERROR %s: %p is not device memory of GPU %d (this entry point takes device pointers)\n",
              name, p, c->device);
      return false;
    }
  return true;
}

bool async_in_flight(const ork_npu *c, const char *name) {
  if (!c || !c->async_busy) return false;
  fprintf(stderr, "[ork] ERROR %s: an ork_async job is in flight on this context; ork_async_wait it first\n",
          name);
  return true;
}

static int env_int(const char *name, int unset) {
  const char *e = getenv(name);
  return e ? atoi(e) : unset;
}

Tuning tuning_from_env() {
  Tuning t;
  t.tc_tn = env_int("ORKB_TC_TN", 0);
  t.tc_na = env_int("ORKB_TC_NA", 0);
  t.tc_stages = env_int("ORKB_TC_STAGES", 0);
  t.tc_pair = env_int("ORKB_TC_PAIR", 0);
  t.tc_sk = env_int("ORKB_TC_SK", 0);
  t.tc_flags = env_int("ORKB_TC_FLAGS", 1);
  t.tc_pre = env_int("ORKB_TC_PRE", 0);
  t.pipe = env_int("ORKB_PIPE", 1);
  t.gemv_kind = env_int("ORKB_GEMV_KIND", -1);
  t.gemv_cpw = env_int("ORKB_GEMV_CPW", 0);
  t.gemv_tr = env_int("ORKB_GEMV_TR", 0);
  t.gemv_nw = env_int("ORKB_GEMV_NW", 0);
  t.layer_fused = env_int("ORKB_LAYER_FUSED", -1);
  return t;
}

ork_w *new_weight(ork_npu *c, int K, int N, int fmt, int dtype, const void *host_resident, size_t bytes) {
  if (!c) return nullptr;
  DeviceGuard dg(c->device);
  ork_w *w = new (std::nothrow) ork_w;
  if (!w) return nullptr;
  w->ctx = c;
  w->K = K;
  w->N = N;
  w->fmt = fmt;
  w->dtype = dtype;
  w->bytes = bytes;
  cudaError_t e = cudaMalloc(&w->d, bytes);
  if (e != cudaSuccess) {
    log_err("weight cudaMalloc", e);
    delete w;
    return nullptr;
  }
  e = cudaMemcpy(w->d, host_resident, bytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    log_err("weight upload", e);
    cudaFree(w->d);
    delete w;
    return nullptr;
  }
  return w;
}

// Launch one matmul on device buffers (A, C already on the context's GPU).
int launch(ork_npu *c, ork_w *w, int M, const void *dA, void *dC) { return launch_on(c, w, M, dA, dC, c->pdl); }

int launch_on(ork_npu *c, ork_w *w, int M, const void *dA, void *dC, bool pdl) {
  RunArgs a{w->d, dA, dC, M, w->K, w->N, w->fmt, &c->tune, c->tune.tc_flags ? c->dF : nullptr};
  int n = 0;
  const int route = route_for(c, w, M);
  if (route < 0) {
    fprintf(stderr, "[ork] ERROR: no kernel for this weight format at K=%d\n", w->K);
    return -1;
  }
  cudaError_t e = route == 1 ? launch_gemm_tc(a, c->stream, pdl, &n) : launch_gemv(a, c->stream, pdl, &n);
  c->launches += (uint64_t)n;
  if (e != cudaSuccess) {
    log_err("kernel launch", e);
    return -1;
  }
  return 0;
}

}  // namespace orkb

namespace {

int finish_sync(ork_npu *c, cudaStream_t s, const char *name) {
  const cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  if (device_error()) {
    fprintf(stderr, "[ork] ERROR [%s]: a kernel's bounded pipeline wait timed out; result discarded\n", name);
    return -1;
  }
  return 0;
}

// A host-buffer run large enough to pay for it, with A and C in pinned memory, goes through in row blocks
// on three streams: block i's activations upload (up), its matmul runs on the context's stream once they
// have landed, and its results read back (down) once it has finished. PCIe moves data both ways at once,
// so the upload of block i + 1 and the readback of block i overlap each other and the kernels; the call
// takes about the larger of the two transfer directions instead of their sum. Blocks hold about 1 MiB of
// results each (2 to 4 blocks, rows a multiple of 16).
constexpr size_t kPipeMinBytes = (size_t)1 << 20;

int run_pipelined(ork_npu *c, ork_w *w, int M, const void *A, void *C, size_t esz, const char *name) {
  const size_t arow = (size_t)w->K * esz, crow = (size_t)w->N * 4;
  const size_t abytes = (size_t)M * arow, cbytes = (size_t)M * crow;
  int nb = (int)((cbytes + kPipeMinBytes - 1) / kPipeMinBytes);
  // at most 4 blocks by default (ORKB_PIPE = 2..8 sets it): the configs[1] step measured 0.930 ms with 4,
  // 0.943 with 8, 0.951-0.984 in one piece -- each block is one more kernel launch
  const int nbmax = c->tune.pipe >= 2 && c->tune.pipe <= 8 ? c->tune.pipe : 4;
  nb = nb < 2 ? 2 : nb > nbmax ? nbmax : nb;
  int R = (M + nb - 1) / nb;
  R = (R + 15) & ~15;
  nb = (M + R - 1) / R;
  if (!grow(&c->dA, &c->capA, abytes) || !grow(&c->dC, &c->capC, cbytes)) return -1;
  // the staging buffers may still be read or written by work queued earlier on the context's stream
  if (cudaEventRecord(c->pev[0], c->stream) != cudaSuccess || cudaStreamWaitEvent(c->up, c->pev[0], 0) != cudaSuccess)
    return -1;
  for (int b = 0; b < nb; b++) {
    const int m0 = b * R, rows = M - m0 < R ? M - m0 : R;
    const uint8_t *ha = (const uint8_t *)A + (size_t)m0 * arow;
    uint8_t *da = (uint8_t *)c->dA + (size_t)m0 * arow, *dc = (uint8_t *)c->dC + (size_t)m0 * crow;
    cudaEvent_t landed = c->pev[1 + 2 * b], done = c->pev[2 + 2 * b];
    if (cudaMemcpyAsync(da, ha, (size_t)rows * arow, cudaMemcpyHostToDevice, c->up) != cudaSuccess ||
        cudaEventRecord(landed, c->up) != cudaSuccess || cudaStreamWaitEvent(c->stream, landed, 0) != cudaSuccess)
      return -1;
    // no programmatic overlap: each block's kernel starts after its upload, not with the previous kernel
    if (launch_on(c, w, rows, da, dc, false)) return -1;
    if (cudaEventRecord(done, c->stream) != cudaSuccess || cudaStreamWaitEvent(c->down, done, 0) != cudaSuccess ||
        cudaMemcpyAsync((uint8_t *)C + (size_t)m0 * crow, dc, (size_t)rows * crow, cudaMemcpyDeviceToHost, c->down) !=
            cudaSuccess)
      return -1;
  }
  if (finish_sync(c, c->down, name)) return -1;
  return finish_sync(c, c->stream, name);
}

// The synchronous run shared by the three public run functions.
int run_sync(ork_npu *c, ork_w *w, int M, const void *A, void *C, int want_dtype, const char *name) {
  if (!c || !w || !A || !C || M < 1) return -1;
  if (async_in_flight(c, name)) return -1;
  if (w->dtype != want_dtype) return -1;  // src/npu/i8/run.c:150, src/npu.c:1829
  const size_t esz = want_dtype == DT_F16 ? 2 : 1;
  const size_t abytes = (size_t)M * w->K * esz, cbytes = (size_t)M * w->N * 4;
  if (overlaps(A, abytes, C, cbytes)) {  // src/npu/core/submit.c:532-539
    fprintf(stderr, "[ork] ERROR [%s]: memory overlap detected! A [%p, +%zu) overlaps with C [%p, +%zu).\n",
            name, A, abytes, C, cbytes);
    return -1;
  }
  DeviceGuard dg(c->device);
  const bool a_dev = is_device_ptr(A, c->device) && ((uintptr_t)A % 16 == 0);
  const bool c_dev = is_device_ptr(C, c->device) && ((uintptr_t)C % 4 == 0);
  if (c->tune.pipe && !a_dev && !c_dev && cbytes >= kPipeMinBytes && M >= 32 && c->up && pinned_host_ptr(A) &&
      pinned_host_ptr(C))
    return run_pipelined(c, w, M, A, C, esz, name);
  const void *dA = A;
  void *dC = C;
  if (!a_dev) {
    if (!grow(&c->dA, &c->capA, abytes)) return -1;
    if (cudaMemcpyAsync(c->dA, A, abytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
    dA = c->dA;
  }
  if (!c_dev) {
    if (!grow(&c->dC, &c->capC, cbytes)) return -1;
    dC = c->dC;
  }
  if (launch(c, w, M, dA, dC)) return -1;
  if (!c_dev && cudaMemcpyAsync(C, dC, cbytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  const cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  if (device_error()) {
    fprintf(stderr, "[ork] ERROR [%s]: a kernel's bounded pipeline wait timed out; result discarded\n", name);
    return -1;
  }
  return 0;
}

int run_async(ork_npu *c, ork_w *w, int M, const void *dA, void *dC, int want_dtype, const char *name) {
  if (!c || !w || !dA || !dC || M < 1 || w->dtype != want_dtype) return -1;
  const size_t esz = want_dtype == DT_F16 ? 2 : 1;
  if (overlaps(dA, (size_t)M * w->K * esz, dC, (size_t)M * w->N * 4)) return -1;
  if ((uintptr_t)dA % 16 || (uintptr_t)dC % 16) return -1;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, name, {dA, dC})) return -1;
  return launch(c, w, M, dA, dC);
}

}  // namespace

extern "C" {

const char *ork_npu_version(void) { return ORK_NPU_VERSION "+b200"; }
uint32_t ork_pack_format_version(void) { return ORK_PACK_FORMAT_VERSION; }

ork_npu *ork_npu_init(void) {
  int dev = 0, n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
    cudaGetLastError();
    fprintf(stderr, "[ork] ERROR ork_npu_init: no CUDA device\n");
    return nullptr;
  }
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return nullptr;
  if (p.major != 10) {
    fprintf(stderr, "[ork] ERROR ork_npu_init: device %d is sm_%d%d; this build targets sm_100a (B200)\n", dev,
            p.major, p.minor);
    return nullptr;
  }
  if (!err_word_init(dev)) {
    fprintf(stderr, "[ork] ERROR ork_npu_init: cannot map the device error word\n");
    return nullptr;
  }
  ork_npu *c = new (std::nothrow) ork_npu;
  if (!c) return nullptr;
  c->device = dev;
  c->tune = tuning_from_env();
  if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete c;
    return nullptr;
  }
  c->stream = c->own_stream;
  bool aux = cudaStreamCreateWithFlags(&c->up, cudaStreamNonBlocking) == cudaSuccess &&
             cudaStreamCreateWithFlags(&c->down, cudaStreamNonBlocking) == cudaSuccess;
  for (cudaEvent_t &e : c->pev) aux = aux && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess;
  if (!aux) {  // the pipelined host-buffer path is an optimisation: without it runs go in one piece
    cudaGetLastError();
    if (c->up) cudaStreamDestroy(c->up);
    if (c->down) cudaStreamDestroy(c->down);
    for (cudaEvent_t &e : c->pev)
      if (e) cudaEventDestroy(e), e = nullptr;
    c->up = c->down = nullptr;
  }
  if (cudaMalloc(&c->dG, 16) != cudaSuccess || cudaMemset(c->dG, 0, 16) != cudaSuccess) {
    if (c->dG) cudaFree(c->dG);
    cudaStreamDestroy(c->own_stream);
    delete c;
    return nullptr;
  }
  // the split-K tile flags are an optimisation: without them split-K orders its zeroing per cluster
  const size_t fbytes = (size_t)orkb::kTcFlagTiles * 2 * sizeof(unsigned int);
  if (cudaMalloc(&c->dF, fbytes) != cudaSuccess || cudaMemset(c->dF, 0, fbytes) != cudaSuccess) {
    cudaGetLastError();
    if (c->dF) cudaFree(c->dF);
    c->dF = nullptr;
  }
  return c;
}

void ork_npu_free(ork_npu *c) {
  if (!c) return;
  {
    DeviceGuard dg(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->dA) cudaFree(c->dA);
    if (c->dC) cudaFree(c->dC);
    if (c->dS) cudaFree(c->dS);
    ring_free(c);
    layer_tabs_free(c);
    if (c->dL) cudaFree(c->dL);
    if (c->dX) cudaFree(c->dX);
    if (c->dG) cudaFree(c->dG);
    if (c->dF) cudaFree(c->dF);
    if (c->hP) cudaFreeHost(c->hP);
    if (c->async_ev) cudaEventDestroy(c->async_ev);
    if (c->up) cudaStreamDestroy(c->up);
    if (c->down) cudaStreamDestroy(c->down);
    for (cudaEvent_t e : c->pev)
      if (e) cudaEventDestroy(e);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
  }
  delete c;
}

ork_w *ork_f16_mm_pack(ork_npu *c, int K, int N, const ork_f16 *B) {
  if (!c || !B || K <= 0 || N <= 0 || K % 32 || N % 16) return nullptr;
  std::vector<uint16_t> t((size_t)K * N);
  transpose_bytes(B, t.data(), K, N, 2);
  return new_weight(c, K, N, FMT_F16, DT_F16, t.data(), t.size() * 2);
}

ork_w *ork_i8_mm_pack(ork_npu *c, int K, int N, const int8_t *B) {
  if (!c || !B || K <= 0 || N <= 0 || K % 32 || N % 32) return nullptr;
  std::vector<int8_t> t((size_t)K * N);
  transpose_bytes(B, t.data(), K, N, 1);
  return new_weight(c, K, N, FMT_I8, DT_I8, t.data(), t.size());
}

ork_w *ork_i8_mm_pack_f32(ork_npu *c, int K, int N, const float *f32, float *bscale_out) {
  if (!c || !f32 || K <= 0 || N <= 0 || K % 32 || N % 32) return nullptr;
  std::vector<int8_t> codes((size_t)K * N);
  std::vector<float> bs(N);
  quant_i8_f32(K, N, f32, codes.data(), bs.data());
  ork_w *w = new_weight(c, K, N, FMT_I8, DT_I8, codes.data(), codes.size());
  if (w && bscale_out) memcpy(bscale_out, bs.data(), (size_t)N * 4);
  return w;
}

static ork_w *i4a8_make(ork_npu *c, int K, int N, const uint8_t *nib, const float *bscale, int qk) {
  ork_w *w = new_weight(c, K, N, qk ? FMT_NF4 : FMT_U4, DT_I8, nib, (size_t)K * N / 2);
  if (!w) return nullptr;
  w->int4_store = true;
  w->quant_kind = qk;
  w->bscale = (float *)malloc((size_t)N * 4);
  if (!w->bscale) {
    ork_w_free(w);
    return nullptr;
  }
  memcpy(w->bscale, bscale, (size_t)N * 4);
  return w;
}

ork_w *ork_i4a8_mm_pack_im(ork_npu *c, int K, int N, const float *f32, const float *imatrix, float *bscale_out) {
  if (!c || !f32 || K <= 0 || N <= 0 || K % 32 || N % 32) return nullptr;
  const int sr = getenv("ORK_SR") != nullptr;   // src/npu/i4/pack.c:32
  const int nf4 = getenv("ORK_NF4") != nullptr;  // src/npu/i4/pack.c:33
  std::vector<uint8_t> nib((size_t)K * N / 2);
  std::vector<float> bs(N);
  quant_i4a8(K, N, f32, imatrix, nf4, sr, nib.data(), bs.data());
  ork_w *w = i4a8_make(c, K, N, nib.data(), bs.data(), nf4);
  if (w && bscale_out) memcpy(bscale_out, bs.data(), (size_t)N * 4);
  return w;
}

ork_w *ork_i4a8_mm_pack(ork_npu *c, int K, int N, const float *f32, float *bscale_out) {
  return ork_i4a8_mm_pack_im(c, K, N, f32, nullptr, bscale_out);
}

ork_w *ork_i4_mm_pack(ork_npu *c, int K, int N, const int8_t *B) {
  if (!c || !B || K <= 0 || N <= 0 || K % 32 || N % 64) return nullptr;
  std::vector<uint8_t> nib((size_t)K * N / 2);
  pack_w4a4(B, K, N, nib.data());
  return new_weight(c, K, N, FMT_U4, DT_I4, nib.data(), nib.size());
}

size_t ork_i4a8_w_dump(const ork_w *w, void *out, size_t cap) {
  if (!w || !w->int4_store || !w->bscale) return 0;
  const size_t need = o4n1_bytes(w->K, w->N);
  if (!out) return need;
  if (cap < need) return 0;
  uint8_t *p = (uint8_t *)out;
  o4n1_header(p, w->K, w->N, w->quant_kind);
  memcpy(p + kO4N1Header, w->bscale, (size_t)w->N * 4);
  DeviceGuard dg(w->ctx->device);
  const cudaError_t e = cudaMemcpy(p + kO4N1Header + (size_t)w->N * 4, w->d, w->bytes, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    log_err("ork_i4a8_w_dump", e);
    return 0;
  }
  return need;
}

ork_w *ork_i4a8_mm_load(ork_npu *c, int K, int N, const void *blob, size_t n) {
  int qk = -1;
  if (!c || !o4n1_check(blob, n, K, N, &qk)) return nullptr;
  const uint8_t *p = (const uint8_t *)blob;
  std::vector<float> bs(N);
  memcpy(bs.data(), p + kO4N1Header, (size_t)N * 4);
  return i4a8_make(c, K, N, p + kO4N1Header + (size_t)N * 4, bs.data(), qk);
}

size_t ork_i4a8_pack_cpu_blob_qerr(ork_npu *c, int K, int N, const float *f32, const float *imatrix, int nf4,
                                   void *out, size_t cap, float *qerr_out) {
  (void)c;
  if (K <= 0 || N <= 0 || K % 32 || N % 32 || !f32) return 0;
  const size_t need = o4n1_bytes(K, N);
  if (!out) return need;
  if (cap < need) return 0;
  nf4 = nf4 ? 1 : 0;
  const int sr = getenv("ORK_SR") != nullptr;  // src/npu/i4/pack.c:831
  uint8_t *p = (uint8_t *)out;
  float *bscale = (float *)(p + kO4N1Header);
  uint8_t *nib = p + kO4N1Header + (size_t)N * 4;
  quant_i4a8(K, N, f32, imatrix, nf4, sr, nib, bscale);
  if (qerr_out) *qerr_out = i4a8_qerr(K, N, f32, imatrix, nf4, nib, bscale);
  o4n1_header(p, K, N, nf4);
  return need;
}

size_t ork_i4a8_pack_cpu_blob(ork_npu *c, int K, int N, const float *f32, const float *imatrix, int nf4,
                              void *out, size_t cap) {
  return ork_i4a8_pack_cpu_blob_qerr(c, K, N, f32, imatrix, nf4, out, cap, nullptr);
}

void ork_w_free(ork_w *w) {
  if (!w) return;
  if (w->d) {
    DeviceGuard dg(w->ctx->device);
    cudaFree(w->d);
  }
  free(w->bscale);
  delete w;
}

void ork_mm_free(ork_npu *c, ork_w *w) {
  (void)c;
  ork_w_free(w);
}

size_t ork_w_bytes(const ork_w *w) { return w ? w->bytes : 0; }

void ork_w_dims(const ork_w *w, int *K, int *N) {
  if (K) *K = w ? w->K : 0;
  if (N) *N = w ? w->N : 0;
}

int ork_w_quant_kind(const ork_w *w) { return w ? w->quant_kind : -1; }

const float *ork_w_bscale(const ork_w *w) { return (w && w->int4_store) ? w->bscale : nullptr; }

int ork_f16_mm_run(ork_npu *c, ork_w *w, int M, const ork_f16 *A, float *C) {
  return run_sync(c, w, M, A, C, DT_F16, "ork_f16_mm_run");
}

int ork_i8_mm_run(ork_npu *c, ork_w *w, int M, const int8_t *A, int32_t *C) {
  return run_sync(c, w, M, A, C, DT_I8, "ork_i8_mm_run");
}

int ork_i4_mm_run(ork_npu *c, ork_w *w, int M, const int8_t *A, int32_t *C) {
  return run_sync(c, w, M, A, C, DT_I4, "ork_i4_mm_run");
}

// The API's explicit CPU int8 matmul (ork-driver include/ork/run.h:132): exact int32, k-outer AXPY over
// row-major B, rows spread over host threads. Not used by any GPU run path.
void ork_i8_mm_run_cpu(int M, int K, int N, const int8_t *A, const int8_t *B, int32_t *C) {
  if (M < 1 || K < 1 || N < 1 || !A || !B || !C) return;
  parallel_for(M, [&](int b, int e) {
    for (int m = b; m < e; m++) {
      int32_t *crow = C + (size_t)m * N;
      memset(crow, 0, (size_t)N * 4);
      for (int k = 0; k < K; k++) {
        const int32_t a = A[(size_t)m * K + k];
        if (!a) continue;
        const int8_t *brow = B + (size_t)k * N;
        for (int n = 0; n < N; n++) crow[n] += a * (int32_t)brow[n];
      }
    }
  });
}

// ---- ork_b200.h ----------------------------------------------------------------------------------

int ork_b200_i8_mm_run_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, int32_t *dC) {
  return run_async(c, w, M, dA, dC, DT_I8, "ork_b200_i8_mm_run_async");
}
int ork_b200_i4_mm_run_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, int32_t *dC) {
  return run_async(c, w, M, dA, dC, DT_I4, "ork_b200_i4_mm_run_async");
}
int ork_b200_f16_mm_run_async(ork_npu *c, ork_w *w, int M, const ork_f16 *dA, float *dC) {
  return run_async(c, w, M, dA, dC, DT_F16, "ork_b200_f16_mm_run_async");
}

size_t ork_b200_staging_bytes(const ork_npu *c) {
  return c ? c->capA + c->capC + c->capS + c->capL + c->capX + c->capP : 0;
}

int ork_b200_reload_tuning(ork_npu *c) {
  if (!c) return -1;
  c->tune = tuning_from_env();
  return 0;
}

int ork_b200_sync(ork_npu *c) {
  if (!c) return -1;
  DeviceGuard dg(c->device);
  const cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    log_err("ork_b200_sync", e);
    return -1;
  }
  if (device_error()) {
    fprintf(stderr, "[ork] ERROR ork_b200_sync: a kernel reported an error (a bounded wait timed out, or a decode position outside the caches)\n");
    return -1;
  }
  return 0;
}

void *ork_b200_stream(ork_npu *c) { return c ? (void *)c->stream : nullptr; }

int ork_b200_set_stream(ork_npu *c, void *s) {
  if (!c) return -1;
  c->stream = s ? (cudaStream_t)s : c->own_stream;
  return 0;
}

int ork_b200_device(const ork_npu *c) { return c ? c->device : -1; }

int ork_b200_set_pdl(ork_npu *c, int on) {
  if (!c) return -1;
  c->pdl = on != 0;
  return 0;
}

uint64_t ork_b200_launches(const ork_npu *c) { return c ? c->launches : 0; }

const void *ork_b200_weight_ptr(const ork_w *w) { return w ? w->d : nullptr; }

size_t ork_b200_weight_read(const ork_w *w, void *out, size_t cap) {
  if (!w) return 0;
  if (!out) return w->bytes;
  if (cap < w->bytes) return 0;
  DeviceGuard dg(w->ctx->device);
  if (cudaMemcpy(out, w->d, w->bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
  return w->bytes;
}

int ork_b200_route(const ork_w *w, int M) { return w ? route_for(w->ctx, w, M) : -1; }

int ork_b200_force_route(ork_npu *c, int route) {
  if (!c || route < -1 || route > 1) return -1;
  c->force_route = route;
  return 0;
}

}  // extern "C"
