// ork_structs.h -- the context and weight objects behind the opaque handles of include/ork_npu.h
// (shared by the C ABI translation units; not installed).
#pragma once
#include <cuda_runtime.h>

#include <stddef.h>
#include <stdint.h>

#include <initializer_list>

#include "ork_internal.h"
#include "ork_b200.h"

struct ork_npu {
  int device = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  void *dA = nullptr;
  size_t capA = 0;
  void *dC = nullptr;
  size_t capC = 0;
  void *dS = nullptr;  // staging for the scale tables of grouped runs
  size_t capS = 0;
  void *ring = nullptr;  // in-flight slots of ork_mm_submit / ork_mm_collect (chain.cpp)
  void *dL = nullptr;    // workspace of the decode layer (layer.cu)
  size_t capL = 0;
  void *dX = nullptr;    // the residual stream between multi-launch layers (layer.cu)
  size_t capX = 0;
  void *ltabs = nullptr; // device tables of persistent-layer pointer lists (layer.cu)
  void *dG = nullptr;    // 16 bytes, zero between calls: the argmax's running key and CTA count (decode_glue.cu)
  unsigned int *dF = nullptr;  // tensor-core split-K tile flags, orkb::kTcFlagTiles x 2 words, zero between launches
  void *hP = nullptr;    // pinned host staging of the ork_async runs (A in, C out), chain.cpp
  size_t capP = 0;
  cudaEvent_t async_ev = nullptr;  // completion of the ork_async job in flight
  // pipelined host-buffer runs (api.cpp run_sync): upload and readback streams beside the context's
  // stream, and the events that chain a run's row blocks through the three
  cudaStream_t up = nullptr, down = nullptr;
  cudaEvent_t pev[1 + 2 * 8] = {};
  bool async_busy = false;         // an ork_async job is in flight (one at a time, as in the reference)
  int last_async_cpu = -1;         // sched_getcpu() of the thread that queued the latest ork_async job
  bool pdl = true;
  int force_route = -1;
  uint64_t launches = 0;
  // tuning variables of the kernel choice (ORKB_*), read once when the context is created
  orkb::Tuning tune;
};

struct ork_w {
  ork_npu *ctx = nullptr;
  int K = 0, N = 0;
  int fmt = orkb::FMT_I8;
  int dtype = orkb::DT_I8;
  int quant_kind = 0;
  bool int4_store = false;  // an ork_i4a8 weight: carries bscale and dumps as O4N1
  int gsize = 0;            // K-group size of a grouped weight (ork_i4_mm_pack_grouped, _load_tiled, set_group)
  void *d = nullptr;
  size_t bytes = 0;
  float *bscale = nullptr;
};

namespace orkb {
// 0 = CUDA-core GEMV, 1 = tcgen05 GEMM, -1 = no kernel for this weight and M.
int route_for(const ork_npu *c, const ork_w *w, int M);
// Sticky device-side error flags (a bounded wait that expired); cleared when read.
bool device_error();

void log_err(const char *what, cudaError_t e);
// Makes the context's device current for a call and restores the caller's device afterwards.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev);
  ~DeviceGuard();
};
// Grows a device staging buffer to at least `need` bytes (1 MiB minimum).
bool grow(void **p, size_t *cap, size_t need);
// Memory of the context's GPU (or managed memory) that a kernel can use in place.
bool is_device_ptr(const void *p, int device);
// The device-pointer entry points (include/ork_b200.h) launch kernels on their pointers directly: every
// non-NULL pointer in `ps` must be memory of the context's GPU (or managed memory), else a message
// naming the call and false, before anything is queued.
bool device_ptrs_ok(const ork_npu *c, const char *name, std::initializer_list<const void *> ps);
// An ork_async job (chain.cpp) owns the context's staging buffers until ork_async_wait: every other run
// on the context is refused meanwhile (message + true), the reference's one-job-in-flight contract
// (include/ork/chain.h:126-133) made a checked error.
bool async_in_flight(const ork_npu *c, const char *name);
bool overlaps(const void *a, size_t an, const void *b, size_t bn);
// Enqueues one decode layer on device pointers (layer.cu); W = {q, k, v, o, gate, up, down}.
int layer_enqueue(ork_npu *c, const struct ork_layer_dims *d, ork_w *const *W, const float *attn_norm,
                  const float *q_norm, const float *ffn_norm, const float *x, const float *Kc, const float *Vc,
                  float *x_out, const struct ork_b200_layer_kv *kv);
// Releases the ork_mm_submit ring of a context (chain.cpp).
void ring_free(ork_npu *c);
// Releases the persistent-layer tables of a context (layer.cu).
void layer_tabs_free(ork_npu *c);
// Launch one matmul on device buffers of the context's GPU (the route of route_for); 0 or -1. launch_on
// chooses programmatic dependent launch explicitly (launch: the context's setting).
int launch(ork_npu *c, ork_w *w, int M, const void *dA, void *dC);
int launch_on(ork_npu *c, ork_w *w, int M, const void *dA, void *dC, bool pdl);
// Pinned (page-locked) host memory, which copies can move asynchronously.
bool pinned_host_ptr(const void *p);
// A new resident weight: device memory of `bytes`, filled from host memory in the resident format.
ork_w *new_weight(ork_npu *c, int K, int N, int fmt, int dtype, const void *host_resident, size_t bytes);
}  // namespace orkb
