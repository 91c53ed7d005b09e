// peers.cu -- column-sharded matmuls with the output gather over NVLink peer memory (one process per
// GPU), no collective library on the data path.
//
// A weight split by output channels over R ranks (each channel has its own scale and codes, ork-driver
// src/npu/i4/pack.c:63-80; the reference splits the same way over its NPU cores, src/npu.c:1356-1398)
// leaves rank g with C[:, g's columns]; every rank needs all of C. A run is the local matmul into a
// scratch C at full speed, then a push kernel, launched as its programmatic dependent (it is resident
// while the matmul drains) with a grid sized from the shard's bytes, that copies the shard's rows into
// every rank's C with 16-byte stores; each push CTA counts itself done on this GPU (acq_rel) and the
// last one signals every rank once: one system-scope fence, then a relaxed add per rank (release.gpu ->
// acquire.gpu -> fence.acq_rel.sys orders every CTA's peer stores before the signals). A rank that needs
// C waits (on its stream, bounded) until every rank's count of signals reaches the runs it has consumed
// plus one.
// (Storing into the peers from the matmul's own epilogue was measured 1.6x slower at M = 1: each of the
// thousands of short matmul CTAs then waits for its NVLink stores to be acknowledged before it can
// release; a few large push CTAs pay that latency once, in parallel.)
// Buffers: symmetric allocations of this library (ork_b200_sym_alloc) exchanged as CUDA IPC handles by
// the caller (64 bytes each, any transport) and mapped with ork_b200_sym_open. No TMA and no multicast:
// plain stores and atomics over NVLink.
//
// Reuse rule: a run stores into every rank's C as soon as it starts on any rank, so before a rank
// issues a run on a table every rank must be done reading that table's C. It holds when each rank reads
// C before it issues its next peer run (on any table) and consecutive runs alternate between at least
// two tables: a rank reuses table T only after waiting on another table's run, which needed every
// peer's signal of that later run, sent after the peer had read T; or when all ranks pass a barrier
// after reading.
// (Every push CTA signalling on its own, with its own system-scope fence and no last-CTA election, was
// measured slower: 21.8 against 20.8 us per M = 1 matmul on two GPUs, 33.6 against 29.8 at M = 8 -- the
// concurrent fences took longer than one fence after the device-scope count.)
#include <cuda_runtime.h>

#include <cstdio>
#include <algorithm>
#include <cstring>
#include <new>

#include "ork_b200.h"
#include "errword.cuh"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"

struct ork_b200_peers {
  ork_npu *ctx = nullptr;
  orkb::PeerTable host{};             // the table's contents (host copy)
  orkb::PeerTable *dev = nullptr;     // the table in device memory (read by the kernels)
  unsigned int *waited = nullptr;     // private device counter
};

namespace orkb {

namespace {

__device__ unsigned int g_peer_error = 0;
constexpr uint64_t kPeerSpin = 4000000000ull;  // ~2 s of SM clock

constexpr int kPushVecs = 256;      // 16-byte vectors (or elements) per push CTA when sizing the grid
constexpr size_t kPushMax = 148 * 8;  // at most eight resident 256-thread CTAs per SM; larger shards grid-stride

// Bounded wait until every rank's count of signals to this rank reaches `target` (lane r watches rank
// r); false when the wait expired (the error flag is then set).
__device__ __forceinline__ bool wait_signals(const PeerTable *__restrict__ pt, int r, unsigned int target) {
  if (r >= pt->n) return true;
  const unsigned int *f = pt->flag[pt->rank] + r;
  const uint64_t t0 = clock64();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if ((int)(v - target) >= 0) return true;
    if (clock64() - t0 > kPeerSpin) {
      { atomicOr(&g_peer_error, 1u); err_word_set(); }
      return false;
    }
    __nanosleep(64);
  }
}

// Copies the local C [M][n] (row stride n) into every rank's C at the shard's offset, grid-striding over
// 16-byte vectors when the row layout allows, then counts the CTA done on this GPU; the run's last push
// CTA (of gridDim.x) signals every rank. The grid is sized per run from M * n. With WAIT, that last CTA
// then also waits (bounded) for every rank's signal of this run and counts the run consumed, so C is
// complete on this rank when the kernel is: the gather costs one launch instead of two.
// The dependent launch (the wait kernel, or the next matmul, which streams its weights before its own
// dependency wait) is released at once; it still reads nothing of this run before the kernel completes.
template <bool WAIT>
__global__ void __launch_bounds__(256) push_kernel(const int32_t *__restrict__ C, int M, int n,
                                                    const PeerTable *__restrict__ pt) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the matmul is complete
  const bool vec = (n % 4 == 0) && (pt->ldc % 4 == 0) && (pt->col0 % 4 == 0);
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  if (vec) {
    const int nv = n / 4;
    const size_t total = (size_t)M * nv;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
      const int m = (int)(e / nv), c = (int)(e % nv) * 4;
      const int4 v = *reinterpret_cast<const int4 *>(C + (size_t)m * n + c);
      const size_t o = (size_t)m * pt->ldc + pt->col0 + c;
      for (int r = 0; r < pt->n; r++) *reinterpret_cast<int4 *>(pt->C[r] + o) = v;
    }
  } else {
    const size_t total = (size_t)M * n;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
      const int m = (int)(e / n), c = (int)(e % n);
      const int32_t v = C[(size_t)m * n + c];
      const size_t o = (size_t)m * pt->ldc + pt->col0 + c;
      for (int r = 0; r < pt->n; r++) pt->C[r][o] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(pt->done) : "memory");
    if (old == gridDim.x - 1u) {
      *pt->done = 0u;
      // one system-scope fence, then relaxed adds (a release pattern for every one of them): a release
      // add per rank would fence once per rank (measured ~1.7 us each on two GPUs, the largest part of the
      // gather)
      asm volatile("fence.acq_rel.sys;" ::: "memory");
      for (int r = 0; r < pt->n; r++)
        asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(pt->flag[r] + pt->rank) : "memory");
      if (WAIT) {
        // the count of consumed runs was last advanced by a wait that completed before this run's
        // matmul started (stream order)
        const unsigned int target = *pt->waited + 1u;
        for (int r = 0; r < pt->n; r++)
          if (!wait_signals(pt, r, target)) break;
        *pt->waited = target;
      }
    }
  }
}

// Tagged-word gather of one run (no signal, no system-scope fence). Every value travels as one 8-byte
// word (value, run tag), which a rank stores into every peer's landing buffer; an aligned 8-byte store is
// single-copy atomic, so a reader that sees the tag sees the value. This rank's own columns go straight
// into its C. Then the grid polls (bounded) the landing words of the other ranks' columns until they carry
// the tag and writes them into C. The tag is this rank's count of tagged runs plus one (read by every
// CTA after the dependency wait; the run's last CTA advances the count). Grid-strides over 16-byte
// vectors of the shard (push) and of C (unpack); its size is capped at what is resident at once, so no
// CTA waits for a peer's data while a CTA that has not started holds back this rank's own push.
__global__ void __launch_bounds__(256) gather_tag_kernel(const int32_t *__restrict__ Cl, int M, int n,
                                                          const PeerTable *__restrict__ pt) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");  // the matmul is complete
  const uint32_t tag = *pt->runs + 1u;
  const int ldc = pt->ldc, col0 = pt->col0, nv = n / 4, lv = ldc / 4, me = pt->rank;
  const size_t stride = (size_t)gridDim.x * blockDim.x, first = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  int32_t *C = pt->C[me];
  const uint64_t hi = (uint64_t)tag << 32;
  for (size_t e = first; e < (size_t)M * nv; e += stride) {
    const int m = (int)(e / nv), c = (int)(e % nv) * 4;
    const int4 v = *reinterpret_cast<const int4 *>(Cl + (size_t)m * n + c);
    const size_t o = (size_t)m * ldc + col0 + c;
    *reinterpret_cast<int4 *>(C + o) = v;
    const uint64_t w0 = hi | (uint32_t)v.x, w1 = hi | (uint32_t)v.y, w2 = hi | (uint32_t)v.z, w3 = hi | (uint32_t)v.w;
    for (int r = 0; r < pt->n; r++) {
      if (r == me) continue;
      uint64_t *L = pt->land[r] + o;
      asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(L), "l"(w0), "l"(w1) : "memory");
      asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(L + 2), "l"(w2), "l"(w3) : "memory");
    }
  }
  bool ok = true;
  const uint64_t *L = pt->land[me];
  for (size_t e = first; e < (size_t)M * lv && ok; e += stride) {
    const int m = (int)(e / lv), c = (int)(e % lv) * 4;
    if (c >= col0 && c < col0 + n) continue;  // this rank's own columns
    const size_t o = (size_t)m * ldc + c;
    uint64_t w[4];
    const uint64_t t0 = clock64();
    while (true) {
      asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w[0]), "=l"(w[1]) : "l"(L + o) : "memory");
      asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w[2]), "=l"(w[3]) : "l"(L + o + 2) : "memory");
      if ((uint32_t)(w[0] >> 32) == tag && (uint32_t)(w[1] >> 32) == tag && (uint32_t)(w[2] >> 32) == tag &&
          (uint32_t)(w[3] >> 32) == tag)
        break;
      if (clock64() - t0 > kPeerSpin) {
        { atomicOr(&g_peer_error, 1u); err_word_set(); }
        ok = false;
        break;
      }
    }
    *reinterpret_cast<int4 *>(C + o) = make_int4((int)(uint32_t)w[0], (int)(uint32_t)w[1], (int)(uint32_t)w[2],
                                                  (int)(uint32_t)w[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(old) : "l"(pt->ldone) : "memory");
    if (old == gridDim.x - 1u) {  // every CTA has read the tag: advance it for the next run
      *pt->ldone = 0u;
      *pt->runs = tag;
    }
  }
}

// One warp: lane r waits until rank r's count of signals here covers one more run than this rank has
// consumed (each run signals each rank once); bounded (an expired wait sets the error flag and lets the
// stream go on).
// Launched as a programmatic dependent of the run and releasing its own dependent at once: the next
// matmul streams its weights while this waits, and reads its activations only after this completes.
// The count of consumed runs is read only after the run before it on the stream is complete (so after
// the previous wait on the same table has counted itself).
__global__ void __launch_bounds__(32) wait_kernel(const PeerTable *__restrict__ pt) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const unsigned int target = *pt->waited + 1u;  // one signal per rank per run
  wait_signals(pt, threadIdx.x, target);
  __syncwarp();
  if (threadIdx.x == 0) *pt->waited = target;
}

}  // namespace

unsigned int peer_error_flag(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_peer_error, sizeof v);
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_peer_error, &z, sizeof z);
  }
  return v;
}

ORKB_ERR_WORD_SETTER(peer_set_err_word)

}  // namespace orkb

using namespace orkb;

namespace {

int peers_run(ork_npu *c, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p, int dtype, bool wait,
              const char *name) {
  if (!c || !w || !dA || !p || p->ctx != c || M < 1 || w->dtype != dtype || w->fmt == FMT_F16) return -1;
  const PeerTable &t = p->host;
  if (w->N + t.col0 > t.ldc || w->N != t.ctas) return -1;  // the table's shard width
  DeviceGuard dg(c->device);
  if ((uintptr_t)dA % 16 || !device_ptrs_ok(c, name, {dA})) return -1;
  if (!grow(&c->dC, &c->capC, (size_t)M * w->N * 4)) return -1;
  if (launch(c, w, M, dA, c->dC)) return -1;
  cudaLaunchConfig_t cfg = {};
  const size_t units = (size_t)M * (w->N % 4 == 0 ? w->N / 4 : w->N);
  cfg.gridDim = dim3((unsigned int)std::min<size_t>(kPushMax, std::max<size_t>(1, (units + kPushVecs - 1) / kPushVecs)));
  cfg.blockDim = dim3(256);
  cfg.stream = c->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = c->pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const int32_t *lc = (const int32_t *)c->dC;
  const PeerTable *dev = p->dev;
  // the tagged-word gather when the table has landing buffers for M rows and the layout is whole
  // 16-byte vectors (every rank's columns and the row stride multiples of 4)
  const bool tagged = wait && M <= t.land_rows && w->N % 4 == 0 && t.ldc % 4 == 0 && t.col0 % 4 == 0;
  if (tagged) {
    // at most four 256-thread CTAs per SM (the kernel's registers allow six), so the whole grid is
    // resident at once once the matmul before it has drained; larger runs grid-stride
    const size_t cv = (size_t)M * t.ldc / 4;
    cfg.gridDim = dim3((unsigned int)std::min<size_t>(148 * 4, std::max<size_t>(1, (cv + kPushVecs - 1) / kPushVecs)));
  }
  const cudaError_t e = tagged ? cudaLaunchKernelEx(&cfg, gather_tag_kernel, lc, M, w->N, dev)
                        : wait ? cudaLaunchKernelEx(&cfg, push_kernel<true>, lc, M, w->N, dev)
                               : cudaLaunchKernelEx(&cfg, push_kernel<false>, lc, M, w->N, dev);
  c->launches += 1;
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  return 0;
}

}  // namespace

extern "C" {

void *ork_b200_sym_alloc(ork_npu *c, size_t bytes, void *handle) {
  if (!c || !bytes || !handle) return nullptr;
  DeviceGuard dg(c->device);
  void *p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return nullptr;
  }
  static_assert(sizeof h == ORK_B200_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof h);
  return p;
}

int ork_b200_sym_free(ork_npu *c, void *p) {
  if (!c || !p) return -1;
  DeviceGuard dg(c->device);
  return cudaFree(p) == cudaSuccess ? 0 : -1;
}

void *ork_b200_sym_open(ork_npu *c, const void *handle) {
  if (!c || !handle) return nullptr;
  DeviceGuard dg(c->device);
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  void *p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

int ork_b200_sym_close(ork_npu *c, void *peer) {
  if (!c || !peer) return -1;
  DeviceGuard dg(c->device);
  return cudaIpcCloseMemHandle(peer) == cudaSuccess ? 0 : -1;
}

ork_b200_peers *ork_b200_peers_create(ork_npu *c, int nranks, int rank, void *const *C, void *const *flags, int ldc,
                                      int col0, int ncols) {
  if (!c || nranks < 1 || nranks > kMaxPeers || rank < 0 || rank >= nranks || !C || !flags || ldc < 1 || col0 < 0 ||
      ncols < 1 || col0 + ncols > ldc)
    return nullptr;
  for (int r = 0; r < nranks; r++)
    if (!C[r] || !flags[r] || (uintptr_t)C[r] % 4 || (uintptr_t)flags[r] % 4) return nullptr;
  DeviceGuard dg(c->device);
  ork_b200_peers *p = new (std::nothrow) ork_b200_peers;
  if (!p) return nullptr;
  p->ctx = c;
  PeerTable &t = p->host;
  t.n = nranks, t.rank = rank, t.ldc = ldc, t.col0 = col0, t.ctas = ncols;
  for (int r = 0; r < nranks; r++) {
    t.C[r] = (int32_t *)C[r];
    t.flag[r] = (unsigned int *)flags[r];
  }
  if (cudaMalloc(&p->dev, sizeof(PeerTable) + 256) != cudaSuccess) {
    delete p;
    return nullptr;
  }
  p->waited = (unsigned int *)((uint8_t *)p->dev + ((sizeof(PeerTable) + 255) & ~(size_t)255));
  t.waited = p->waited;
  t.done = p->waited + 1;
  t.runs = p->waited + 2;
  t.ldone = p->waited + 3;
  t.land_rows = 0;
  if (cudaMemset(p->waited, 0, 16) != cudaSuccess ||
      cudaMemcpy(p->dev, &t, sizeof t, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(p->dev);
    delete p;
    return nullptr;
  }
  return p;
}

int ork_b200_peers_land(ork_b200_peers *p, void *const *land, int rows) {
  if (!p || !land || rows < 1) return -1;
  PeerTable &t = p->host;
  for (int r = 0; r < t.n; r++)
    if (!land[r] || (uintptr_t)land[r] % 16) return -1;
  DeviceGuard dg(p->ctx->device);
  for (int r = 0; r < t.n; r++) t.land[r] = (uint64_t *)land[r];
  t.land_rows = rows;
  cudaStreamSynchronize(p->ctx->stream);  // no kernel of this table in flight while its copy changes
  return cudaMemcpy(p->dev, &t, sizeof t, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -1;
}

void ork_b200_peers_destroy(ork_b200_peers *p) {
  if (!p) return;
  DeviceGuard dg(p->ctx->device);
  cudaStreamSynchronize(p->ctx->stream);
  cudaFree(p->dev);
  delete p;
}

int ork_b200_i8_mm_run_peers_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p) {
  return peers_run(c, w, M, dA, p, DT_I8, false, "ork_b200_i8_mm_run_peers_async");
}

int ork_b200_i4_mm_run_peers_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p) {
  return peers_run(c, w, M, dA, p, DT_I4, false, "ork_b200_i4_mm_run_peers_async");
}

int ork_b200_i8_mm_run_gather_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p) {
  return peers_run(c, w, M, dA, p, DT_I8, true, "ork_b200_i8_mm_run_gather_async");
}

int ork_b200_i4_mm_run_gather_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, ork_b200_peers *p) {
  return peers_run(c, w, M, dA, p, DT_I4, true, "ork_b200_i4_mm_run_gather_async");
}

int ork_b200_copy(ork_npu *c, void *dst, const void *src, size_t bytes) {
  if (!c || !dst || !src) return -1;
  if (!bytes) return 0;
  DeviceGuard dg(c->device);
  if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  return cudaStreamSynchronize(c->stream) == cudaSuccess ? 0 : -1;
}

int ork_b200_peers_wait_async(ork_npu *c, ork_b200_peers *p) {
  if (!c || !p || p->ctx != c) return -1;
  DeviceGuard dg(c->device);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  cfg.stream = c->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = c->pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  const PeerTable *dev = p->dev;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, wait_kernel, dev);
  c->launches += 1;
  if (e != cudaSuccess) {
    log_err("ork_b200_peers_wait_async", e);
    return -1;
  }
  return 0;
}

}  // extern "C"
