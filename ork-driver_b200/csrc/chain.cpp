// chain.cpp -- batches of independent matmuls and the asynchronous submit / collect pair.
//
// ork-driver runs a batch of independent matmuls (its MoE experts, a layer's projections) as one chained
// NPU submit to amortise the per-submit cost (src/npu/i8/chain.c:56-71, include/ork/dynamic.h:14-30); the
// offline meaning of a batch is each task computed exactly (src/npu/core/buf.c:560-564). On B200 the cost
// being amortised is the kernel launch: every decode-sized task (M <= 8) of one weight format goes into
// ONE launch of the staged decode kernel (launch_gemv_batched, a task table as kernel parameter), larger
// tasks follow on the same stream through the ordinary route, and host buffers are staged once for the
// whole batch. ork_mm_submit / ork_mm_collect (include/ork/run.h:119-120; the reference serves them only
// through its daemon's ring) are a ring of in-flight slots, each with its own device buffers and event.
#include <cuda_runtime.h>
#include <sched.h>

#include <cstdio>
#include <cstring>
#include <vector>

#include "ork_b200.h"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"

using namespace orkb;

namespace {

struct TaskV {
  ork_w *w;
  int M;
  const void *A;
  void *C;
  int cs;  // C row stride in elements
};

size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

// How a batch treats its buffers and when it returns:
//   SYNC      host or device buffers; waits, every C complete on return (the reference's run calls);
//   DEVICE    device buffers of the context's GPU only; queued on the stream, returns at once;
//   DEFERRED  host or device buffers; queued on the stream, returns at once. Host A is copied through
//             the context's pinned staging unless it is pinned already; a host C that is not pinned is
//             read back into pinned staging and copied to the caller at ork_async_wait (`out`).
enum class Mode { SYNC, DEVICE, DEFERRED };

// A result row block left in pinned staging, copied to the caller's C when the job is waited for.
struct Scatter {
  void *dst;
  size_t src_off;       // in the context's pinned staging
  size_t row_bytes, dst_pitch;
  int rows;
};

bool pinned_host(const void *p) {
  cudaPointerAttributes at;
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

bool grow_pinned(ork_npu *c, size_t need) {
  if (c->capP >= need) return true;
  if (c->hP) cudaFreeHost(c->hP);
  c->hP = nullptr;
  c->capP = 0;
  const size_t sz = need < ((size_t)1 << 20) ? ((size_t)1 << 20) : need;
  if (cudaHostAlloc(&c->hP, sz, cudaHostAllocPortable) != cudaSuccess) {
    c->hP = nullptr;
    return false;
  }
  c->capP = sz;
  return true;
}

int run_batch(ork_npu *c, int S, const std::vector<TaskV> &t, int want_dtype, const char *name,
              Mode mode = Mode::SYNC, std::vector<Scatter> *out = nullptr) {
  if (!c || S < 0) return -1;
  if (S == 0) return 0;
  const bool dev_only = mode == Mode::DEVICE, deferred = mode == Mode::DEFERRED;
  const size_t esz = want_dtype == DT_F16 ? 2 : 1;
  for (int i = 0; i < S; i++) {
    const TaskV &v = t[i];
    if (!v.w || v.w->dtype != want_dtype || v.M < 1 || !v.A || !v.C || v.cs < v.w->N) return -1;
    const size_t ab = (size_t)v.M * v.w->K * esz, cb = ((size_t)(v.M - 1) * v.cs + v.w->N) * 4;
    if (overlaps(v.A, ab, v.C, cb)) {  // src/npu/core/submit.c:532-539
      fprintf(stderr, "[ork] ERROR [%s]: memory overlap detected in task %d (A and C).\n", name, i);
      return -1;
    }
  }
  DeviceGuard dg(c->device);
  // staging of host buffers: one region per task in the context's A and C buffers (and, for deferred
  // jobs, in its pinned host staging: pageable A is copied there first, pageable C read back there)
  std::vector<size_t> aoff(S, (size_t)-1), coff(S, (size_t)-1), hpa(S, (size_t)-1), hpc(S, (size_t)-1);
  std::vector<const void *> dA(S);
  std::vector<void *> dC(S);
  std::vector<bool> batched(S);
  size_t atot = 0, ctot = 0, ptot = 0;
  for (int i = 0; i < S; i++) {
    const TaskV &v = t[i];
    const size_t ab = (size_t)v.M * v.w->K * esz, cb = (size_t)v.M * v.w->N * 4;
    if (dev_only && !device_ptrs_ok(c, name, {v.A, v.C})) return -1;
    const bool a_dev = dev_only || (is_device_ptr(v.A, c->device) && (uintptr_t)v.A % 16 == 0);
    const bool c_dev = dev_only || (is_device_ptr(v.C, c->device) && (uintptr_t)v.C % 4 == 0);
    batched[i] = route_for(c, v.w, v.M) == 0 && batched_supports(v.w->fmt, v.M, v.w->K);
    // device pointers of the device-only form: no staging, so a strided C needs the batched kernel
    if (dev_only && ((uintptr_t)v.A % 16 || (uintptr_t)v.C % 4 || (!batched[i] && v.cs != v.w->N))) return -1;
    if (!a_dev) {
      aoff[i] = atot;
      atot += up256(ab);
      if (deferred && !pinned_host(v.A)) {
        hpa[i] = ptot;
        ptot += up256(ab);
      }
    }
    // a C the kernel cannot write in place: host memory, or a strided device C on the per-task route
    if (!c_dev || (!batched[i] && v.cs != v.w->N)) {
      coff[i] = ctot;
      ctot += up256(cb);
      if (deferred && !c_dev && !pinned_host(v.C)) {
        hpc[i] = ptot;
        ptot += up256(cb);
      }
    }
  }
  if (atot && !grow(&c->dA, &c->capA, atot)) return -1;
  if (ctot && !grow(&c->dC, &c->capC, ctot)) return -1;
  if (ptot && !grow_pinned(c, ptot)) return -1;
  for (int i = 0; i < S; i++) {
    const TaskV &v = t[i];
    if (aoff[i] != (size_t)-1) {
      const size_t ab = (size_t)v.M * v.w->K * esz;
      dA[i] = (uint8_t *)c->dA + aoff[i];
      const void *src = v.A;
      if (hpa[i] != (size_t)-1) {  // pageable A: into pinned staging now, so the copy below is asynchronous
        memcpy((uint8_t *)c->hP + hpa[i], v.A, ab);
        src = (uint8_t *)c->hP + hpa[i];
      }
      if (cudaMemcpyAsync((void *)dA[i], src, ab, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
    } else {
      dA[i] = v.A;
    }
    dC[i] = coff[i] != (size_t)-1 ? (uint8_t *)c->dC + coff[i] : v.C;
  }
  // one batched launch per weight format for the decode-sized tasks
  for (int fmt = FMT_F16; fmt <= FMT_NF4; fmt++) {
    std::vector<ChainTask> bt;
    for (int i = 0; i < S; i++) {
      const TaskV &v = t[i];
      if (!batched[i] || v.w->fmt != fmt) continue;
      const int cs = coff[i] != (size_t)-1 ? v.w->N : v.cs;  // staged C regions are contiguous
      bt.push_back(ChainTask{v.w->d, dA[i], dC[i], v.M, v.w->K, v.w->N, cs, fmt});
    }
    if (bt.empty()) continue;
    int nl = 0;
    const cudaError_t e = launch_gemv_batched(bt.data(), (int)bt.size(), c->stream, c->pdl, &nl);
    c->launches += (uint64_t)nl;
    if (e != cudaSuccess) {
      log_err(name, e);
      return -1;
    }
  }
  for (int i = 0; i < S; i++)
    if (!batched[i] && launch(c, t[i].w, t[i].M, dA[i], dC[i])) return -1;
  // results that were staged: to the caller's C at its row stride, or to pinned staging (deferred jobs)
  for (int i = 0; i < S; i++) {
    if (coff[i] == (size_t)-1) continue;
    const TaskV &v = t[i];
    const size_t rowb = (size_t)v.w->N * 4;
    if (hpc[i] != (size_t)-1) {
      if (cudaMemcpyAsync((uint8_t *)c->hP + hpc[i], dC[i], rowb * v.M, cudaMemcpyDeviceToHost, c->stream) !=
          cudaSuccess)
        return -1;
      out->push_back(Scatter{v.C, hpc[i], rowb, (size_t)v.cs * 4, v.M});
      continue;
    }
    if (cudaMemcpy2DAsync(v.C, (size_t)v.cs * 4, dC[i], rowb, rowb, (size_t)v.M, cudaMemcpyDefault, c->stream) !=
        cudaSuccess)
      return -1;
  }
  if (mode != Mode::SYNC) return 0;
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

std::vector<TaskV> views_i8(int S, const ork_mm_task_i8 *tasks) {
  std::vector<TaskV> t(S > 0 ? S : 0);
  for (int i = 0; i < S; i++) {
    const ork_mm_task_i8 &k = tasks[i];
    t[i] = TaskV{k.w, k.M, k.A, k.C, (k.cstride > 0 || !k.w) ? k.cstride : k.w->N};
  }
  return t;
}

std::vector<TaskV> views_i4(int S, const ork_mm_task_i4 *tasks) {
  std::vector<TaskV> t(S > 0 ? S : 0);
  for (int i = 0; i < S; i++) {
    const ork_mm_task_i4 &k = tasks[i];
    t[i] = TaskV{k.w, k.M, k.A, k.C, k.w ? k.w->N : 0};
  }
  return t;
}


// ---- submit / collect -----------------------------------------------------------------------------

constexpr int kSlots = 8;

struct Slot {
  void *dA = nullptr, *dC = nullptr;
  size_t capA = 0, capC = 0;
  cudaEvent_t ev = nullptr;
  bool busy = false;
  int gen = 0;
  size_t cbytes = 0;
};

struct Ring {
  Slot s[kSlots];
};

Ring *ring_of(ork_npu *c) {
  if (!c->ring) c->ring = new (std::nothrow) Ring;
  return (Ring *)c->ring;
}

}  // namespace

namespace orkb {
// Releases the submit ring's device buffers and events (ork_npu_free).
void ring_free(ork_npu *c) {
  if (!c || !c->ring) return;
  Ring *r = (Ring *)c->ring;
  for (Slot &s : r->s) {
    if (s.dA) cudaFree(s.dA);
    if (s.dC) cudaFree(s.dC);
    if (s.ev) cudaEventDestroy(s.ev);
  }
  delete r;
  c->ring = nullptr;
}
}  // namespace orkb

extern "C" {

int ork_i8_mm_run_chain(ork_npu *c, int S, const ork_mm_task_i8 *tasks) {
  if (S > 0 && !tasks) return -1;
  if (async_in_flight(c, "ork_i8_mm_run_chain")) return -1;
  return run_batch(c, S, views_i8(S, tasks), DT_I8, "ork_i8_mm_run_chain");
}

int ork_b200_i8_mm_run_chain_async(ork_npu *c, int S, const ork_mm_task_i8 *tasks) {
  if (S > 0 && !tasks) return -1;
  return run_batch(c, S, views_i8(S, tasks), DT_I8, "ork_b200_i8_mm_run_chain_async", Mode::DEVICE);
}

int ork_i8_mm_run_stream(ork_npu *c, int S, const ork_mm_task_i8 *tasks) { return ork_i8_mm_run_chain(c, S, tasks); }

int ork_i4_mm_run_chain(ork_npu *c, int S, const ork_mm_task_i4 *tasks) {
  if (S > 0 && !tasks) return -1;
  if (async_in_flight(c, "ork_i4_mm_run_chain")) return -1;
  return run_batch(c, S, views_i4(S, tasks), DT_I4, "ork_i4_mm_run_chain");
}

// include/ork/chain.h:123: the int4 twin of ork_i8_mm_run_stream. The reference deals the tasks round-robin
// over its NPU cores; here the whole GPU serves the batch, as for the int4 chain.
int ork_i4_mm_run_stream(ork_npu *c, int S, const ork_mm_task_i4 *tasks) { return ork_i4_mm_run_chain(c, S, tasks); }

int ork_i4_mm_run_experts(ork_npu *c, const ork_mm_task_i4 *ex, int ntask, int nc) {
  (void)nc;  // NPU core count: the whole GPU serves the batch
  return ork_i4_mm_run_chain(c, ntask, ex);
}

int ork_mm_submit(ork_npu *c, ork_w *w, int M, const void *A) {
  if (!c || !w || M < 1 || !A) return -1;
  if (async_in_flight(c, "ork_mm_submit")) return -1;
  Ring *r = ring_of(c);
  if (!r) return -1;
  int si = -1;
  for (int i = 0; i < kSlots; i++)
    if (!r->s[i].busy) {
      si = i;
      break;
    }
  if (si < 0) return -1;  // every slot in flight: collect first
  Slot &s = r->s[si];
  DeviceGuard dg(c->device);
  const size_t ab = (size_t)M * w->K * (w->dtype == DT_F16 ? 2 : 1), cb = (size_t)M * w->N * 4;
  if (!s.ev && cudaEventCreateWithFlags(&s.ev, cudaEventDisableTiming) != cudaSuccess) return -1;
  if (!grow(&s.dA, &s.capA, ab) || !grow(&s.dC, &s.capC, cb)) return -1;
  if (cudaMemcpyAsync(s.dA, A, ab, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  if (launch(c, w, M, s.dA, s.dC)) return -1;
  if (cudaEventRecord(s.ev, c->stream) != cudaSuccess) return -1;
  s.busy = true;
  s.cbytes = cb;
  s.gen = (s.gen + 1) % 1000000;
  return s.gen * kSlots + si;
}

int ork_mm_collect(ork_npu *c, int ticket, void *C) {
  if (!c || !c->ring || ticket < 0 || !C) return -1;
  Ring *r = (Ring *)c->ring;
  Slot &s = r->s[ticket % kSlots];
  if (!s.busy || s.gen != ticket / kSlots) return -1;
  DeviceGuard dg(c->device);
  s.busy = false;
  cudaError_t e = cudaEventSynchronize(s.ev);
  if (e == cudaSuccess) e = cudaMemcpy(C, s.dC, s.cbytes, cudaMemcpyDefault);
  if (e != cudaSuccess) {
    log_err("ork_mm_collect", e);
    return -1;
  }
  if (device_error()) {
    fprintf(stderr, "[ork] ERROR ork_mm_collect: a kernel's bounded pipeline wait timed out; result discarded\n");
    return -1;
  }
  return 0;
}

// ---- ork_async: runs over host buffers that return at once (include/ork/chain.h:124-143) ---------------
//
// The reference gets CPU || NPU overlap by running its blocking submit on a worker thread. A GPU is
// asynchronous already, so here a launcher queues the whole job on the context's stream -- A into device
// staging (through pinned host staging when A is pageable), the kernels, C back to pinned staging (or
// straight into C when C is pinned or device memory) -- records an event and returns. ork_async_wait
// waits for the event, copies staged results to the caller's C and reports the job's status. No thread
// is created. One job per context at a time (a second launch returns NULL, every other run on the
// context returns -1 until the wait), the task arrays and buffers must stay valid until the wait.

}  // extern "C"

struct ork_async {
  ork_npu *c = nullptr;
  int rc = -1;  // < 0: the job was refused when queued and nothing is in flight
  std::vector<Scatter> out;
};

namespace {

ork_async *async_launch(ork_npu *c, int S, const std::vector<TaskV> &t, int dtype, const char *name) {
  if (c->async_busy) {
    fprintf(stderr, "[ork] ERROR %s: an ork_async job is already in flight on this context\n", name);
    return nullptr;
  }
  ork_async *h = new (std::nothrow) ork_async;
  if (!h) return nullptr;
  h->c = c;
#if defined(__linux__)
  c->last_async_cpu = sched_getcpu();
#endif
  DeviceGuard dg(c->device);
  if (!c->async_ev && cudaEventCreateWithFlags(&c->async_ev, cudaEventDisableTiming) != cudaSuccess) return h;
  if (run_batch(c, S, t, dtype, name, Mode::DEFERRED, &h->out) != 0) {
    // whatever was queued finishes before the handle is handed back, so a refused job leaves nothing
    // in flight on the context's buffers
    cudaStreamSynchronize(c->stream);
    h->out.clear();
    return h;
  }
  if (cudaEventRecord(c->async_ev, c->stream) != cudaSuccess) {
    cudaStreamSynchronize(c->stream);
    h->out.clear();
    return h;
  }
  h->rc = 0;
  c->async_busy = true;
  return h;
}

ork_async *async_run(ork_npu *c, ork_w *w, int M, const void *A, void *C, int dtype, const char *name) {
  std::vector<TaskV> t{TaskV{w, M, A, C, w->N}};
  return async_launch(c, 1, t, dtype, name);
}

}  // namespace

extern "C" {

// Launchers: NULL for a NULL context or weight, M < 1, an int8 run on a weight of another kind, an empty
// or NULL task list (the reference's refusals, src/npu.c:2212-2222, src/npu/i8/run.c:778-784), or a job
// already in flight; other argument errors are reported by ork_async_wait, as the reference's worker
// reports them.
ork_async *ork_mm_run_async(ork_npu *c, ork_w *w, int M, const ork_f16 *A, float *C) {
  if (!c || !w || M < 1) return nullptr;
  return async_run(c, w, M, A, C, DT_F16, "ork_mm_run_async");
}
ork_async *ork_i8_mm_run_async(ork_npu *c, ork_w *w, int M, const int8_t *A, int32_t *C) {
  if (!c || !w || w->dtype != DT_I8 || M < 1) return nullptr;
  return async_run(c, w, M, A, C, DT_I8, "ork_i8_mm_run_async");
}
ork_async *ork_i4_mm_run_async(ork_npu *c, ork_w *w, int M, const int8_t *A, int32_t *C) {
  if (!c || !w || M < 1) return nullptr;
  return async_run(c, w, M, A, C, DT_I4, "ork_i4_mm_run_async");
}
ork_async *ork_i8_mm_run_chain_async(ork_npu *c, int S, const ork_mm_task_i8 *tasks) {
  if (!c || S < 1 || !tasks) return nullptr;
  return async_launch(c, S, views_i8(S, tasks), DT_I8, "ork_i8_mm_run_chain_async");
}
ork_async *ork_i4_mm_run_chain_async(ork_npu *c, int S, const ork_mm_task_i4 *tasks) {
  if (!c || S < 1 || !tasks) return nullptr;
  return async_launch(c, S, views_i4(S, tasks), DT_I4, "ork_i4_mm_run_chain_async");
}
ork_async *ork_i8_mm_run_stream_async(ork_npu *c, int S, const ork_mm_task_i8 *tasks) {
  if (!c || S < 1 || !tasks) return nullptr;
  return async_launch(c, S, views_i8(S, tasks), DT_I8, "ork_i8_mm_run_stream_async");
}
ork_async *ork_i4_mm_run_stream_async(ork_npu *c, int S, const ork_mm_task_i4 *tasks) {
  if (!c || S < 1 || !tasks) return nullptr;
  return async_launch(c, S, views_i4(S, tasks), DT_I4, "ork_i4_mm_run_stream_async");
}

int ork_async_wait(ork_async *h) {
  if (!h) return -1;
  int rc = h->rc;
  ork_npu *c = h->c;
  if (rc == 0) {
    DeviceGuard dg(c->device);
    const cudaError_t e = cudaEventSynchronize(c->async_ev);
    c->async_busy = false;
    if (e != cudaSuccess) {
      log_err("ork_async_wait", e);
      rc = -1;
    } else if (device_error()) {
      fprintf(stderr, "[ork] ERROR ork_async_wait: a kernel's bounded pipeline wait timed out; result discarded\n");
      rc = -1;
    } else {
      for (const Scatter &s : h->out)
        for (int r = 0; r < s.rows; r++)
          memcpy((uint8_t *)s.dst + (size_t)r * s.dst_pitch, (const uint8_t *)c->hP + s.src_off + (size_t)r * s.row_bytes,
                 s.row_bytes);
    }
  }
  delete h;
  return rc;
}

int ork_npu_last_async_cpu(ork_npu *c) { return c ? c->last_async_cpu : -1; }

}  // extern "C"
