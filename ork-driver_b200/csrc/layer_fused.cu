// layer_fused.cu -- the decode layer (ork_i8_mm_layer, ork-driver include/ork/chain.h:105-110) as ONE
// persistent kernel per layer on B200.
//
// At M = 1 a Qwen3-1.7B layer streams ~50 MB of int8 weights, ~8 us at HBM speed, but as nine dependent
// launches (layer.cu) it takes ~45 us: every launch pays its ramp-up and drain, and the glue runs on one
// CTA. Here one cooperative launch of one CTA per SM runs the layer in five phases:
//   A  every CTA: RMSNorm + int8 quantization of x into its shared memory (redundant -- the row is a
//      few KB); its share of the q / k / v rows
//   B  split-KV attention: items (head, chunk of keys) spread over the CTAs, each writing its chunk's max,
//      exp-sum and exp-weighted V row; then CTA h merges head h -> ao, max |ao| of the head
//   C  every CTA: quantization of ao with the max over the heads; its share of the o rows
//   D  every CTA: x1 = x + Co / sa, RMSNorm + quantization; its share of the gate AND the up rows (the same
//      channels), so SwiGLU runs in the epilogue -> h, this CTA's max |h|
//   E  every CTA: quantization of h with the max over the CTAs; its share of the down rows, the residual
//      in the epilogue -> x_out
// Phases hand data to each other through 64-bit words holding the value and the launch's epoch, so a
// reader can tell this launch's values from stale ones without a memory fence. Where few CTAs read a
// value (an attention item's q / k / v, a head's chunk partials) they poll the words themselves; for the
// all-to-all hand-offs (ao, o, h) one thread per CTA polls an arrival count first. (Every CTA takes part in
// every hand-off, so a CTA that has all of a phase's inputs knows every CTA is past the phase that read
// what it is about to overwrite.) The launch's epoch is one more than the last launch's: the last CTA to
// finish advances it and clears the counts.
// The weights do not depend on the data, so one producer warp per CTA streams the CTA's rows of all
// seven weights, in phase order, through a ring of shared-memory slots (bulk asynchronous copies,
// cp.async.bulk, one per slot, marked evict-first in L2: they are read once per token) from the kernel's
// first cycle: while the CTA waits for data or runs attention, the next phases' rows are landing.
// Each slot belongs to one compute warp, which takes all its rows at once (lanes across K, one activation
// load shared by the rows, a butterfly reduction of up to eight row sums).
//
// The glue is glue.cuh's, in the reference's operation order, except the softmax, which is online per
// warp (rescaled partial maxima, as in the split-KV merge); every CTA computes the redundant reductions in
// the same order, so the values all CTAs hold agree bit for bit. Integer matmul results are exact.
// Waits are bounded (mbarriers and data polls, ~2 s of SM clock): on expiry the kernel records the error
// and runs on, so it always ends; the producer waits for its last copies before it exits.
#include <cuda_runtime.h>

#include <algorithm>

#include "glue.cuh"
#include "nibble.cuh"
#include "errword.cuh"
#include "ork_internal.h"

namespace orkb {

namespace {

constexpr int kCW = 16;              // compute warps
constexpr int kCT = kCW * 32;        // compute threads (they synchronise on named barrier 1)
constexpr int kFThreads = kCT + 32;  // + the producer warp
constexpr int kMaxSlots = 32;
constexpr int kFMaxSplit = 256;
constexpr int kRowsPass = 8;  // rows a warp reduces together
constexpr int kLB = 4;        // row elements a thread loads at once in the glue
constexpr int kHB = 12;       // SwiGLU elements a thread loads at once (F <= 6144 in one round)
constexpr uint64_t kSpin = 4000000000ull;
constexpr int kSmemMax = 227 * 1024 - 2048;  // dynamic part; the static barriers, tables and scratch use <= 2 KB

__device__ unsigned int g_fused_error = 0;

using glue::q8;

__device__ __forceinline__ uint32_t su32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(kCT) : "memory"); }

__device__ __forceinline__ float warp_sum(float v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ float c_sum(float v, float *red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  cbar();
  if (l == 0) red[w] = v;
  cbar();
  return warp_sum(l < kCW ? red[l] : 0.0f);
}

__device__ float c_max(float v, float *red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  cbar();
  if (l == 0) red[w] = v;
  cbar();
  return warp_max(l < kCW ? red[l] : -3.0e38f);
}

// Error bits: 1 a ring wait expired, 2 a data wait expired, 4 the device-read position does not fit the
// caches (attention skipped). A wait gives up when it has waited ~2 s, or early when another wait
// already gave up, so a failed launch ends after one expiry instead of one per wait; launches after it
// fail fast until the host reads and clears the flag.
__device__ __forceinline__ bool gave_up() { return (*(volatile unsigned int *)&g_fused_error & 3u) != 0u; }

// The waiting thread sleeps in the barrier until the phase completes (the hint caps one sleep at 1 ms), so
// a warp that waits issues almost nothing while the others compute.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kSpin || gave_up()) {
      { atomicOr(&g_fused_error, 1u); err_word_set(); }
      return false;
    }
  }
}

// Epoch-tagged words: value bits low, epoch high; one aligned 64-bit access each, so a reader that sees
// the epoch sees the value.
__device__ __forceinline__ void ll_put(uint64_t *p, uint32_t v, uint32_t ep) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((uint64_t)ep << 32) | v) : "memory");
}
__device__ __forceinline__ void ll_putf(uint64_t *p, float v, uint32_t ep) { ll_put(p, __float_as_uint(v), ep); }

__device__ __forceinline__ uint64_t ll_load(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Arrival counters for the all-to-all hand-offs (ao, o, h: every CTA reads all of them): after issuing
// its tagged words a CTA adds one (relaxed, fire-and-forget), and one thread per reader polls the count
// -- one word polled per CTA instead of the whole vector. No fence: a word whose epoch is not yet visible
// when the count is is simply re-polled.
__device__ __forceinline__ void arrive(unsigned int *c) {
  cbar();
  if (threadIdx.x == 0) asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(c) : "memory");
}

__device__ void await_count(const unsigned int *c, unsigned int n) {
  if (threadIdx.x == 0) {
    const uint64_t t0 = clock64();
    while (true) {
      unsigned int v;
      asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
      if (v >= n) break;
      if (clock64() - t0 > kSpin || gave_up()) {
        { atomicOr(&g_fused_error, 2u); err_word_set(); }
        break;
      }
    }
  }
  cbar();
}

// re-poll one word until it carries epoch ep (bounded); w is its first read
__device__ __noinline__ uint32_t ll_wait(const uint64_t *p, uint64_t w, uint32_t ep) {
  const uint64_t t0 = clock64();
  while ((uint32_t)(w >> 32) != ep) {
    if (clock64() - t0 > kSpin || gave_up()) {
      { atomicOr(&g_fused_error, 2u); err_word_set(); }
      break;
    }
    w = ll_load(p);
  }
  return (uint32_t)w;
}

// N words at p[i0 + u * stride] (those below n; the others read as written): ll_issue puts the loads in
// flight, ll_finish re-polls any not yet written. Several vectors issued before the first finish cost one
// round trip together.
template <int N>
__device__ __forceinline__ void ll_issue(const uint64_t *p, int i0, int stride, int n, uint32_t ep, uint64_t (&w)[N]) {
#pragma unroll
  for (int u = 0; u < N; u++) w[u] = i0 + u * stride < n ? ll_load(p + i0 + u * stride) : ((uint64_t)ep << 32);
}
template <int N>
__device__ __forceinline__ void ll_finish(const uint64_t *p, int i0, int stride, uint32_t ep, const uint64_t (&w)[N],
                                          uint32_t (&v)[N]) {
#pragma unroll
  for (int u = 0; u < N; u++)
    v[u] = (uint32_t)(w[u] >> 32) == ep ? (uint32_t)w[u] : ll_wait(p + i0 + u * stride, w[u], ep);
}
template <int N>
__device__ __forceinline__ void ll_get_n(const uint64_t *p, int i0, int stride, int n, uint32_t ep, uint32_t (&v)[N]) {
  uint64_t w[N];
  ll_issue<N>(p, i0, stride, n, ep, w);
  ll_finish<N>(p, i0, stride, ep, w, v);
}

// The layer's pointer table, 8-byte words copied into shared memory by asynchronous copies (the next
// layer's while this one runs), so no phase starts with a dependent global load of a pointer.
constexpr int kLwWords = (int)(sizeof(FusedLayerW) / 8);
static_assert(sizeof(FusedLayerW) % 8 == 0, "the layer table copies in 8-byte words");
__device__ __forceinline__ void lw_fetch(FusedLayerW *dst, const FusedLayerW *src, int t) {
  if (t < kLwWords) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(su32(dst) + 8u * t),
                 "l"(reinterpret_cast<const uint64_t *>(src) + t)
                 : "memory");
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
}
__device__ __forceinline__ void lw_landed(int t) {
  if (t < kLwWords) asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---- the CTA's rows of each phase ---------------------------------------------------------------
struct Range {
  int w, r0, r1;  // weight (0..6), rows [r0, r1)
};

__device__ __forceinline__ int wK(const FusedArgs &a, int w) { return w == 3 ? a.H * a.dk : w == 6 ? a.F : a.D; }

template <int FMT>
__device__ __forceinline__ uint32_t row_bytes(int K) {
  return FMT == FMT_I8 ? (uint32_t)K : (uint32_t)K / 2;
}

__device__ __forceinline__ void share(int N, int b, int G, int &lo, int &hi) {
  lo = (int)(((unsigned)N * (unsigned)b) / (unsigned)G);
  hi = (int)(((unsigned)N * (unsigned)(b + 1)) / (unsigned)G);
}

// phase 0 = q/k/v, 1 = o, 2 = gate/up, 3 = down: balanced contiguous shares of the rows per CTA (q, k, v
// as one concatenation; gate and up the same channels)
__device__ int ranges(const FusedArgs &a, int p, int b, int G, Range *r) {
  int n = 0, lo, hi;
  if (p == 0) {
    const int Nq = a.H * a.dk, Nk = a.Hkv * a.dk;
    share(Nq + 2 * Nk, b, G, lo, hi);
    const int edge[4] = {0, Nq, Nq + Nk, Nq + 2 * Nk};
    for (int w = 0; w < 3; w++) {
      const int s = max(lo, edge[w]), e = min(hi, edge[w + 1]);
      if (s < e) r[n++] = Range{w, s - edge[w], e - edge[w]};
    }
  } else if (p == 1 || p == 3) {
    share(a.D, b, G, lo, hi);
    if (lo < hi) r[n++] = Range{p == 1 ? 3 : 6, lo, hi};
  } else {
    share(a.F, b, G, lo, hi);
    if (lo < hi) {
      r[n++] = Range{4, lo, hi};
      r[n++] = Range{5, lo, hi};
    }
  }
  return n;
}

// ---- producer: the CTA's rows of all phases, in consumption order, through the ring -------------
template <int FMT>
__device__ void produce(const FusedArgs &a, uint32_t ring, uint32_t full0, uint32_t empty0, int G) {
  const uint32_t ns = (uint32_t)a.nslots;
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  uint32_t k = 0, s = 0, use = 0;
  for (int lp = 0; lp < 4 * a.nl; lp++) {  // every layer's phases in order: the stream never pauses
    const int p = lp & 3;
    const FusedLayerW *lw = a.lw ? a.lw + (lp >> 2) : &a.lw0;
    Range r[3];
    const int n = ranges(a, p, blockIdx.x, G, r);
    for (int i = 0; i < n; i++) {
      const uint32_t rowB = row_bytes<FMT>(wK(a, r[i].w));
      const int rps = (int)(a.slot / rowB);
      const uint8_t *W = lw->W[r[i].w];
      for (int r0 = r[i].r0; r0 < r[i].r1; r0 += rps, k++) {
        const int nr = min(rps, r[i].r1 - r0);
        if (use > 0) mbar_wait(empty0 + 8 * s, (use - 1) & 1);  // the slot's previous rows consumed
        const uint32_t bytes = (uint32_t)nr * rowB, fb = full0 + 8 * s;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb), "r"(bytes) : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
            "%4;" ::"r"(ring + s * a.slot),
            "l"(W + (size_t)r0 * rowB), "r"(bytes), "r"(fb), "l"(pol)
            : "memory");
        if (++s == ns) {
          s = 0;
          use++;
        }
      }
    }
  }
  // leave no copy in flight: wait for the last ring's worth to land (immediate unless a wait expired)
  for (uint32_t j = k > ns ? k - ns : 0; j < k; j++) mbar_wait(full0 + 8 * (j % ns), (j / ns) & 1);
}

// ---- consumers: each slot to one warp, its rows together ----------------------------------------
// Sum of v[0..7] over the warp's lanes for eight rows at once: three exchange steps each halve the rows a
// lane holds, two more finish the sum. Lane l then holds the total of row ((l >> 4) & 1) * 4 +
// ((l >> 3) & 1) * 2 + ((l >> 2) & 1).
__device__ __forceinline__ int reduce8(int (&v)[kRowsPass], int lane) {
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int send = h16 ? v[i] : v[i + 4], keep = h16 ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int send = h8 ? v[i] : v[i + 2], keep = h8 ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const int send = h4 ? v[0] : v[1], keep = h4 ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return v[0];
}

// up to eight rows of one slot against the activation row; the sums come back as reduce8 leaves them
template <int FMT>
__device__ __forceinline__ int rows_dot(uint32_t w, uint32_t a8, uint32_t rowB, int nr, int lane, const Nf4Tables &tb) {
  int acc[kRowsPass];
#pragma unroll
  for (int r = 0; r < kRowsPass; r++) acc[r] = 0;
  const int nch = (int)(rowB / 16);
  for (int c = lane; c < nch; c += 32) {
    if constexpr (FMT == FMT_I8) {
      const uint4 av = lds128(a8 + 16u * c);
#pragma unroll
      for (int r = 0; r < kRowsPass; r++)
        if (r < nr) {
          const uint4 wv = lds128(w + (uint32_t)r * rowB + 16u * c);
          acc[r] = dp4a(av.x, wv.x, acc[r]);
          acc[r] = dp4a(av.y, wv.y, acc[r]);
          acc[r] = dp4a(av.z, wv.z, acc[r]);
          acc[r] = dp4a(av.w, wv.w, acc[r]);
        }
    } else {  // 32 nibbles -> 32 int8 codes in k order, against 32 activation bytes
      const uint4 a0 = lds128(a8 + 32u * c), a1 = lds128(a8 + 32u * c + 16u);
#pragma unroll
      for (int r = 0; r < kRowsPass; r++)
        if (r < nr) {
          const uint4 wv = lds128(w + (uint32_t)r * rowB + 16u * c);
          const uint2 e0 = expand8<FMT>(wv.x, tb), e1 = expand8<FMT>(wv.y, tb);
          const uint2 e2 = expand8<FMT>(wv.z, tb), e3 = expand8<FMT>(wv.w, tb);
          int s = acc[r];
          s = dp4a(a0.x, e0.x, s);
          s = dp4a(a0.y, e0.y, s);
          s = dp4a(a0.z, e1.x, s);
          s = dp4a(a0.w, e1.y, s);
          s = dp4a(a1.x, e2.x, s);
          s = dp4a(a1.y, e2.y, s);
          s = dp4a(a1.z, e3.x, s);
          s = dp4a(a1.w, e3.y, s);
          acc[r] = s;
        }
    }
  }
  return reduce8(acc, lane);
}

// One phase of the CTA: its row ranges and where the row results go. Thread 0 writes it to shared memory
// before the phase; the compute warps read it there (uniform loads, no per-thread copies).
// A CTA's rows of one phase and how they fill the ring: the same for every layer, so computed once per
// launch (the divisions stay out of the phases).
struct PhaseGeo {
  int n;                    // row ranges
  Range r[3];
  int rps[3], nslot[3];     // rows per slot, slots
  uint32_t rowB[3];         // bytes per row
  uint32_t nsq[3], nsr[3];  // slots / ring size, slots % ring size
};
// The running slot index kc of the consumers as kc / ns and kc % ns.
struct Cursor {
  uint32_t base, rem;
};
template <int FMT>
__device__ void phase_geo(const FusedArgs &a, int p, int G, PhaseGeo &g) {
  g.n = ranges(a, p, blockIdx.x, G, g.r);
  const uint32_t ns = (uint32_t)a.nslots;
  for (int i = 0; i < g.n; i++) {
    const uint32_t rowB = row_bytes<FMT>(wK(a, g.r[i].w));
    const int rps = (int)(a.slot / rowB), nslot = (g.r[i].r1 - g.r[i].r0 + rps - 1) / rps;
    g.rowB[i] = rowB, g.rps[i] = rps, g.nslot[i] = nslot;
    g.nsq[i] = (uint32_t)nslot / ns, g.nsr[i] = (uint32_t)nslot % ns;
  }
}

struct Plan {
  uint64_t *C[3];  // phase 0: q, k, v (by weight); phase 1: o
  int *loc;       // phase 2: this CTA's gate results, then its up results (nf each)
  int f0, nf;
  float *out;     // phase 3: x_out = x1 + v / s (the last layer), or
  uint64_t *xl;   // phase 3: the next layer's x as tagged words
  const float *x1;
  float s;
};

// Consume the planned phase's slots (the sequence the producer issued, from slot kc). Ring slot s belongs
// to warp s % kCW for all its uses, so one warp consumes each slot's uses in order: a warp never waits on
// a slot's next use before that slot's previous use landed (a parity wait two phases ahead would pass at
// once and let the producer re-arm a barrier whose copy is still in flight). A warp visits only its own
// slots' indices, in increasing order (its ring slots w and w + kCW interleaved), from the cursor and the
// precomputed geometry, with no division: walking every index with a runtime modulo cost the slowest warp
// ~5,000 cycles a phase. Returns the advanced cursor.
static_assert(kMaxSlots <= 2 * kCW, "a warp owns at most two ring slots");
template <int FMT>
__device__ __noinline__ Cursor consume(const FusedArgs &a, const PhaseGeo &g, const Plan &pl, int p, Cursor cur, uint32_t ring,
                                         uint32_t full0, uint32_t empty0, uint32_t a8, const Nf4Tables tb,
                                         uint32_t ep) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ns = (uint32_t)a.nslots;
  const int lr = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);  // row of reduce8's lane
  const int n = g.n;
#pragma unroll
  for (int i = 0; i < 3; i++) {
    if (i >= n) break;
    const int w = g.r[i].w, rb = g.r[i].r0, re = g.r[i].r1;
    const uint32_t rowB = g.rowB[i];
    const int rps = g.rps[i], nslot = g.nslot[i];
    uint64_t *C = p == 0 ? pl.C[w] : pl.C[0];
    // index kc + q sits in ring slot (kc + q) % ns with parity ((kc + q) / ns) & 1
    const uint32_t base = cur.base, rem = cur.rem;
    uint32_t nq[2], wr[2];  // next index of each of the warp's ring slots, and its use count
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const uint32_t sj = (uint32_t)(warp + j * kCW);
      nq[j] = sj >= ns ? 0xffffffffu : sj >= rem ? sj - rem : sj + ns - rem;
      wr[j] = base + (sj >= rem ? 0u : 1u);
    }
    while (true) {
      const int j = nq[1] < nq[0] ? 1 : 0;
      const uint32_t q32 = nq[j];
      if (q32 >= (uint32_t)nslot) break;
      const int q = (int)q32;
      const uint32_t s = (uint32_t)(warp + j * kCW), par = wr[j] & 1u;
      nq[j] += ns;
      wr[j] += 1u;
      const int r0 = rb + q * rps, nr = min(rps, re - r0);
      const bool ok = mbar_wait(full0 + 8 * s, par);
      for (int j0 = 0; j0 < nr; j0 += kRowsPass) {
        const int m = min(kRowsPass, nr - j0);
        const int v = ok ? rows_dot<FMT>(ring + s * a.slot + (uint32_t)j0 * rowB, a8, rowB, m, lane, tb) : 0;
        if ((lane & 3) == 0 && lr < m) {
          const int row = r0 + j0 + lr;
          if (p <= 1)
            ll_put(C + row, (uint32_t)v, ep);
          else if (p == 2)
            pl.loc[(w == 4 ? 0 : pl.nf) + row - pl.f0] = v;
          else if (pl.out)
            pl.out[row] = pl.x1[row] + v / pl.s;
          else
            ll_putf(pl.xl + row, pl.x1[row] + v / pl.s, ep);
        }
      }
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(empty0 + 8 * s) : "memory");
    }
    cur.base += g.nsq[i];
    cur.rem += g.nsr[i];
    if (cur.rem >= ns) {
      cur.rem -= ns;
      cur.base++;
    }
  }
  return cur;
}

// ---- phase B: one split-KV attention item, warp-centric -------------------------------------------
// A head vector of dk = 32 * PER values, lane holding elements lane + 32 i, from its raw int32 projection:
// dequantized, RMS-normed with gain g (if any), rotated at pos. The NeoX pair (d, d + dk / 2) is
// (i, i + PER / 2) in the same lane.
template <int PER>
__device__ __forceinline__ void head_vec(const uint32_t (&c)[PER], float sx, bool has_g, const float (&g)[PER], int pos,
                                         float base, int lane, float (&v)[PER]) {
  constexpr int dk = 32 * PER;
#pragma unroll
  for (int i = 0; i < PER; i++) v[i] = (int32_t)c[i] / sx;
  if (has_g) {
    float sq = 0.0f;
#pragma unroll
    for (int i = 0; i < PER; i++) sq += v[i] * v[i];
    const float rr = glue::rms_recip(warp_sum(sq), dk);
#pragma unroll
    for (int i = 0; i < PER; i++) v[i] = v[i] * rr * g[i];
  }
#pragma unroll
  for (int i = 0; i < PER / 2; i++) {
    const float th = glue::rope_angle(pos, base, lane + 32 * i, dk);
    const float c = cosf(th), s = sinf(th), x0 = v[i], x1 = v[i + PER / 2];
    v[i] = x0 * c - x1 * s;
    v[i + PER / 2] = x0 * s + x1 * c;
  }
}

// Keys jb and jb + kCW of the cache (zeros at or past j1): a warp's step of two keys, lane holding
// elements lane + 32 i of each row.
template <int PER>
__device__ __forceinline__ void load_keys(const float *Kh, const float *Vh, int jb, int j1, int lane,
                                          float (&kr)[2][PER], float (&vr)[2][PER]) {
  constexpr int dk = 32 * PER;
#pragma unroll
  for (int u = 0; u < 2; u++) {
    const int j = jb + u * kCW;
    const bool in = j < j1;
    const float *kp = Kh + (size_t)j * dk + lane, *vp = Vh + (size_t)j * dk + lane;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      kr[u][i] = in ? kp[32 * i] : 0.0f;
      vr[u][i] = in ? vp[32 * i] : 0.0f;
    }
  }
}

// Item (h, sp) of S: keys [sp * kpc, min(nk, sp * kpc + kpc)) of query head h. Warp w takes keys
// j0 + w + 16 u with an online softmax (running max, rescaled sums); the CTA then combines its warps'
// maxima, sums and V rows into the item's partials. y: scratch, [kCW][dk] rows then 2 * kCW floats.
// The first step's cached rows and the norm gains do not depend on this launch's data, so their loads
// are issued before q is checked (the token's own key, not yet in the cache, replaces its row when it is
// used).
template <int PER>
__device__ void attend(const FusedArgs &a, const FusedLayerW &lw, int h, int sp, int kpc, int nkv, int nk, int pos,
                       float sx, float *y, uint32_t ep) {
  constexpr int dk = 32 * PER;
  const int t = threadIdx.x, lane = t & 31, wp = t >> 5;
  const int grp = a.H / a.Hkv, hk = h / grp, Sg = a.Sg;
  const bool ext = a.ext != 0;
  const int j0 = sp * kpc, j1 = min(nk, j0 + kpc);
  const bool own = ext && j0 <= nkv && nkv < j1;
  const float *Kh = lw.Kc + (size_t)hk * a.hstride * dk, *Vh = lw.Vc + (size_t)hk * a.hstride * dk;
  // the first poll of q goes out ahead of the key rows' loads (a poll queued behind them would return
  // later); q is checked after they are issued
  uint64_t wq[PER];
  ll_issue<PER>(a.q + h * dk, lane, 32, dk, ep, wq);
  float kr[2][PER], vr[2][PER];
  int jb = j0 + wp;
  load_keys<PER>(Kh, Vh, jb, j1, lane, kr, vr);
  const bool hq = lw.q_norm != nullptr, hk_ = lw.k_norm != nullptr;
  float gq[PER], gk[PER];
#pragma unroll
  for (int i = 0; i < PER; i++) {
    gq[i] = hq ? lw.q_norm[lane + 32 * i] : 1.0f;
    gk[i] = hk_ && own ? lw.k_norm[lane + 32 * i] : 1.0f;
  }
  // the raw q (and the token's own k, v): q first (what is awaited); the token's k and v, written in the
  // same phase, in one round after
  uint32_t cq[PER], ck[PER], cv[PER];
  ll_finish<PER>(a.q + h * dk, lane, 32, ep, wq, cq);
  {
    uint64_t wk[PER], wv[PER];
    ll_issue<PER>(a.k + hk * dk, lane, 32, own ? dk : 0, ep, wk);
    ll_issue<PER>(a.v + hk * dk, lane, 32, own ? dk : 0, ep, wv);
    ll_finish<PER>(a.k + hk * dk, lane, 32, ep, wk, ck);
    ll_finish<PER>(a.v + hk * dk, lane, 32, ep, wv, cv);
  }
  float q[PER], kn[PER], vn[PER];
  head_vec<PER>(cq, sx, hq, gq, pos, a.base, lane, q);
  if (own) {
    head_vec<PER>(ck, sx, hk_, gk, pos, a.base, lane, kn);
#pragma unroll
    for (int i = 0; i < PER; i++) vn[i] = (int32_t)cv[i] / sx;
    if (h % grp == 0 && wp == 0)  // the group's first query head stores the token's k and v
#pragma unroll
      for (int i = 0; i < PER; i++) {
        lw.Kc[((size_t)hk * a.hstride + nkv) * dk + lane + 32 * i] = kn[i];
        lw.Vc[((size_t)hk * a.hstride + nkv) * dk + lane + 32 * i] = vn[i];
      }
  }
  float m = -3.0e38f, z = 0.0f, acc[PER];
#pragma unroll
  for (int i = 0; i < PER; i++) acc[i] = 0.0f;
  while (jb < j1) {  // two keys of this warp per step, loaded before the step
#pragma unroll
    for (int u = 0; u < 2; u++)
      if (own && jb + u * kCW == nkv)
#pragma unroll
        for (int i = 0; i < PER; i++) kr[u][i] = kn[i], vr[u][i] = vn[i];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      if (jb + u * kCW >= j1) break;
      float sv = 0.0f;
#pragma unroll
      for (int i = 0; i < PER; i++) sv += q[i] * kr[u][i];
      sv = warp_sum(sv) * a.scale;
      const float mn = fmaxf(m, sv), c = expf(m - mn), e = expf(sv - mn);
      z = z * c + e;
#pragma unroll
      for (int i = 0; i < PER; i++) acc[i] = acc[i] * c + e * vr[u][i];
      m = mn;
    }
    jb += 2 * kCW;
    if (jb < j1) load_keys<PER>(Kh, Vh, jb, j1, lane, kr, vr);
  }
  float *rows = y, *wm = y + kCW * dk, *wz = wm + kCW;
#pragma unroll
  for (int i = 0; i < PER; i++) rows[wp * dk + lane + 32 * i] = acc[i];
  if (lane == 0) {
    wm[wp] = m;
    wz[wp] = z;
  }
  cbar();
  float M = -3.0e38f;
#pragma unroll
  for (int w = 0; w < kCW; w++) M = fmaxf(M, wm[w]);
  if (t < dk) {
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kCW; w++) o += rows[w * dk + t] * expf(wm[w] - M);
    ll_putf(a.po + ((size_t)h * Sg + sp) * dk + t, o, ep);
  }
  if (t == 0) {
    float Z = 0.0f;
#pragma unroll
    for (int w = 0; w < kCW; w++) Z += wz[w] * expf(wm[w] - M);
    ll_putf(a.pm + h * Sg + sp, M, ep);
    ll_putf(a.pz + h * Sg + sp, Z, ep);
  }
  cbar();  // the scratch is free for the next item
}

// Head h's S chunks merged into ao (rescaled to the running max, eight chunks' polls in flight) and the
// head's max |ao|. Every thread of the CTA calls it (the max is a CTA reduction); threads d < dk merge.
template <int PER>
__device__ void merge_head(const FusedArgs &a, int h, int S, float *red, uint32_t ep) {
  constexpr int dk = 32 * PER;
  const int t = threadIdx.x, Sg = a.Sg;
  float om = 0.0f;
  if (t < dk) {
    float Mh = -3.0e38f, Z = 0.0f, o = 0.0f;
    for (int i0 = 0; i0 < S; i0 += 8) {
      // the chunk maxima first (they are what is awaited); the sums and V rows, written with them, in one
      // round after (polled together before the maxima land, every word would be re-polled in turn)
      uint32_t vm[8], vz[8], vo[8];
      ll_get_n<8>(a.pm + h * Sg, i0, 1, S, ep, vm);
      uint64_t wz[8], wo[8];
      ll_issue<8>(a.pz + h * Sg, i0, 1, S, ep, wz);
      ll_issue<8>(a.po + (size_t)h * Sg * dk + t, i0 * dk, dk, S * dk, ep, wo);
      ll_finish<8>(a.pz + h * Sg, i0, 1, ep, wz, vz);
      ll_finish<8>(a.po + (size_t)h * Sg * dk + t, i0 * dk, dk, ep, wo, vo);
      float mb = Mh;
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (i0 + u < S) mb = fmaxf(mb, __uint_as_float(vm[u]));
      const float c = expf(Mh - mb);
      Z *= c;
      o *= c;
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (i0 + u < S) {
          const float w = expf(__uint_as_float(vm[u]) - mb);
          Z += __uint_as_float(vz[u]) * w;
          o += __uint_as_float(vo[u]) * w;
        }
      Mh = mb;
    }
    o /= Z;
    ll_putf(a.ao + h * dk + t, o, ep);
    om = fabsf(o);
  }
  om = c_max(om, red);
  if (t == 0) ll_putf(a.amax + h, om, ep);
  arrive(a.sync + 0);
}

// ---- the kernel ------------------------------------------------------------------------------------
template <int FMT, int PER>
__global__ void __launch_bounds__(kFThreads, 1) layer_fused_kernel(const __grid_constant__ FusedArgs a, Nf4Tables tb) {
  constexpr int dk = 32 * PER;
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[kMaxSlots], empty[kMaxSlots];
  __shared__ float red[32];
  __shared__ Plan plan;
  __shared__ PhaseGeo geo[4];
  __shared__ __align__(16) FusedLayerW slw[2];
  const int G = gridDim.x;
  const uint32_t ring = su32(sm), full0 = su32(full), empty0 = su32(empty);
  if (threadIdx.x == 0) {
    for (int s = 0; s < a.nslots; s++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(empty0 + 8 * s));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int p = 0; p < 4; p++) phase_geo<FMT>(a, p, G, geo[p]);
  }
  __syncthreads();
  if (threadIdx.x >= kCT) {  // the producer warp: one lane streams, the others are done
    if (threadIdx.x == kCT) produce<FMT>(a, ring, full0, empty0, G);
    return;
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int t = threadIdx.x;
  if (a.lw) {
    lw_fetch(&slw[0], a.lw, t);
    if (a.nl > 1) lw_fetch(&slw[1], a.lw + 1, t);
    lw_landed(t);
  } else if (t < kLwWords) {
    reinterpret_cast<uint64_t *>(&slw[0])[t] = reinterpret_cast<const uint64_t *>(&a.lw0)[t];
  }
  cbar();
  const int D = a.D, F = a.F, Nq = a.H * dk;
  const uint32_t ep0 = *(volatile unsigned int *)a.epoch + 1u;  // the first layer's tag; layer l: ep0 + l
  const uint32_t a8 = ring + a.off_a8;
  int8_t *a8p = reinterpret_cast<int8_t *>(sm + a.off_a8);
  float *xs = reinterpret_cast<float *>(sm + a.off_x);  // x, ao, then x1 (kept to the end of the layer)
  float *ys = reinterpret_cast<float *>(sm + a.off_y);  // norm gains / attention scratch / h
  int *loc = reinterpret_cast<int *>(sm + a.off_loc);   // this CTA's gate and up results
  Cursor kc = {0u, 0u};
  const bool ext = a.ext != 0;
  const int pos = a.dpos ? *a.dpos : a.pos;
  const int nkv = a.dpos ? *a.dpos : a.nkv;
  const int nk = ext ? nkv + 1 : nkv;
  const int Sg = a.Sg;
  const int kpc = max(32, (nk + 32 * Sg - 1) / (32 * Sg) * 32);
  const bool bad = nk < 1 || kpc > a.kpc || nkv > a.hstride || (ext && nkv >= a.hstride);
  const int S = bad ? 1 : (nk + kpc - 1) / kpc;
  if (bad && blockIdx.x == 0 && t == 0) { atomicOr(&g_fused_error, 4u); err_word_set(); }
  int f0, f1;
  share(F, blockIdx.x, G, f0, f1);
  const int nf = f1 - f0;

  for (int l = 0; l < a.nl; l++) {
    const FusedLayerW &lw = slw[l & 1];
    const uint32_t ep = ep0 + (uint32_t)l;
    const bool first = l == 0, last = l == a.nl - 1;
    // the next layer's table into the other copy (layer l - 1, its last user, is done in every thread)
    if (!first && l + 1 < a.nl) lw_fetch(&slw[(l + 1) & 1], a.lw + l + 1, t);
    if (t == 0) {  // phase A's plan
      plan.C[0] = a.q, plan.C[1] = a.k, plan.C[2] = a.v;
    }

    // ---- A: RMSNorm + quant of x (the previous layer's output after its hand-off); q, k, v ----
    if (!first) await_count(a.sync + 4, (unsigned int)(l * G));
    float ss = 0.0f;
    for (int i0 = t; i0 < D; i0 += kLB * kCT) {  // kLB elements per thread in flight: loads, then stores
      float v[kLB], g[kLB];
      if (first) {
#pragma unroll
        for (int u = 0; u < kLB; u++) v[u] = i0 + u * kCT < D ? a.x[i0 + u * kCT] : 0.0f;
      } else {
        uint32_t w[kLB];
        ll_get_n<kLB>(a.xl, i0, kCT, D, ep - 1u, w);
#pragma unroll
        for (int u = 0; u < kLB; u++) v[u] = __uint_as_float(w[u]);
      }
#pragma unroll
      for (int u = 0; u < kLB; u++) g[u] = i0 + u * kCT < D ? lw.attn_norm[i0 + u * kCT] : 0.0f;
#pragma unroll
      for (int u = 0; u < kLB; u++) {
        const int i = i0 + u * kCT;
        if (i < D) {
          xs[i] = v[u];
          ys[i] = g[u];
          ss += v[u] * v[u];
        }
      }
    }
    ss = c_sum(ss, red);
    float r = glue::rms_recip(ss, D);
    float mx = 1e-6f;
    for (int i = t; i < D; i += kCT) mx = fmaxf(mx, fabsf(xs[i] * r * ys[i]));
    mx = c_max(mx, red);
    const float sx = glue::qscale(mx);
    for (int i = t; i < D; i += kCT) a8p[i] = q8(xs[i] * r * ys[i], sx);
    cbar();
    kc = consume<FMT>(a, geo[0], plan, 0, kc, ring, full0, empty0, a8, tb, ep);

    // ---- B: attention items, then the merge of head h by CTA h ----
    if (bad) {  // no attention: ao is zero (the error is reported), so the phases after still complete
      for (int h = blockIdx.x; h < a.H; h += G) {
        for (int d = t; d < dk; d += kCT) ll_putf(a.ao + h * dk + d, 0.0f, ep);
        if (t == 0) ll_putf(a.amax + h, 0.0f, ep);
        arrive(a.sync + 0);
      }
    } else {
      for (int it = blockIdx.x; it < a.H * S; it += G)
        attend<PER>(a, lw, it % a.H, it / a.H, kpc, nkv, nk, pos, sx, ys, ep);
      for (int h = blockIdx.x; h < a.H; h += G) merge_head<PER>(a, h, S, red, ep);
    }

    // ---- C: ao and the head maxima, quantization; o ----
    await_count(a.sync + 0, (unsigned int)((l + 1) * a.H));
    float om = 0.0f;
    for (int e0 = t; e0 < Nq || e0 < a.H; e0 += kLB * kCT) {  // the head maxima and ao: one round
      uint64_t wm[kLB], wo[kLB];
      uint32_t vm[kLB], vo[kLB];
      ll_issue<kLB>(a.amax, e0, kCT, a.H, ep, wm);
      ll_issue<kLB>(a.ao, e0, kCT, Nq, ep, wo);
      ll_finish<kLB>(a.amax, e0, kCT, ep, wm, vm);
      ll_finish<kLB>(a.ao, e0, kCT, ep, wo, vo);
#pragma unroll
      for (int u = 0; u < kLB; u++) {
        if (e0 + u * kCT < a.H) om = fmaxf(om, __uint_as_float(vm[u]));
        if (e0 + u * kCT < Nq) xs[e0 + u * kCT] = __uint_as_float(vo[u]);
      }
    }
    om = c_max(om, red);
    const float sa = glue::qscale(om);
    for (int e = t; e < Nq; e += kCT) a8p[e] = q8(xs[e], sa);
    if (t == 0) {
      plan.C[0] = a.o;
    }
    cbar();
    kc = consume<FMT>(a, geo[1], plan, 1, kc, ring, full0, empty0, a8, tb, ep);
    arrive(a.sync + 1);

    // ---- D: x1 = x + Co / sa, RMSNorm + quant; gate and up; SwiGLU ----
    await_count(a.sync + 1, (unsigned int)((l + 1) * G));
    ss = 0.0f;
    for (int i0 = t; i0 < D; i0 += kLB * kCT) {  // gains, x and Co: one round
      float v[kLB], g[kLB];
      uint32_t c[kLB];
#pragma unroll
      for (int u = 0; u < kLB; u++) g[u] = i0 + u * kCT < D ? lw.ffn_norm[i0 + u * kCT] : 0.0f;
      uint64_t wx[kLB], wo[kLB];
      if (!first) ll_issue<kLB>(a.xl, i0, kCT, D, ep - 1u, wx);
      ll_issue<kLB>(a.o, i0, kCT, D, ep, wo);
      if (first) {
#pragma unroll
        for (int u = 0; u < kLB; u++) v[u] = i0 + u * kCT < D ? a.x[i0 + u * kCT] : 0.0f;
      } else {
        uint32_t w[kLB];
        ll_finish<kLB>(a.xl, i0, kCT, ep - 1u, wx, w);
#pragma unroll
        for (int u = 0; u < kLB; u++) v[u] = __uint_as_float(w[u]);
      }
      ll_finish<kLB>(a.o, i0, kCT, ep, wo, c);
#pragma unroll
      for (int u = 0; u < kLB; u++) {
        const int i = i0 + u * kCT;
        if (i < D) {
          const float x1 = v[u] + (int32_t)c[u] / sa;
          xs[i] = x1;
          ys[i] = g[u];
          ss += x1 * x1;
        }
      }
    }
    ss = c_sum(ss, red);
    r = glue::rms_recip(ss, D);
    mx = 1e-6f;
    for (int i = t; i < D; i += kCT) mx = fmaxf(mx, fabsf(xs[i] * r * ys[i]));
    mx = c_max(mx, red);
    const float sf = glue::qscale(mx);
    for (int i = t; i < D; i += kCT) a8p[i] = q8(xs[i] * r * ys[i], sf);
    if (t == 0) {
      plan.loc = loc, plan.f0 = f0, plan.nf = nf;
    }
    cbar();
    kc = consume<FMT>(a, geo[2], plan, 2, kc, ring, full0, empty0, a8, tb, ep);
    cbar();
    float hm = 0.0f;
    for (int i = t; i < nf; i += kCT) {
      const float hv = glue::silu_mul(loc[i] / sf, loc[nf + i] / sf);
      ll_putf(a.h + f0 + i, hv, ep);
      hm = fmaxf(hm, fabsf(hv));
    }
    hm = c_max(hm, red);
    if (t == 0) ll_putf(a.hmax + blockIdx.x, hm, ep);
    arrive(a.sync + 2);

    // ---- E: quantization of h; down with the residual -> the next layer's x (or x_out) ----
    await_count(a.sync + 2, (unsigned int)((l + 1) * G));
    hm = 0.0f;
    for (int i0 = t; i0 < F || i0 < G; i0 += kHB * kCT) {  // the CTA maxima and h: one round
      uint64_t wm[2], wh[kHB];
      uint32_t vm[2], vh[kHB];
      ll_issue<2>(a.hmax, i0, kCT, G, ep, wm);
      ll_issue<kHB>(a.h, i0, kCT, F, ep, wh);
      ll_finish<2>(a.hmax, i0, kCT, ep, wm, vm);
      ll_finish<kHB>(a.h, i0, kCT, ep, wh, vh);
#pragma unroll
      for (int u = 0; u < 2; u++)
        if (i0 + u * kCT < G) hm = fmaxf(hm, __uint_as_float(vm[u]));
#pragma unroll
      for (int u = 0; u < kHB; u++)
        if (i0 + u * kCT < F) ys[i0 + u * kCT] = __uint_as_float(vh[u]);
    }
    hm = c_max(hm, red);
    const float sc = glue::qscale(hm);
    for (int i = t; i < F; i += kCT) a8p[i] = q8(ys[i], sc);
    if (t == 0) {
      plan.out = last ? a.x_out : nullptr, plan.xl = last ? nullptr : a.xl, plan.x1 = xs, plan.s = sc;
    }
    cbar();
    kc = consume<FMT>(a, geo[3], plan, 3, kc, ring, full0, empty0, a8, tb, ep);
    lw_landed(t);  // the next layer's table (long landed); the arrival's barrier publishes it
    if (!last) arrive(a.sync + 4);
  }

  // the last CTA to finish clears the counts and records the last layer's tag for the next launch
  cbar();
  if (t == 0 && atomicAdd(a.sync + 3, 1u) == (unsigned int)G - 1) {
#pragma unroll
    for (int i = 0; i < 5; i++) a.sync[i] = 0u;
    *(volatile unsigned int *)a.epoch = ep0 + (uint32_t)a.nl - 1u;
  }
}

template <int FMT, int PER>
cudaError_t launch_one(const FusedArgs &a, int G, cudaStream_t s) {
  auto kern = layer_fused_kernel<FMT, PER>;
  {
    const cudaError_t e = smem_attr((const void *)kern, kSmemMax);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = a.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident at once: the grid barriers need it
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a, nf4_tables());
}

template <int FMT>
cudaError_t launch_fmt(const FusedArgs &a, int G, cudaStream_t s) {
  switch (a.dk) {
    case 64: return launch_one<FMT, 2>(a, G, s);
    case 128: return launch_one<FMT, 4>(a, G, s);
    case 256: return launch_one<FMT, 8>(a, G, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int fused_grid(int device) {
  static int sms[64] = {};
  if (device < 0 || device >= 64) return 0;
  if (!sms[device] && cudaDeviceGetAttribute(&sms[device], cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
    sms[device] = 0;
  return sms[device];
}

int fused_splits(int H, int maxk, int G) {
  return std::max(1, std::min({kFMaxSplit, std::max(1, G / H), (maxk + 31) / 32}));
}

int fused_kpc(int maxk, int Sg) { return std::max(32, (maxk + 32 * Sg - 1) / (32 * Sg) * 32); }

// Shared memory: the ring at offset 0, then the activation row (int8, the longest of D, H*dk, F), x / ao /
// x1 (floats), the scratch (norm gains, an attention item's warp rows, h), this CTA's gate and up
// results. Slots hold a whole number of rows of every weight: a multiple of the longest row, about
// 12 KB.
bool fused_plan(FusedArgs *a, int fmt, int G) {
  if (fmt != FMT_I8 && fmt != FMT_U4 && fmt != FMT_NF4) return false;
  if ((a->dk != 64 && a->dk != 128 && a->dk != 256) || G < 1 || a->Sg > kFMaxSplit) return false;
  auto up = [](size_t x) { return (x + 127) & ~(size_t)127; };
  const int Nq = a->H * a->dk;
  const int Ks[3] = {a->D, Nq, a->F};
  size_t maxrow = 0;
  for (int K : Ks) {
    const size_t rb = fmt == FMT_I8 ? (size_t)K : (size_t)K / 2;
    if (rb % 16 || (fmt != FMT_I8 && K % 32)) return false;
    maxrow = std::max(maxrow, rb);
  }
  const size_t a8 = up((size_t)std::max({a->D, Nq, a->F}));
  const size_t xs = up((size_t)std::max(a->D, Nq) * 4);
  const size_t ys = up((size_t)std::max({a->D, a->F, kCW * a->dk + 2 * kCW}) * 4);
  const size_t loc = up((size_t)2 * ((a->F + G - 1) / G + 1) * 4);
  const size_t slot = up(maxrow * std::max<size_t>(1, 12288 / maxrow));
  const size_t fixed = a8 + xs + ys + loc;
  if (fixed + 2 * slot > (size_t)kSmemMax) return false;
  const int ns = (int)std::min<size_t>(kMaxSlots, (kSmemMax - fixed) / slot);
  a->slot = (uint32_t)slot;
  a->nslots = ns;
  a->off_a8 = (uint32_t)(slot * ns);
  a->off_x = a->off_a8 + (uint32_t)a8;
  a->off_y = a->off_x + (uint32_t)xs;
  a->off_loc = a->off_y + (uint32_t)ys;
  a->smem = a->off_loc + (uint32_t)loc;
  return true;
}

cudaError_t launch_layer_fused(const FusedArgs &a, int fmt, int G, cudaStream_t s) {
  switch (fmt) {
    case FMT_I8: return launch_fmt<FMT_I8>(a, G, s);
    case FMT_U4: return launch_fmt<FMT_U4>(a, G, s);
    case FMT_NF4: return launch_fmt<FMT_NF4>(a, G, s);
    default: return cudaErrorInvalidValue;
  }
}

unsigned int fused_error_flag(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_fused_error, sizeof v);
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_fused_error, &z, sizeof z);
  }
  return v;
}

ORKB_ERR_WORD_SETTER(fused_set_err_word)

}  // namespace orkb
