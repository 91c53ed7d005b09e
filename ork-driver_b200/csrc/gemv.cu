// gemv.cu -- decode-path matmul (M <= 8 rows of activations per launch) on CUDA cores, sm_100a.
//
// C[m][n] = sum_k A[m][k] * B[k][n] with the weight resident K-major (one output channel per row, see
// ork_internal.h). The path is HBM-bound: every weight byte is read exactly once per launch.
//
// Staging: a CTA owns TR consecutive output channels, i.e. one contiguous TR x rowB block of the
// resident weight. At kernel start a single thread requests the whole block with bulk asynchronous
// copies (cp.async.bulk, the TMA engine's 1-D form), one per group of 8 channels, each completing on its
// own mbarrier -- so every byte a CTA will ever read is in flight immediately, with no register cost,
// and a warp starts computing as soon as its 8 channels have landed. The copies are issued before
// griddepcontrol.wait, so under programmatic dependent launch the weight stream of the next matmul
// overlaps the tail of the previous one; activations are read only after the wait.
//
// Arithmetic, in registers:
//   int8  : 4 x dp4a per 16 weight bytes and activation row;
//   int4  : each 16-byte chunk of nibbles (32 k) is expanded once to its int8 codes (expand8,
//           nibble.cuh: sign-extended uniform codes, or the NF4 table through prmt) and then multiplied
//           with dp4a like int8 -- the expansion is shared by all MT activation rows;
//   fp16  : converted to fp32 and accumulated with FFMA.
// Every integer result is exact int32, identical to ork-driver's CPU oracle (src/npu/core/buf.c:428).
//
// A second, direct-load kernel (gemv_direct_kernel) serves the shapes where staging whole rows per CTA
// does not pay: a warp streams its CPW channel rows through a register ring of 128-bit loads and reads
// the activations through L1 (see choose() for where each kernel is used).
//
// Work mapping (staged kernel): eight lanes cover one channel, 16 bytes each, so one warp-wide shared-memory read moves
// 4 channels x 128 contiguous bytes and the activation chunk it multiplies is shared by the 4 channel
// groups; each lane holds R = 2 channels (8 per warp) to reuse every activation load twice. The WK warps
// that share a channel group split K; partials are reduced with a butterfly shuffle across the 8 lanes,
// then across the K-split warps in shared memory.
#include <cuda_fp16.h>

#include <cstdlib>

#include <type_traits>

#include "nibble.cuh"
#include "errword.cuh"
#include "ork_internal.h"
#include "requant.cuh"

namespace orkb {

namespace {

constexpr int kR = 2;        // channels per lane
constexpr int kWarps = 4;    // warps per CTA
constexpr uint64_t kWaitCycles = 4000000000ull;

__device__ unsigned int g_gemv_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// Bounded mbarrier wait (parity 0: each barrier completes exactly once per launch).
__device__ __forceinline__ bool mbar_wait0(uint32_t bar) {
  const uint64_t t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kWaitCycles) {
      { atomicOr(&g_gemv_error, 1u); err_word_set(); }
      return false;
    }
  }
}

template <int FMT> struct Acc { using T = int; };
template <> struct Acc<FMT_F16> { using T = float; };

// Butterfly reduction of V values across the 8 lanes that share (lane >> 3): a halving step trades half
// of the values with the partner lane, so 8 lanes reduce V values with V-1 shuffles instead of 3V.
template <int NV, int OFF, typename T>
__device__ __forceinline__ void bfly_step(T *v, int lane) {
  if constexpr (NV > 1) {
    constexpr int H = NV / 2;
    const bool up = (lane & OFF) != 0;
#pragma unroll
    for (int i = 0; i < H; i++) {
      T send = up ? v[i] : v[i + H];
      T keep = up ? v[i + H] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
    }
  } else {
    v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
  }
}

using Tables = Nf4Tables;

// acc[r*MT+m] += <activation chunk of row m, weight chunk of channel r> for one 16-byte weight chunk per
// channel. `sa` is the shared-memory address of activation row 0 at the chunk's first k, `a_row` the
// activation row pitch in bytes.
template <int FMT, int MT, typename T>
__device__ __forceinline__ void mac_chunk(const uint4 (&wv)[kR], uint32_t sa, uint32_t a_row, int M, T *acc,
                                          const Tables &tb) {
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  uint32_t wx[NIB ? kR : 1][8];  // nibble chunks expanded once to int8 codes in k order
  if constexpr (NIB) {
#pragma unroll
    for (int r = 0; r < kR; r++) {
      const uint32_t ww[4] = {wv[r].x, wv[r].y, wv[r].z, wv[r].w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint2 e = expand8<FMT>(ww[q], tb);
        wx[r][2 * q] = e.x;
        wx[r][2 * q + 1] = e.y;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; m++) {
    if (m >= M) break;
    const uint32_t arow = sa + (uint32_t)m * a_row;
    if constexpr (FMT == FMT_I8) {
      const uint4 a = lds128(arow);
#pragma unroll
      for (int r = 0; r < kR; r++) {
        T &c = acc[r * MT + m];
        c = dp4a(a.x, wv[r].x, c);
        c = dp4a(a.y, wv[r].y, c);
        c = dp4a(a.z, wv[r].z, c);
        c = dp4a(a.w, wv[r].w, c);
      }
    } else if constexpr (FMT == FMT_U4 || FMT == FMT_NF4) {
      const uint4 a0 = lds128(arow), a1 = lds128(arow + 16);  // 32 activations, k order
      const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int r = 0; r < kR; r++) {
        T &c = acc[r * MT + m];
#pragma unroll
        for (int q = 0; q < 8; q++) c = dp4a(aw[q], wx[r][q], c);
      }
    } else {  // FMT_F16
      const uint4 a = lds128(arow);
      const __half2 *ah = reinterpret_cast<const __half2 *>(&a);
      float2 af[4];
#pragma unroll
      for (int q = 0; q < 4; q++) af[q] = __half22float2(ah[q]);
#pragma unroll
      for (int r = 0; r < kR; r++) {
        const __half2 *wh = reinterpret_cast<const __half2 *>(&wv[r]);
        T &c = acc[r * MT + m];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float2 wf = __half22float2(wh[q]);
          c = fmaf(af[q].x, wf.x, c);
          c = fmaf(af[q].y, wf.y, c);
        }
      }
    }
  }
}

// TR channels per CTA (8 per warp-row group), WK = 4 / (TR / 8) warps split K.
// One CTA's work of the staged kernel: channels [n0, n0 + TR) of the weight at W (N channels of K), the
// activations A (M rows), C rows at a stride of cstride elements.
// One result to C: the raw sum, or for int8-compute formats the requantized output stage.
template <typename T>
__device__ __forceinline__ void store_out(void *C, const OutStage &os, size_t idx, T v) {
  if constexpr (std::is_floating_point<T>::value) {  // fp16 weights: fp32 sums, no output stage
    reinterpret_cast<float *>(C)[idx] = v;
  } else {
    if (os.mode == OUT_I32) {
      reinterpret_cast<int32_t *>(C)[idx] = v;
      return;
    }
    int64_t p = (int64_t)v * os.mult;
    if (os.mode == OUT_EWMUL) p *= os.G[idx];
    const int64_t q = requant_rne(p, os.shift);
    if (os.mode == OUT_I16)
      reinterpret_cast<int16_t *>(C)[idx] = (int16_t)(q > 32767 ? 32767 : q < -32768 ? -32768 : q);
    else
      reinterpret_cast<int8_t *>(C)[idx] = (int8_t)(q > 127 ? 127 : q < -128 ? -128 : q);
  }
}

template <int FMT, int MT, int TR, int NW = kWarps, int P = 2>
__device__ __forceinline__ void gemv_block(const uint8_t *__restrict__ W, const uint8_t *__restrict__ A,
                                           void *__restrict__ Cout, int M, int K, int N, int n0, int cstride,
                                           const Tables &tb, const OutStage &os) {
  using T = typename Acc<FMT>::T;
  constexpr int WR = TR / (4 * kR);  // warp-row groups
  constexpr int WK = NW / WR;        // warps splitting K
  static_assert(WK >= 1 && NW % WR == 0, "whole warp-row groups");
  constexpr int V = kR * MT;
  constexpr int NGRP = TR / 8;       // 8-channel copy groups (one mbarrier each)
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[NGRP + 1];  // one per 8-channel weight group, then activations
  __shared__ T red[WK > 1 ? WK : 1][TR][MT];

  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 3, j = lane & 7;
  const int wr = warp / WK, wk = warp % WK;
  const int rows = min(TR, N - n0);
  const size_t rowB = (FMT == FMT_F16) ? (size_t)K * 2 : (FMT == FMT_I8) ? (size_t)K : (size_t)K / 2;
  const size_t a_row = (FMT == FMT_F16) ? (size_t)K * 2 : (size_t)K;
  const uint32_t sW = smem_u32(smem);

  if (threadIdx.x == 0) {
    for (int q = 0; q <= NGRP; q++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[q])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint8_t *src = W + (size_t)n0 * rowB;
    for (int q = 0; q < NGRP; q++) {
      const int r0 = q * 8, nr = min(8, rows - r0);
      const uint32_t bar = smem_u32(&bars[q]);
      const uint32_t bytes = nr > 0 ? (uint32_t)(nr * rowB) : 0u;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
      if (nr > 0)
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         sW + (uint32_t)(r0 * rowB)),
                     "l"(src + (size_t)r0 * rowB), "r"(bytes), "r"(bar)
                     : "memory");
    }
  }
  // The activations are read only after the wait (the previous kernel may write them); an L2 prefetch
  // of them before it has no effect on the values read and saves the HBM latency when they are cold (a
  // prefetch is a hint: the copy after the wait reads the current data through L2 either way). One CTA
  // in eight asks.
  if (threadIdx.x == 0 && (blockIdx.x & 7) == 0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(A), "r"((uint32_t)(M * a_row)) : "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the activations (written by the previous kernel) come after the wait: one copy of the M x K block
  const uint32_t sA = sW + (uint32_t)(TR * rowB);
  if (threadIdx.x == 0) {
    const uint32_t bar = smem_u32(&bars[NGRP]), bytes = (uint32_t)(M * a_row);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sA),
                 "l"(A), "r"(bytes), "r"(bar)
                 : "memory");
  }
  __syncthreads();  // barrier init visible to every thread

  T acc[V];
#pragma unroll
  for (int i = 0; i < V; i++) acc[i] = T(0);

  // this lane's channels: local rows wr*8 + g + 4r, r < kR (the warp-row group is one copy group)
  const int lrow0 = wr * 8 + g;
  const int S = (int)((rowB + 127) / 128);
  const uint32_t base0 = sW + (uint32_t)(lrow0 * rowB) + (uint32_t)(j * 16);
  const uint32_t a_k = (FMT == FMT_U4 || FMT == FMT_NF4) ? 2u : 1u;  // activation bytes per weight byte
  // The weights land long before the activations (they were requested before the dependency wait), so
  // the warp's first P chunks per lane move from shared memory into registers while the activations are
  // still in flight: after they land only the multiply-adds remain (the shared-memory read of a CTA's
  // weight block is a second pass over every weight byte, which would otherwise start only then). P is
  // sized to the chunks a warp actually has (its registers bound how many CTAs, this launch's and the
  // next one's, share an SM).
  uint4 pre[P][kR];
  const bool live = wr * 8 < rows;
  const bool okw = mbar_wait0(smem_u32(&bars[wr]));
  if (okw && live) {
#pragma unroll
    for (int p = 0; p < P; p++) {
      const int s = wk + p * WK;
      if ((uint32_t)s * 128u + (uint32_t)j * 16u < rowB) {
#pragma unroll
        for (int r = 0; r < kR; r++) pre[p][r] = lds128(base0 + (uint32_t)(4 * r * rowB) + (uint32_t)(s * 128));
      }
    }
  }
  const bool ok = okw && mbar_wait0(smem_u32(&bars[NGRP]));
  if (ok && live) {
#pragma unroll
    for (int p = 0; p < P; p++) {
      const uint32_t o = (uint32_t)(wk + p * WK) * 128u + (uint32_t)j * 16u;
      if (o < rowB) mac_chunk<FMT, MT, T>(pre[p], sA + a_k * o, (uint32_t)a_row, M, acc, tb);
    }
#pragma unroll 4
    for (int s = wk + P * WK; s < S; s += WK) {
      const uint32_t o = (uint32_t)s * 128u + (uint32_t)j * 16u;
      if (o >= rowB) break;
      uint4 wv[kR];
#pragma unroll
      for (int r = 0; r < kR; r++) wv[r] = lds128(base0 + (uint32_t)(4 * r * rowB) + (uint32_t)(s * 128));
      mac_chunk<FMT, MT, T>(wv, sA + a_k * o, (uint32_t)a_row, M, acc, tb);
    }
  }

  bfly_step<V, 4>(acc, lane);
  bfly_step<(V / 2 > 1 ? V / 2 : 1), 2>(acc, lane);
  bfly_step<(V / 4 > 1 ? V / 4 : 1), 1>(acc, lane);
  constexpr int HELD = V >= 8 ? V / 8 : 1;
  int base = 0;
  if (V >= 2 && (j & 4)) base += V / 2;
  if (V >= 4 && (j & 2)) base += V / 4;
  if (V >= 8 && (j & 1)) base += V / 8;
  const bool writer = (V >= 8) || (V == 4 && !(j & 1)) || (V == 2 && !(j & 3)) || (V == 1 && j == 0);

  if constexpr (WK == 1) {
    if (writer) {
#pragma unroll
      for (int i = 0; i < HELD; i++) {
        const int idx = base + i, r = idx / MT, m = idx % MT;
        const int lr = lrow0 + 4 * r;
        if (m < M && lr < rows) store_out<T>(Cout, os, (size_t)m * cstride + n0 + lr, acc[i]);
      }
    }
  } else {
    if (writer) {
#pragma unroll
      for (int i = 0; i < HELD; i++) {
        const int idx = base + i, r = idx / MT, m = idx % MT;
        red[wk][lrow0 + 4 * r][m] = acc[i];
      }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < TR * MT; t += NW * 32) {
      const int m = t / TR, lr = t % TR;
      if (m < M && lr < rows) {
        T s = red[0][lr][m];
#pragma unroll
        for (int q = 1; q < WK; q++) s += red[q][lr][m];
        store_out<T>(Cout, os, (size_t)m * cstride + n0 + lr, s);
      }
    }
  }
}

template <int FMT, int MT, int TR, int NW, int P>
__global__ void __launch_bounds__(NW * 32)
gemv_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ A, void *__restrict__ Cout, int M, int K,
            int N, Tables tb) {
  gemv_block<FMT, MT, TR, NW, P>(W, A, Cout, M, K, N, (int)blockIdx.x * TR, N, tb, OutStage{});
}

// Batched (chain / MoE) variant: many independent matmuls of one weight format in one launch. Task t
// owns CTAs [block0[t], block0[t + 1]); each CTA finds its task by binary search and runs the staged
// kernel's block for it. The task table travels as a kernel parameter.
constexpr int kMaxBatch = 96;
struct BatchTask {
  const uint8_t *W;
  const uint8_t *A;
  void *C;
  int M, K, N, cstride, block0;
  OutStage os;
};
struct BatchTable {
  BatchTask t[kMaxBatch];
  int n;
};

template <int FMT, int MT, int TR>
__global__ void __launch_bounds__(kWarps * 32) gemv_batched_kernel(const __grid_constant__ BatchTable bt, Tables tb) {
  int lo = 0, hi = bt.n - 1;
  const int b = (int)blockIdx.x;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (bt.t[mid].block0 <= b) lo = mid;
    else hi = mid - 1;
  }
  const BatchTask &t = bt.t[lo];
  gemv_block<FMT, MT, TR>(t.W, t.A, t.C, t.M, t.K, t.N, (b - t.block0) * TR, t.cstride, tb, t.os);
}

// Grouped variant (per-K-group scales): same staging and arithmetic as gemv_kernel, but each warp walks
// a contiguous range of 128-byte weight segments and flushes its lane partials into a shared-memory
// table P[group][channel][row] with integer atomics whenever the lane's chunk moves into the next K
// group -- exact int32 per group whatever the lane order. After a block barrier one thread per
// (channel, row) combines the groups in ascending order in fp32 with explicitly rounded multiplies and
// adds (no contraction), the arithmetic of ork-driver's orki_cpu_gemm_grouped (src/npu/core/buf.c:
// 501-520): c = 0; for g: c += ((float)P_g * aScale[m][g]) * bScale[g][n].
template <int FMT, int MT, int TR>
__global__ void __launch_bounds__(kWarps * 32)
gemv_grouped_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ A, const float *__restrict__ aS,
                    const float *__restrict__ bS, float *__restrict__ C, int M, int K, int N, int G, Tables tb) {
  static_assert(FMT != FMT_F16, "grouped scales apply to integer weights");
  constexpr int WR = TR / (4 * kR);
  constexpr int WK = kWarps / WR;
  constexpr int V = kR * MT;
  constexpr int NGRP = TR / 8;
  constexpr int KPB = (FMT == FMT_I8) ? 1 : 2;  // k values per weight byte
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[NGRP + 1];

  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gq = lane >> 3, j = lane & 7;
  const int wr = warp / WK, wk = warp % WK;
  const int n0 = blockIdx.x * TR;
  const int rows = min(TR, N - n0);
  const size_t rowB = (size_t)K / KPB;
  const size_t a_row = (size_t)K;
  const int Sk = K / G;
  const int gbytes = G / KPB;  // weight bytes per group (a multiple of the 16-byte lane chunk)
  const int share = gbytes % 128 == 0 ? 8 : (128 % gbytes == 0 ? gbytes / 16 : 1);
  const uint32_t sW = smem_u32(smem);
  const uint32_t sA = sW + (uint32_t)(TR * rowB);
  int *P = reinterpret_cast<int *>(smem + TR * rowB + ((M * a_row + 15) & ~(size_t)15));

  if (threadIdx.x == 0) {
    for (int q = 0; q <= NGRP; q++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&bars[q])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    const uint8_t *src = W + (size_t)n0 * rowB;
    for (int q = 0; q < NGRP; q++) {
      const int r0 = q * 8, nr = min(8, rows - r0);
      const uint32_t bar = smem_u32(&bars[q]);
      const uint32_t bytes = nr > 0 ? (uint32_t)(nr * rowB) : 0u;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
      if (nr > 0)
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         sW + (uint32_t)(r0 * rowB)),
                     "l"(src + (size_t)r0 * rowB), "r"(bytes), "r"(bar)
                     : "memory");
    }
  }
  for (int t = threadIdx.x; t < Sk * TR * MT; t += kWarps * 32) P[t] = 0;
  if (threadIdx.x == 0 && (blockIdx.x & 7) == 0)  // L2 prefetch of the activations (see gemv_block)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(A), "r"((uint32_t)(M * a_row)) : "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    const uint32_t bar = smem_u32(&bars[NGRP]), bytes = (uint32_t)(M * a_row);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(sA),
                 "l"(A), "r"(bytes), "r"(bar)
                 : "memory");
  }
  __syncthreads();  // barrier init and the zeroed table visible to every thread

  using T = int;
  T acc[V];
#pragma unroll
  for (int i = 0; i < V; i++) acc[i] = 0;

  const int lrow0 = wr * 8 + gq;
  // warp-uniform (the group flush below shuffles across the warp)
  const bool ok = __all_sync(0xffffffffu, mbar_wait0(smem_u32(&bars[wr])) && mbar_wait0(smem_u32(&bars[NGRP])));
  const int S = (int)((rowB + 127) / 128);
  const int s0 = (int)((long long)S * wk / WK), s1 = (int)((long long)S * (wk + 1) / WK);
  if (ok && wr * 8 < rows) {
    const uint32_t base0 = sW + (uint32_t)(lrow0 * rowB) + (uint32_t)(j * 16);
    const uint32_t a_k = (uint32_t)KPB;
    for (int s = s0; s < s1; s++) {
      const uint32_t o = (uint32_t)s * 128u + (uint32_t)j * 16u;
      const bool live = o < rowB;
      if (live) {
        uint4 wv[kR];
#pragma unroll
        for (int r = 0; r < kR; r++) wv[r] = lds128(base0 + (uint32_t)(4 * r * rowB) + (uint32_t)(s * 128));
        mac_chunk<FMT, MT, T>(wv, sA + a_k * o, (uint32_t)a_row, M, acc, tb);
      }
      // Flush the lane partials into P at the end of a group. When the lanes of a channel group share
      // groups in aligned power-of-two sets (share = 2, 4 or 8 lanes: a group of 32 or 64 bytes, or whole
      // 128-byte segments), the set is first reduced with xor-shuffles -- its flush points are the same
      // for the whole warp -- and one lane per set adds; otherwise every lane adds its own partial.
      const int grp = (int)(o / (uint32_t)gbytes);
      if (share > 1) {
        const bool last = share < 8 || (s + 1 >= s1) || (uint32_t)(s + 1) * 128u >= rowB ||
                          (int)((uint32_t)(s + 1) * 128u / (uint32_t)gbytes) != grp;
        if (last) {
#pragma unroll
          for (int r = 0; r < kR; r++) {
            const int lr = lrow0 + 4 * r;
#pragma unroll
            for (int m = 0; m < MT; m++) {
              T v = acc[r * MT + m];
              for (int off = 1; off < share; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
              if (live && (j & (share - 1)) == 0 && m < M && lr < rows && v != 0)
                atomicAdd(&P[(grp * TR + lr) * MT + m], v);
              acc[r * MT + m] = 0;
            }
          }
        }
      } else {
        const uint32_t on = o + 128u;
        const bool last = (s + 1 >= s1) || on >= rowB || (int)(on / (uint32_t)gbytes) != grp;
        if (live && last) {
#pragma unroll
          for (int r = 0; r < kR; r++) {
            const int lr = lrow0 + 4 * r;
#pragma unroll
            for (int m = 0; m < MT; m++) {
              const T v = acc[r * MT + m];
              if (m < M && lr < rows && v != 0) atomicAdd(&P[(grp * TR + lr) * MT + m], v);
              acc[r * MT + m] = 0;
            }
          }
        }
      }
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < TR * MT; t += kWarps * 32) {
    const int m = t / TR, lr = t % TR;
    if (m < M && lr < rows) {
      const int n = n0 + lr;
      float c = 0.0f;
      for (int g = 0; g < Sk; g++)
        c = __fadd_rn(c, __fmul_rn(__fmul_rn((float)P[(g * TR + lr) * MT + m], aS[(size_t)m * Sk + g]),
                                   bS[(size_t)g * N + n]));
      C[(size_t)m * N + n] = c;
    }
  }
}

// Direct-load decode kernel. One warp owns CPW consecutive output channels and their whole K row; lane
// l reads 16-byte chunks l, l+32, l+64, ... of every row (each warp load is 512 contiguous bytes) with
// 128-bit loads that bypass L1, keeping U chunks per channel in flight in a register ring -- the first U
// are issued before griddepcontrol.wait, so under programmatic launch they overlap the previous kernel.
// Activations come through the L1 read-only path (every warp of an SM reads the same M x K block).
// Partials are reduced across the 32 lanes with halving butterflies.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ldg_a(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Sum NV values (a power of two <= 32) over the 32 lanes: while more than one value is left, lanes OFF
// apart trade halves; afterwards lane l holds the total of value (l * NV) >> 5, and lanes l with
// l % (32 / NV) == 0 are the unique holders.
template <int NV, int OFF, typename T>
__device__ __forceinline__ void bfly32(T *v, int lane) {
  if constexpr (OFF >= 1) {
    if constexpr (NV > 1) {
      constexpr int H = NV / 2;
      const bool up = (lane & OFF) != 0;
#pragma unroll
      for (int i = 0; i < H; i++) {
        const T send = up ? v[i] : v[i + H];
        const T keep = up ? v[i + H] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, OFF);
      }
      bfly32<H, OFF / 2>(v, lane);
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], OFF);
      bfly32<1, OFF / 2>(v, lane);
    }
  }
}

// acc[r*MT+m] += <activation row m at k of chunk `ch`, weight chunk of channel r>, activations read from
// global memory (L1).
template <int FMT, int MT, int CPW, typename T>
__device__ __forceinline__ void mac_regs(const uint4 (&wv)[CPW], const uint8_t *__restrict__ a0, size_t a_row, int M,
                                         T *acc, const Tables &tb) {
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  uint32_t wx[NIB ? CPW : 1][8];
  if constexpr (NIB) {
#pragma unroll
    for (int r = 0; r < CPW; r++) {
      const uint32_t ww[4] = {wv[r].x, wv[r].y, wv[r].z, wv[r].w};
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint2 e = expand8<FMT>(ww[q], tb);
        wx[r][2 * q] = e.x;
        wx[r][2 * q + 1] = e.y;
      }
    }
  }
#pragma unroll
  for (int m = 0; m < MT; m++) {
    if (m >= M) break;
    const uint8_t *ar = a0 + (size_t)m * a_row;
    if constexpr (FMT == FMT_I8) {
      const uint4 a = ldg_a(ar);
#pragma unroll
      for (int r = 0; r < CPW; r++) {
        T &c = acc[r * MT + m];
        c = dp4a(a.x, wv[r].x, c);
        c = dp4a(a.y, wv[r].y, c);
        c = dp4a(a.z, wv[r].z, c);
        c = dp4a(a.w, wv[r].w, c);
      }
    } else if constexpr (NIB) {
      const uint4 x0 = ldg_a(ar), x1 = ldg_a(ar + 16);
      const uint32_t aw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
      for (int r = 0; r < CPW; r++) {
        T &c = acc[r * MT + m];
#pragma unroll
        for (int q = 0; q < 8; q++) c = dp4a(aw[q], wx[r][q], c);
      }
    } else {  // FMT_F16
      const uint4 a = ldg_a(ar);
      const __half2 *ah = reinterpret_cast<const __half2 *>(&a);
      float2 af[4];
#pragma unroll
      for (int q = 0; q < 4; q++) af[q] = __half22float2(ah[q]);
#pragma unroll
      for (int r = 0; r < CPW; r++) {
        const __half2 *wh = reinterpret_cast<const __half2 *>(&wv[r]);
        T &c = acc[r * MT + m];
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const float2 wf = __half22float2(wh[q]);
          c = fmaf(af[q].x, wf.x, c);
          c = fmaf(af[q].y, wf.y, c);
        }
      }
    }
  }
}

constexpr int kDirectWarps = 8;

template <int FMT, int MT, int CPW, int U>
__global__ void __launch_bounds__(kDirectWarps * 32)
gemv_direct_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ A, void *__restrict__ Cout, int M,
                   int K, int N, Tables tb) {
  using T = typename Acc<FMT>::T;
  constexpr int V = CPW * MT;
  asm volatile("griddepcontrol.launch_dependents;");
  const int lane = threadIdx.x & 31;
  const int n0 = ((int)blockIdx.x * kDirectWarps + (int)(threadIdx.x >> 5)) * CPW;
  const size_t rowB = (FMT == FMT_F16) ? (size_t)K * 2 : (FMT == FMT_I8) ? (size_t)K : (size_t)K / 2;
  const size_t a_row = (FMT == FMT_F16) ? (size_t)K * 2 : (size_t)K;
  const uint32_t a_k = (FMT == FMT_U4 || FMT == FMT_NF4) ? 2u : 1u;  // activation bytes per weight byte
  const int nch = (int)(rowB / 16);
  const bool active = n0 < N;
  const uint8_t *wrow[CPW];
#pragma unroll
  for (int r = 0; r < CPW; r++) wrow[r] = W + (size_t)min(n0 + r, N - 1) * rowB;  // clamped rows read, unused

  uint4 ring[U][CPW];
#pragma unroll
  for (int u = 0; u < U; u++) {
    const int ch = lane + 32 * u;
#pragma unroll
    for (int r = 0; r < CPW; r++)
      if (active && ch < nch) ring[u][r] = ldg_stream(wrow[r] + (size_t)ch * 16);
  }
  // L2 prefetch of the activations before the wait (a hint only: they are read through L1 after it)
  if (threadIdx.x == 0 && (blockIdx.x & 7) == 0)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(A), "r"((uint32_t)(M * a_row)) : "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (!active) return;

  T acc[V];
#pragma unroll
  for (int i = 0; i < V; i++) acc[i] = T(0);
  for (int base = lane; base < nch; base += 32 * U) {
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int ch = base + 32 * u;
      if (ch < nch) {
        uint4 wv[CPW];
#pragma unroll
        for (int r = 0; r < CPW; r++) wv[r] = ring[u][r];
        const int nx = ch + 32 * U;  // refill this slot with the chunk U steps ahead
        if (nx < nch) {
#pragma unroll
          for (int r = 0; r < CPW; r++) ring[u][r] = ldg_stream(wrow[r] + (size_t)nx * 16);
        }
        mac_regs<FMT, MT, CPW, T>(wv, A + (size_t)ch * 16 * a_k, a_row, M, acc, tb);
      }
    }
  }
  bfly32<V, 16>(acc, lane);
  if (lane % (32 / V) == 0) {
    const int idx = (lane * V) >> 5, r = idx / MT, m = idx % MT;
    if (m < M && n0 + r < N) reinterpret_cast<T *>(Cout)[(size_t)m * N + n0 + r] = acc[0];
  }
}

struct Cfg {
  int mt, tr;
  int nw = kWarps;      // warps per CTA of the staged kernel
  bool direct = false;  // the direct-load kernel (cpw channels per warp) instead of the staged one
  int cpw = 2;
};

// Kernel and tile choice, measured on B200 over K in {2048, 6144, 8192}, N in {2048 .. 28672},
// M in {1, 4, 8}, int8 / uniform int4 / NF4 (weights cycled through more than L2):
// - the staged kernel with 8-channel CTAs (the smallest block, so the most CTAs share an SM and the
//   next launch's copies overlap this one) is best or within ~5% on most shapes;
// - the direct-load kernel wins where each staged CTA would carry a large activation block (M = 8 with
//   K >= 8192: up to 2x), on nibble weights with short rows (K <= 2048, N <= 8192: 5-20%), and is the
//   only one for rows that do not fit the staged kernel's shared memory (any K).
Cfg choose(int fmt, int M, int K, int N, const Tuning &tu) {
  Cfg c;
  c.mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  const size_t rowB = fmt_row_bytes(fmt, K);
  const bool nib = fmt == FMT_U4 || fmt == FMT_NF4;
  c.tr = 8;
  // 8 weight rows and 8 activation rows in shared memory; rows that fit only with this launch's own
  // activation rows (up to c.mt) are staged when even a one-channel-per-warp direct grid (N / 8 CTAs)
  // would be under two CTAs per SM, and otherwise go to the direct kernel with one channel per warp
  // while its four-channel grid (N / 32) would not fill the SMs. The 70B down projection's column
  // shards, NF4 M = 1 (weights cycled past L2): 28672x1024 staged 6.2 us against 15.8 direct,
  // 28672x2048 12.3 against 17.1, 28672x4096 direct with one channel 19.9 against 24.0 staged and 27.4
  // with four; at full width (28672x8192) four channels per warp, 30.7 against 34.1 with one
  const size_t esz = fmt == FMT_F16 ? 2 : 1;
  const bool fits8 = rowB * 8 + (size_t)8 * K * esz <= 196 * 1024;
  const bool staged_fits = fits8 || (rowB * 8 + (size_t)c.mt * K * esz <= 196 * 1024 && N / 8 < 296);
  if (!staged_fits || (c.mt == 8 && K >= 8192)) {
    c.direct = true;
    c.cpw = (!staged_fits || (c.mt == 8 && fmt != FMT_NF4)) ? 4 : 2;
    if (!fits8 && c.mt == 1 && N / 32 < 148) c.cpw = 1;
  } else if (nib && K <= 2048 && N <= 8192) {
    c.direct = true;
    c.cpw = 2;
  }
  // 8 warps per 8-channel CTA (K split 8 ways: the post-dependency dot product of a CTA halves) for one
  // row on weights of 8 Mi elements or more with N <= 8192 (measured: 2048x6144 3.65 -> 3.46 us, 6144x2048
  // 3.73 -> 3.66, 8192x8192 12.74 -> 12.46; slower on 2048x12288 and no gain on 2048x2048)
  if (!c.direct && c.mt == 1 && c.tr == 8 && (size_t)K * N >= ((size_t)8 << 20) && N <= 8192) c.nw = 8;
  // tuning overrides (the context's ORKB_GEMV_* values)
  if (tu.gemv_kind >= 0) c.direct = tu.gemv_kind == 1 || !staged_fits;
  if (tu.gemv_cpw == 1 || tu.gemv_cpw == 2 || tu.gemv_cpw == 4) c.cpw = tu.gemv_cpw;
  if ((tu.gemv_tr == 8 || tu.gemv_tr == 16 || tu.gemv_tr == 32) &&
      (size_t)tu.gemv_tr * rowB + (size_t)c.mt * K * 2 <= 196 * 1024)
    c.tr = tu.gemv_tr;
  if (tu.gemv_nw == 4 || tu.gemv_nw == 8 || tu.gemv_nw == 16) c.nw = tu.gemv_nw;
  // only the (channels, warps) pairs that are built: fall back to 4 warps
  if (!((c.nw == 4) || (c.nw == 8 && c.tr <= 16) || (c.nw == 16 && c.tr >= 16))) c.nw = 4;
  return c;
}

// Weight chunks per lane that a warp preloads into registers (gemv_block): one-row launches of at most
// 8192 channels take as many as the warp has, up to 8 (4 for nibbles, whose chunks expand to twice the
// registers); wider weights (their grids run several waves, which the larger register footprint
// lengthens: 2048x12288 5.3 -> 5.9 us) and larger M (whose dot product dwarfs the preload) keep 2.
// Measured at M = 1: 6144x2048 3.66 -> 3.42 us, 8192x8192 12.5 -> 11.6 us, 2048x2048 / 2048x6144 unchanged.
template <int FMT, int MT, int TR, int NW>
int preload_chunks(int K, int N) {
  if (MT > 1 || N > 8192) return 2;
  const int S = (int)((fmt_row_bytes(FMT, K) + 127) / 128), WK = NW / (TR / 8);
  const int c = (S + WK - 1) / WK;
  return c <= 2 ? 2 : (c <= 4 || FMT == FMT_U4 || FMT == FMT_NF4) ? 4 : 8;
}

template <int FMT, int MT, int TR, int NW>
cudaError_t launch_one(const RunArgs &a, const uint8_t *Ab, void *Cb, int m, cudaStream_t s, bool pdl,
                       const Tables &tb) {
  const size_t smem = (size_t)TR * fmt_row_bytes(FMT, a.K) + (size_t)m * (FMT == FMT_F16 ? 2 : 1) * a.K;
  const int P = preload_chunks<FMT, MT, TR, NW>(a.K, a.N);
  auto kern = MT > 1 || P == 2 ? gemv_kernel<FMT, MT, TR, NW, 2>
              : P == 4         ? gemv_kernel<FMT, MT, TR, NW, (MT > 1 ? 2 : 4)>
                               : gemv_kernel<FMT, MT, TR, NW, (MT > 1 ? 2 : 8)>;
  {  // the full dynamic budget (the static part adds ~1 KB), once per device
    const cudaError_t e = smem_attr((const void *)kern, 200 * 1024);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + TR - 1) / TR);
  cfg.blockDim = dim3(NW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, (const uint8_t *)a.W, Ab, Cb, m, a.K, a.N, tb);
}

template <int FMT>
cudaError_t dispatch_fmt(const RunArgs &a, const Cfg &c, const uint8_t *Ab, void *Cb, int m, cudaStream_t s,
                         bool pdl, const Tables &tb) {
  // (channels per CTA, warps): 4 warps for 8 / 16 / 32 channels, 8 warps for 8 / 16, 16 warps for 16 / 32
#define ORKB_GEMV_CASE(MT_, TR_, NW_) \
  if (c.mt == MT_ && c.tr == TR_ && c.nw == NW_) return launch_one<FMT, MT_, TR_, NW_>(a, Ab, Cb, m, s, pdl, tb);
#define ORKB_GEMV_MT(MT_)                                                                  \
  ORKB_GEMV_CASE(MT_, 8, 4) ORKB_GEMV_CASE(MT_, 16, 4) ORKB_GEMV_CASE(MT_, 32, 4)           \
  ORKB_GEMV_CASE(MT_, 8, 8) ORKB_GEMV_CASE(MT_, 16, 8) ORKB_GEMV_CASE(MT_, 16, 16)          \
  ORKB_GEMV_CASE(MT_, 32, 16)
  ORKB_GEMV_MT(1) ORKB_GEMV_MT(2) ORKB_GEMV_MT(4) ORKB_GEMV_MT(8)
#undef ORKB_GEMV_MT
#undef ORKB_GEMV_CASE
  return cudaErrorInvalidConfiguration;
}


template <int FMT, int MT, int TR>
cudaError_t launch_grouped_one(const GroupedArgs &a, const uint8_t *Ab, const float *aSb, float *Cb, int m,
                               cudaStream_t s, bool pdl, const Tables &tb) {
  const size_t rowB = fmt_row_bytes(FMT, a.K);
  const size_t smem = (size_t)TR * rowB + (((size_t)m * a.K + 15) & ~(size_t)15) + (size_t)(a.K / a.G) * TR * MT * 4;
  auto kern = gemv_grouped_kernel<FMT, MT, TR>;
  {  // the full dynamic budget (the static part adds ~1 KB), once per device
    const cudaError_t e = smem_attr((const void *)kern, 200 * 1024);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + TR - 1) / TR);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, (const uint8_t *)a.W, Ab, aSb, a.bS, Cb, m, a.K, a.N, a.G, tb);
}

// shared memory of one grouped CTA: staged weight rows, activations, the group table
size_t grouped_smem(int fmt, int K, int G, int mt, int tr) {
  return (size_t)tr * fmt_row_bytes(fmt, K) + (((size_t)mt * K + 15) & ~(size_t)15) + (size_t)(K / G) * tr * mt * 4;
}

template <int FMT>
cudaError_t dispatch_grouped(const GroupedArgs &a, int mt, int tr, const uint8_t *Ab, const float *aSb, float *Cb,
                             int m, cudaStream_t s, bool pdl, const Tables &tb) {
#define ORKB_GG_CASE(MT_, TR_) \
  if (mt == MT_ && tr == TR_) return launch_grouped_one<FMT, MT_, TR_>(a, Ab, aSb, Cb, m, s, pdl, tb);
  ORKB_GG_CASE(1, 8) ORKB_GG_CASE(1, 16) ORKB_GG_CASE(1, 32)
  ORKB_GG_CASE(2, 8) ORKB_GG_CASE(2, 16) ORKB_GG_CASE(2, 32)
  ORKB_GG_CASE(4, 8) ORKB_GG_CASE(4, 16) ORKB_GG_CASE(4, 32)
  ORKB_GG_CASE(8, 8) ORKB_GG_CASE(8, 16) ORKB_GG_CASE(8, 32)
#undef ORKB_GG_CASE
  return cudaErrorInvalidConfiguration;
}

template <int FMT, int MT, int CPW, int U>
cudaError_t launch_direct(const RunArgs &a, const uint8_t *Ab, void *Cb, int m, cudaStream_t s, bool pdl,
                          const Tables &tb) {
  cudaLaunchConfig_t cfg = {};
  const int warps = (a.N + CPW - 1) / CPW;
  cfg.gridDim = dim3((warps + kDirectWarps - 1) / kDirectWarps);
  cfg.blockDim = dim3(kDirectWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_direct_kernel<FMT, MT, CPW, U>, (const uint8_t *)a.W, Ab, Cb, m, a.K, a.N,
                            tb);
}

template <int FMT>
cudaError_t dispatch_direct(const RunArgs &a, int mt, int cpw, const uint8_t *Ab, void *Cb, int m, cudaStream_t s,
                            bool pdl, const Tables &tb) {
#define ORKB_GD_CASE(MT_, CPW_, U_) \
  if (mt == MT_ && cpw == CPW_) return launch_direct<FMT, MT_, CPW_, U_>(a, Ab, Cb, m, s, pdl, tb);
  ORKB_GD_CASE(1, 1, 8) ORKB_GD_CASE(1, 2, 4) ORKB_GD_CASE(1, 4, 2)
  ORKB_GD_CASE(2, 1, 8) ORKB_GD_CASE(2, 2, 4) ORKB_GD_CASE(2, 4, 2)
  ORKB_GD_CASE(4, 1, 4) ORKB_GD_CASE(4, 2, 4) ORKB_GD_CASE(4, 4, 2)
  ORKB_GD_CASE(8, 1, 4) ORKB_GD_CASE(8, 2, 2) ORKB_GD_CASE(8, 4, 2)
#undef ORKB_GD_CASE
  return cudaErrorInvalidConfiguration;
}

template <int FMT, int MT>
cudaError_t launch_batched_one(const BatchTable &bt, int blocks, size_t smem, cudaStream_t s, bool pdl,
                               const Tables &tb) {
  auto kern = gemv_batched_kernel<FMT, MT, 8>;
  {  // the full dynamic budget (the static part adds ~1 KB), once per device
    const cudaError_t e = smem_attr((const void *)kern, 200 * 1024);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, bt, tb);
}

template <int FMT>
cudaError_t dispatch_batched(const BatchTable &bt, int mt, int blocks, size_t smem, cudaStream_t s, bool pdl,
                             const Tables &tb) {
  switch (mt) {
    case 1: return launch_batched_one<FMT, 1>(bt, blocks, smem, s, pdl, tb);
    case 2: return launch_batched_one<FMT, 2>(bt, blocks, smem, s, pdl, tb);
    case 4: return launch_batched_one<FMT, 4>(bt, blocks, smem, s, pdl, tb);
    default: return launch_batched_one<FMT, 8>(bt, blocks, smem, s, pdl, tb);
  }
}

}  // namespace

cudaError_t launch_gemv(const RunArgs &a, cudaStream_t s, bool pdl, int *launches) {
  if ((uintptr_t)a.W % 16 || (uintptr_t)a.A % 16) return cudaErrorMisalignedAddress;
  const Tables tb = nf4_tables();
  const size_t a_row = (a.fmt == FMT_F16) ? (size_t)a.K * 2 : (size_t)a.K;
  const size_t c_row = (size_t)a.N * 4;
  for (int m0 = 0; m0 < a.M; m0 += 8) {
    const int m = a.M - m0 < 8 ? a.M - m0 : 8;
    static const Tuning none;
    const Cfg c = choose(a.fmt, m, a.K, a.N, a.tune ? *a.tune : none);
    const uint8_t *Ab = (const uint8_t *)a.A + (size_t)m0 * a_row;
    void *Cb = (uint8_t *)a.C + (size_t)m0 * c_row;
    cudaError_t e;
    if (c.direct) {
      switch (a.fmt) {
        case FMT_I8: e = dispatch_direct<FMT_I8>(a, c.mt, c.cpw, Ab, Cb, m, s, pdl, tb); break;
        case FMT_U4: e = dispatch_direct<FMT_U4>(a, c.mt, c.cpw, Ab, Cb, m, s, pdl, tb); break;
        case FMT_NF4: e = dispatch_direct<FMT_NF4>(a, c.mt, c.cpw, Ab, Cb, m, s, pdl, tb); break;
        case FMT_F16: e = dispatch_direct<FMT_F16>(a, c.mt, c.cpw, Ab, Cb, m, s, pdl, tb); break;
        default: return cudaErrorInvalidValue;
      }
      if (e != cudaSuccess) return e;
      if (launches) ++*launches;
      continue;
    }
    switch (a.fmt) {
      case FMT_I8: e = dispatch_fmt<FMT_I8>(a, c, Ab, Cb, m, s, pdl, tb); break;
      case FMT_U4: e = dispatch_fmt<FMT_U4>(a, c, Ab, Cb, m, s, pdl, tb); break;
      case FMT_NF4: e = dispatch_fmt<FMT_NF4>(a, c, Ab, Cb, m, s, pdl, tb); break;
      case FMT_F16: e = dispatch_fmt<FMT_F16>(a, c, Ab, Cb, m, s, pdl, tb); break;
      default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
  }
  return cudaSuccess;
}

unsigned int gemv_error_flag(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof v);
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_gemv_error, &z, sizeof z);
  }
  return v;
}

ORKB_ERR_WORD_SETTER(gemv_set_err_word)

}  // namespace orkb

namespace orkb {

bool grouped_supports(int fmt, int K, int G) {
  if (G <= 0 || K % G) return false;
  if (fmt == FMT_I8) {
    if (G % 16) return false;
  } else if (fmt == FMT_U4 || fmt == FMT_NF4) {
    if (G % 32) return false;
  } else {
    return false;
  }
  return grouped_smem(fmt, K, G, 8, 8) <= 196 * 1024;
}

cudaError_t launch_gemv_grouped(const GroupedArgs &a, cudaStream_t s, bool pdl, int *launches) {
  if ((uintptr_t)a.W % 16 || (uintptr_t)a.A % 16 || (uintptr_t)a.C % 4) return cudaErrorMisalignedAddress;
  if (!grouped_supports(a.fmt, a.K, a.G)) return cudaErrorInvalidValue;
  if ((size_t)a.K % 16) return cudaErrorMisalignedAddress;  // activation rows stay 16-byte aligned
  const Tables tb = nf4_tables();
  const int Sk = a.K / a.G;
  for (int m0 = 0; m0 < a.M; m0 += 8) {
    const int m = a.M - m0 < 8 ? a.M - m0 : 8;
    const int mt = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
    int tr = 8;  // as the plain decode kernel: staged rows <= 48 KB so several CTAs share an SM
    for (int t : {16, 32})
      if ((size_t)t * fmt_row_bytes(a.fmt, a.K) <= 48 * 1024 && grouped_smem(a.fmt, a.K, a.G, mt, t) <= 196 * 1024 &&
          (a.N + t - 1) / t >= 2 * 148)
        tr = t;
    const uint8_t *Ab = (const uint8_t *)a.A + (size_t)m0 * a.K;
    const float *aSb = a.aS + (size_t)m0 * Sk;
    float *Cb = a.C + (size_t)m0 * a.N;
    cudaError_t e;
    switch (a.fmt) {
      case FMT_I8: e = dispatch_grouped<FMT_I8>(a, mt, tr, Ab, aSb, Cb, m, s, pdl, tb); break;
      case FMT_U4: e = dispatch_grouped<FMT_U4>(a, mt, tr, Ab, aSb, Cb, m, s, pdl, tb); break;
      case FMT_NF4: e = dispatch_grouped<FMT_NF4>(a, mt, tr, Ab, aSb, Cb, m, s, pdl, tb); break;
      default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
  }
  return cudaSuccess;
}

}  // namespace orkb

namespace orkb {

bool batched_supports(int fmt, int M, int K) {
  return M >= 1 && M <= 8 && K > 0 && fmt_row_bytes(fmt, K) * 8 + (size_t)M * K * (fmt == FMT_F16 ? 2 : 1) <= 196 * 1024;
}

cudaError_t launch_gemv_batched(const ChainTask *t, int n, cudaStream_t s, bool pdl, int *launches) {
  const Tables tb = nf4_tables();
  for (int i0 = 0; i0 < n; i0 += kMaxBatch) {
    const int cnt = n - i0 < kMaxBatch ? n - i0 : kMaxBatch;
    BatchTable bt;
    bt.n = cnt;
    int blocks = 0, mmax = 1;
    size_t smem = 0;
    const int fmt = t[i0].fmt;
    for (int j = 0; j < cnt; j++) {
      const ChainTask &c = t[i0 + j];
      if (c.fmt != fmt || !batched_supports(c.fmt, c.M, c.K)) return cudaErrorInvalidValue;
      if ((uintptr_t)c.W % 16 || (uintptr_t)c.A % 16) return cudaErrorMisalignedAddress;
      if (c.os.mode != OUT_I32 && c.fmt == FMT_F16) return cudaErrorInvalidValue;
      bt.t[j] = BatchTask{(const uint8_t *)c.W, (const uint8_t *)c.A, c.C, c.M, c.K, c.N, c.cstride, blocks, c.os};
      blocks += (c.N + 7) / 8;
      mmax = c.M > mmax ? c.M : mmax;
      const size_t sm = fmt_row_bytes(c.fmt, c.K) * 8 + (size_t)c.M * c.K * (c.fmt == FMT_F16 ? 2 : 1);
      smem = sm > smem ? sm : smem;
    }
    const int mt = mmax <= 1 ? 1 : mmax <= 2 ? 2 : mmax <= 4 ? 4 : 8;
    cudaError_t e;
    switch (fmt) {
      case FMT_I8: e = dispatch_batched<FMT_I8>(bt, mt, blocks, smem, s, pdl, tb); break;
      case FMT_U4: e = dispatch_batched<FMT_U4>(bt, mt, blocks, smem, s, pdl, tb); break;
      case FMT_NF4: e = dispatch_batched<FMT_NF4>(bt, mt, blocks, smem, s, pdl, tb); break;
      case FMT_F16: e = dispatch_batched<FMT_F16>(bt, mt, blocks, smem, s, pdl, tb); break;
      default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
  }
  return cudaSuccess;
}

}  // namespace orkb

extern "C" int ork_b200_gemv_choice(int fmt, int M, int K, int N, int *out) {
  if (!out || fmt < orkb::FMT_F16 || fmt > orkb::FMT_NF4 || M < 1 || M > 8 || K < 1 || N < 1) return -1;
  const orkb::Cfg c = orkb::choose(fmt, M, K, N, orkb::tuning_from_env());
  out[0] = c.direct ? 1 : 0;
  out[1] = c.direct ? c.cpw : 0;
  out[2] = c.direct ? 0 : c.tr;
  out[3] = c.mt;
  return 0;
}
