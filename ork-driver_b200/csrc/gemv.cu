// gemv.cu -- decode-path matmul (M <= 8 rows of activations per launch) on CUDA cores, sm_100a.
//
// C[m][n] = sum_k A[m][k] * B[k][n] with the weight resident K-major (one output channel per row, see
// ork_internal.h). The path is HBM-bound: every weight byte is read exactly once per launch, with
// 128-bit loads that bypass L1, and the arithmetic is done in registers:
//   int8  : 4 x dp4a per 16 weight bytes and activation row;
//   int4  : the nibble is moved to the top of a byte ((w<<4)&0xF0F0F0F0 / w&0xF0F0F0F0), so each byte
//           holds 16*code; dp4a then accumulates 16*dot exactly and the lane's sum is shifted right by 4
//           before the cross-lane reduction (exact: every partial is a multiple of 16);
//   NF4   : the nibble indexes two 8-entry byte tables with prmt -- pos = lut[8..15] (selected when bit 3
//           is set) and neg = -lut[0..7] (selected when bit 3 is clear; prmt's sign-replicate mode
//           yields 0 for the other half because every table byte is >= 0), dot = dp4a(pos) - dp4a(neg);
//   fp16  : converted to fp32 and accumulated with FFMA.
// Every integer result is exact int32, identical to ork-driver's CPU oracle (src/npu/core/buf.c:428).
//
// Work mapping: a warp owns 4*R output channels. Eight lanes cover one channel, each loading 16 B, so
// one warp-wide load moves 4 channels x 128 contiguous bytes and the activation chunk it multiplies is
// shared (broadcast) by the 4 channel groups. The warps of a CTA may split K (KS > 1); partial sums are
// reduced with a butterfly shuffle across the 8 lanes, then across the K-split warps in shared memory.
//
// Programmatic dependent launch: the kernel triggers its dependents immediately and issues its first
// weight loads before griddepcontrol.wait, so when launched with the PDL attribute the weight stream
// overlaps the previous kernel's tail; activations are only read after the wait.
#include <cuda_fp16.h>

#include "ork_internal.h"

namespace orkb {

namespace {

constexpr int kU = 4;  // 128-byte steps in flight per lane and row

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ldg_keep(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
  return __dp4a((int)a, (int)b, c);
}

// prmt.b32 in its default mode. Emitted directly because the selector's bit 3 (replicate the sign of
// the selected byte) is part of the NF4 lookup, and __byte_perm only honours the low 3 bits.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
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

template <int FMT, int MT, int R, int KS, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
gemv_kernel(const uint8_t *__restrict__ W, const uint8_t *__restrict__ A, void *__restrict__ Cout,
            int M, int K, int N, uint32_t t_neg0, uint32_t t_neg1, uint32_t t_pos0, uint32_t t_pos1) {
  using T = typename Acc<FMT>::T;
  constexpr int WR = WARPS / KS;
  constexpr int ROWS_W = 4 * R;
  constexpr int ROWS_CTA = WR * ROWS_W;
  constexpr int V = R * MT;

  asm volatile("griddepcontrol.launch_dependents;");

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 3, j = lane & 7;
  const int wr = warp / KS, wk = warp % KS;
  const int cta_row0 = blockIdx.x * ROWS_CTA;
  const int row0 = cta_row0 + wr * ROWS_W + g;
  const size_t rowB = (FMT == FMT_F16) ? (size_t)K * 2 : (FMT == FMT_I8) ? (size_t)K : (size_t)K / 2;
  const int S = (int)((rowB + 127) / 128);
  const size_t a_row_bytes = (FMT == FMT_F16) ? (size_t)K * 2 : (size_t)K;

  T acc[V];
  T neg[(FMT == FMT_NF4) ? V : 1];
#pragma unroll
  for (int i = 0; i < V; i++) acc[i] = T(0);
#pragma unroll
  for (int i = 0; i < ((FMT == FMT_NF4) ? V : 1); i++) neg[i] = T(0);

  const uint8_t *wrow[R];
  bool rowok[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int n = row0 + 4 * r;
    rowok[r] = n < N;
    wrow[r] = W + (size_t)(rowok[r] ? n : 0) * rowB;
  }

  bool waited = false;
  for (int s0 = wk; s0 < S; s0 += KS * kU) {
    uint4 wv[kU][R];
    bool ok[kU];
#pragma unroll
    for (int u = 0; u < kU; u++) {
      const int s = s0 + u * KS;
      const size_t o = (size_t)s * 128 + (size_t)j * 16;
      ok[u] = (s < S) && (o < rowB);
#pragma unroll
      for (int r = 0; r < R; r++)
        wv[u][r] = (ok[u] && rowok[r]) ? ldg_stream(wrow[r] + o) : make_uint4(0, 0, 0, 0);
    }
    if (!waited) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      waited = true;
    }
#pragma unroll
    for (int u = 0; u < kU; u++) {
      if (!ok[u]) continue;
      const size_t o = (size_t)(s0 + u * KS) * 128 + (size_t)j * 16;
#pragma unroll
      for (int m = 0; m < MT; m++) {
        if (m >= M) break;
        const uint8_t *arow = A + (size_t)m * a_row_bytes;
        if constexpr (FMT == FMT_I8) {
          const uint4 a = ldg_keep(arow + o);
#pragma unroll
          for (int r = 0; r < R; r++) {
            T &c = acc[r * MT + m];
            c = dp4a(a.x, wv[u][r].x, c);
            c = dp4a(a.y, wv[u][r].y, c);
            c = dp4a(a.z, wv[u][r].z, c);
            c = dp4a(a.w, wv[u][r].w, c);
          }
        } else if constexpr (FMT == FMT_U4) {
          const uint4 a0 = ldg_keep(arow + 2 * o), a1 = ldg_keep(arow + 2 * o + 16);
          const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          uint32_t ev[4], od[4];
#pragma unroll
          for (int q = 0; q < 4; q++) {
            ev[q] = prmt(aw[2 * q], aw[2 * q + 1], 0x6420);
            od[q] = prmt(aw[2 * q], aw[2 * q + 1], 0x7531);
          }
#pragma unroll
          for (int r = 0; r < R; r++) {
            const uint32_t ww[4] = {wv[u][r].x, wv[u][r].y, wv[u][r].z, wv[u][r].w};
            T &c = acc[r * MT + m];
#pragma unroll
            for (int q = 0; q < 4; q++) {
              c = dp4a(ev[q], (ww[q] << 4) & 0xF0F0F0F0u, c);
              c = dp4a(od[q], ww[q] & 0xF0F0F0F0u, c);
            }
          }
        } else if constexpr (FMT == FMT_NF4) {
          const uint4 a0 = ldg_keep(arow + 2 * o), a1 = ldg_keep(arow + 2 * o + 16);
          const uint32_t aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
          for (int r = 0; r < R; r++) {
            const uint32_t ww[4] = {wv[u][r].x, wv[u][r].y, wv[u][r].z, wv[u][r].w};
            T &c = acc[r * MT + m];
            T &d = neg[r * MT + m];
#pragma unroll
            for (int q = 0; q < 4; q++) {
              const uint32_t w = ww[q], x = ww[q] ^ 0x88888888u;
              c = dp4a(aw[2 * q], prmt(t_pos0, t_pos1, x), c);
              c = dp4a(aw[2 * q + 1], prmt(t_pos0, t_pos1, x >> 16), c);
              d = dp4a(aw[2 * q], prmt(t_neg0, t_neg1, w), d);
              d = dp4a(aw[2 * q + 1], prmt(t_neg0, t_neg1, w >> 16), d);
            }
          }
        } else {  // FMT_F16
          const uint4 a = ldg_keep(arow + o);
          const __half2 *ah = reinterpret_cast<const __half2 *>(&a);
          float2 af[4];
#pragma unroll
          for (int q = 0; q < 4; q++) af[q] = __half22float2(ah[q]);
#pragma unroll
          for (int r = 0; r < R; r++) {
            const __half2 *wh = reinterpret_cast<const __half2 *>(&wv[u][r]);
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
  }
  if (!waited) asm volatile("griddepcontrol.wait;" ::: "memory");

  // per-lane finalisation (linear, so it commutes with the reduction)
  if constexpr (FMT == FMT_U4) {
#pragma unroll
    for (int i = 0; i < V; i++) acc[i] >>= 4;
  } else if constexpr (FMT == FMT_NF4) {
#pragma unroll
    for (int i = 0; i < V; i++) acc[i] -= neg[i];
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

  T *C = reinterpret_cast<T *>(Cout);
  if constexpr (KS == 1) {
    if (writer) {
#pragma unroll
      for (int i = 0; i < HELD; i++) {
        const int idx = base + i, r = idx / MT, m = idx % MT;
        const int n = row0 + 4 * r;
        if (m < M && n < N) C[(size_t)m * N + n] = acc[i];
      }
    }
  } else {
    __shared__ T red[KS][ROWS_CTA][MT];
    if (writer) {
#pragma unroll
      for (int i = 0; i < HELD; i++) {
        const int idx = base + i, r = idx / MT, m = idx % MT;
        red[wk][wr * ROWS_W + g + 4 * r][m] = acc[i];
      }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < ROWS_CTA * MT; t += WARPS * 32) {
      const int m = t / ROWS_CTA, rl = t % ROWS_CTA, n = cta_row0 + rl;
      if (m < M && n < N) {
        T s = red[0][rl][m];
#pragma unroll
        for (int q = 1; q < KS; q++) s += red[q][rl][m];
        C[(size_t)m * N + n] = s;
      }
    }
  }
}

struct Cfg {
  int mt, ks;
};

// Pick the row tile (M rows per launch, padded to 1/2/4/8) and how many warps of a CTA split K: enough
// CTAs to cover the 148 SMs a couple of times, while each warp still walks a few 128-byte steps.
Cfg choose(int fmt, int M, int K, int N) {
  Cfg c;
  c.mt = M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : 8;
  const int S = (int)((fmt_row_bytes(fmt, K) + 127) / 128);
  c.ks = 1;
  auto ctas = [N](int ks) { const int rows = (4 / ks) * 8; return (N + rows - 1) / rows; };  // WARPS=4, R=2
  while (c.ks < 4 && ctas(c.ks) < 2 * 148 && S / (2 * c.ks) >= 2) c.ks *= 2;
  return c;
}

template <int FMT, int MT, int KS>
cudaError_t launch_one(const RunArgs &a, const uint8_t *Ab, void *Cb, int m, cudaStream_t s, bool pdl,
                       uint32_t tn0, uint32_t tn1, uint32_t tp0, uint32_t tp1) {
  constexpr int WARPS = 4, R = 2;
  constexpr int ROWS_CTA = (WARPS / KS) * 4 * R;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + ROWS_CTA - 1) / ROWS_CTA);
  cfg.blockDim = dim3(WARPS * 32);
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_kernel<FMT, MT, R, KS, WARPS>, (const uint8_t *)a.W, Ab, Cb, m, a.K,
                            a.N, tn0, tn1, tp0, tp1);
}

template <int FMT>
cudaError_t dispatch_fmt(const RunArgs &a, const Cfg &c, const uint8_t *Ab, void *Cb, int m, cudaStream_t s,
                         bool pdl, uint32_t tn0, uint32_t tn1, uint32_t tp0, uint32_t tp1) {
#define ORKB_GEMV_CASE(MT_, KS_)                                                          \
  if (c.mt == MT_ && c.ks == KS_)                                                         \
    return launch_one<FMT, MT_, KS_>(a, Ab, Cb, m, s, pdl, tn0, tn1, tp0, tp1);
  ORKB_GEMV_CASE(1, 1) ORKB_GEMV_CASE(1, 2) ORKB_GEMV_CASE(1, 4)
  ORKB_GEMV_CASE(2, 1) ORKB_GEMV_CASE(2, 2) ORKB_GEMV_CASE(2, 4)
  ORKB_GEMV_CASE(4, 1) ORKB_GEMV_CASE(4, 2) ORKB_GEMV_CASE(4, 4)
  ORKB_GEMV_CASE(8, 1) ORKB_GEMV_CASE(8, 2) ORKB_GEMV_CASE(8, 4)
#undef ORKB_GEMV_CASE
  return cudaErrorInvalidConfiguration;
}

uint32_t pack4(int8_t a, int8_t b, int8_t c, int8_t d) {
  return (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) | ((uint32_t)(uint8_t)c << 16) |
         ((uint32_t)(uint8_t)d << 24);
}

}  // namespace

cudaError_t launch_gemv(const RunArgs &a, cudaStream_t s, bool pdl, int *launches) {
  const int8_t *L = kNf4Lut;
  const uint32_t tn0 = pack4(-L[0], -L[1], -L[2], -L[3]), tn1 = pack4(-L[4], -L[5], -L[6], -L[7]);
  const uint32_t tp0 = pack4(L[8], L[9], L[10], L[11]), tp1 = pack4(L[12], L[13], L[14], L[15]);
  const size_t a_row = (a.fmt == FMT_F16) ? (size_t)a.K * 2 : (size_t)a.K;
  const size_t c_row = (size_t)a.N * 4;
  for (int m0 = 0; m0 < a.M; m0 += 8) {
    const int m = a.M - m0 < 8 ? a.M - m0 : 8;
    const Cfg c = choose(a.fmt, m, a.K, a.N);
    const uint8_t *Ab = (const uint8_t *)a.A + (size_t)m0 * a_row;
    void *Cb = (uint8_t *)a.C + (size_t)m0 * c_row;
    cudaError_t e;
    switch (a.fmt) {
      case FMT_I8: e = dispatch_fmt<FMT_I8>(a, c, Ab, Cb, m, s, pdl, tn0, tn1, tp0, tp1); break;
      case FMT_U4: e = dispatch_fmt<FMT_U4>(a, c, Ab, Cb, m, s, pdl, tn0, tn1, tp0, tp1); break;
      case FMT_NF4: e = dispatch_fmt<FMT_NF4>(a, c, Ab, Cb, m, s, pdl, tn0, tn1, tp0, tp1); break;
      case FMT_F16: e = dispatch_fmt<FMT_F16>(a, c, Ab, Cb, m, s, pdl, tn0, tn1, tp0, tp1); break;
      default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
    if (launches) ++*launches;
  }
  return cudaSuccess;
}

}  // namespace orkb
