// layer.cu -- the whole decode layer (ork_i8_mm_layer, ork-driver include/ork/chain.h:105-110) on B200.
//
// The reference runs one token (M = 1) through a Llama/Qwen-style layer with fp32 glue on its CPU and
// seven int8 matmuls on its NPU (src/npu/i8/chain.c:106-122, glue in src/spine_kernels.h). Here the glue
// runs in small fused kernels between the library's matmuls, every launch chained with programmatic
// dependent launch so the next matmul streams its weights while the glue runs:
//   1 norm_quant      RMSNorm(x) * attn_norm -> per-tensor int8 (s = 127 / max|.|)        1 CTA
//   2 matmul batch    q, k, v projections in one batched decode launch
//   3 attention       split-KV: per query head and chunk of keys, dequant, RMSNorm(q_norm), RoPE NeoX,
//                     the chunk's softmax partials; the last CTA of a head merges its chunks, the last
//                     head's CTA quantizes all heads' output (global max)          H x S CTAs
//   4 matmul          o projection
//   5 norm_quant      x1 = x + Co / sa, RMSNorm(x1) * ffn_norm -> int8                     1 CTA
//   6 matmul batch    gate, up
//   7 swiglu_quant    silu(Cg / sf) * (Cu / sf) -> int8                                    1 CTA
//   8 matmul          down
//   9 residual        x_out = x1 + Cd / sac
// Folding the glue into the matmuls' prologues was measured slower: each matmul CTA would recompute the
// whole row's norm or SwiGLU, and at M = 1 the matmuls are latency- not bandwidth-bound.
// The glue uses the same formulas and operation order as the reference element by element; sums and
// maxima are tree reductions and expf/sinf/cosf/powf are CUDA's, so results agree with the reference to
// rounding (a quantization code can flip where a value sits on a rounding boundary).
// Decode extension (ork_b200_i8_mm_layer_async in ork_b200.h): the token's k (dequantized, k-normed, rotated)
// and v are written into the caches at slot nkv and attention covers nkv + 1 keys; the position can be
// read from device memory so a captured graph replays across tokens.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "glue.cuh"
#include "ork_b200.h"
#include "errword.cuh"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"

namespace orkb {

namespace {

constexpr int kGlueThreads = 1024;
constexpr int kAttnThreads = 256;

__device__ __forceinline__ void pdl_start() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// block-wide sum / max of one value per thread (blockDim.x a multiple of 32, <= 1024)
__device__ float block_sum(float v, float *red) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < nw ? red[l] : 0.0f;
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ float block_max(float v, float *red) {
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  v = l < nw ? red[l] : -3.0e38f;
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

using glue::q8;

// RMSNorm + per-tensor int8 quantization of one row of n values (spine_rmsnorm + spine_quant). With Co
// given, the row is first formed as x1 = x + Co / *sa_in and stored to x1.
__global__ void __launch_bounds__(kGlueThreads)
norm_quant_kernel(const float *__restrict__ x, const int32_t *__restrict__ Co, const float *__restrict__ sa_in,
                  float *__restrict__ x1, const float *__restrict__ g, int n, int8_t *__restrict__ q,
                  float *__restrict__ s_out) {
  extern __shared__ float row[];
  __shared__ float red[32];
  pdl_start();
  pdl_wait();
  const float sa = Co ? *sa_in : 1.0f;
  const int bd = blockDim.x;
  float ss = 0.0f;
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * bd) {  // four elements per thread in flight
    float xv[4];
    int32_t cv[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = i0 + k * bd;
      xv[k] = i < n ? x[i] : 0.0f;
      cv[k] = (Co && i < n) ? Co[i] : 0;
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = i0 + k * bd;
      if (i < n) {
        float v = xv[k];
        if (Co) {
          v = v + cv[k] / sa;
          x1[i] = v;
        }
        row[i] = v;
        ss += v * v;
      }
    }
  }
  ss = block_sum(ss, red);
  const float r = glue::rms_recip(ss, n);
  float mx = 1e-6f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float y = row[i] * r * g[i];
    row[i] = y;
    mx = fmaxf(mx, fabsf(y));
  }
  mx = block_max(mx, red);
  const float s = glue::qscale(mx);
  for (int i = threadIdx.x; i < n; i += blockDim.x) q[i] = q8(row[i], s);
  if (threadIdx.x == 0) *s_out = s;
}

// SwiGLU of the gate/up projections + int8 quantization (spine_silu_glu + spine_quant).
__global__ void __launch_bounds__(kGlueThreads)
swiglu_quant_kernel(const int32_t *__restrict__ Cg, const int32_t *__restrict__ Cu, const float *__restrict__ sf_in,
                    int n, int8_t *__restrict__ q, float *__restrict__ s_out) {
  extern __shared__ float row[];
  __shared__ float red[32];
  pdl_start();
  pdl_wait();
  const float sf = *sf_in;
  const int bd = blockDim.x;
  float mx = 1e-6f;
  for (int i0 = threadIdx.x; i0 < n; i0 += 4 * bd) {  // four elements per thread in flight
    int32_t gv[4], uv[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = i0 + k * bd;
      gv[k] = i < n ? Cg[i] : 0;
      uv[k] = i < n ? Cu[i] : 0;
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int i = i0 + k * bd;
      if (i < n) {
        const float gi = gv[k] / sf, ui = uv[k] / sf;
        const float a = glue::silu_mul(gi, ui);
        row[i] = a;
        mx = fmaxf(mx, fabsf(a));
      }
    }
  }
  mx = block_max(mx, red);
  const float s = glue::qscale(mx);
  for (int i = threadIdx.x; i < n; i += blockDim.x) q[i] = q8(row[i], s);
  if (threadIdx.x == 0) *s_out = s;
}

__global__ void __launch_bounds__(kGlueThreads)
residual_kernel(const float *__restrict__ x1, const int32_t *__restrict__ Cd, const float *__restrict__ s_in, int n,
                float *__restrict__ out) {
  pdl_start();
  pdl_wait();
  const float s = *s_in;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = x1[i] + Cd[i] / s;
}

constexpr int kAttnWarps = kAttnThreads / 32;

// Sticky flag: a layer launch met a position outside its caches (the device-read position of a captured
// graph); its attention is skipped and the error reported by the next synchronising call.
__device__ unsigned int g_layer_error = 0;
constexpr int kMaxSplit = 256;  // split-KV CTAs per head at most

struct AttnArgs {
  const int32_t *Cq, *Ck, *Cv;
  const float *sx;
  const float *q_norm, *k_norm;
  const float *Kc, *Vc;  // caches [Hkv][hstride][dk]
  float *Kw, *Vw;        // extension: where the token's k / v are written (the caches), or null
  int H, Hkv, dk, nkv, pos, hstride;
  const int *dpos;  // extension: position (= cached tokens) read on the device, or null
  int kpc;          // most keys per split CTA (a multiple of 32): gridDim.y * kpc covers the most keys
  float scale, base;
  float *pm, *pz, *po;  // split partials: max [H][gridDim.y], exp-sum [H][gridDim.y], V rows [H][gridDim.y][dk]
  float *ao;            // [H][dk] fp32 attention output
  unsigned int *gmax;   // bits of the running max |ao| (non-negative floats order as their bits)
  unsigned int *hcount; // [H] split CTAs done per head, left at zero
  unsigned int *count;  // heads done, left at zero
  int8_t *ao8;
  float *sa;
};

// RMSNorm (gain g) + RoPE NeoX of one head vector held in shared memory (dk values, dk / 2 <= blockDim)
__device__ void norm_rope(float *v, const float *g, int dk, int pos, float base, float *red) {
  const int t = threadIdx.x;
  float sq = 0.0f;
  for (int d = t; d < dk; d += blockDim.x) sq += v[d] * v[d];
  if (g) {
    sq = block_sum(sq, red);
    const float r = glue::rms_recip(sq, dk);
    for (int d = t; d < dk; d += blockDim.x) v[d] = v[d] * r * g[d];
    __syncthreads();
  }
  const int h = dk / 2;
  float a = 0.0f, b = 0.0f, c = 0.0f, s = 0.0f;
  if (t < h) {
    const float th = glue::rope_angle(pos, base, t, dk);
    c = cosf(th);
    s = sinf(th);
    a = v[t];
    b = v[t + h];
  }
  __syncthreads();
  if (t < h) {
    v[t] = a * c - b * s;
    v[t + h] = a * s + b * c;
  }
  __syncthreads();
}

// Split-KV decode attention. The nk keys of a head are cut into S <= gridDim.y chunks of kpc keys, kpc the
// smallest multiple of 32 that covers nk (nk may be read on the device, so S is decided there and CTAs
// past it return at once); CTA (h, sp) scores its chunk with
// one warp per key (lanes across dk, four keys per warp in flight), and writes the chunk's max, exp-sum and
// exp-weighted V row. The last CTA of a head merges the S partials rescaled to the head's max, and the last
// head quantizes all heads' output with the global max.
__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ float sm[];  // q[dk], k[dk], v[dk], scores[kpc], partial rows [warps][dk], weights[kMaxSplit]
  __shared__ float red[32];
  __shared__ bool last_split, last_head;
  pdl_start();
  pdl_wait();
  const int h = blockIdx.x, sp = blockIdx.y, t = threadIdx.x, dk = a.dk, Sg = gridDim.y;
  const int grp = a.H / a.Hkv, hk = h / grp;
  const bool ext = a.Kw != nullptr;
  const int pos = a.dpos ? *a.dpos : a.pos;
  const int nkv = a.dpos ? *a.dpos : a.nkv;
  const int nk = ext ? nkv + 1 : nkv;
  const int kpc = max(32, (nk + 32 * Sg - 1) / (32 * Sg) * 32);  // <= a.kpc, the shared-memory size
  if (nk < 1 || kpc > a.kpc || nkv > a.hstride || (ext && nkv >= a.hstride)) {
    if (h == 0 && sp == 0 && t == 0) { atomicOr(&g_layer_error, 1u); err_word_set(); }
    return;
  }
  const int S = (nk + kpc - 1) / kpc;
  if (sp >= S) return;
  const int j0 = sp * kpc, j1 = min(nk, j0 + kpc), n = j1 - j0;
  const bool own = ext && j0 <= nkv && nkv < j1;  // the token's own key falls in this chunk
  float *q = sm, *kn = sm + dk, *vn = sm + 2 * dk, *sc = sm + 3 * dk, *part = sc + a.kpc, *wts = part + kAttnWarps * dk;
  const int lane = t & 31, wp = t >> 5, per = dk / 32;
  const float sx = *a.sx;
  for (int d = t; d < dk; d += blockDim.x) q[d] = a.Cq[h * dk + d] / sx;
  __syncthreads();
  norm_rope(q, a.q_norm, dk, pos, a.base, red);
  if (own) {
    for (int d = t; d < dk; d += blockDim.x) {
      kn[d] = a.Ck[hk * dk + d] / sx;
      vn[d] = a.Cv[hk * dk + d] / sx;
    }
    __syncthreads();
    norm_rope(kn, a.k_norm, dk, pos, a.base, red);
    if (h % grp == 0)  // the group's first query head stores the token's k and v
      for (int d = t; d < dk; d += blockDim.x) {
        a.Kw[((size_t)hk * a.hstride + nkv) * dk + d] = kn[d];
        a.Vw[((size_t)hk * a.hstride + nkv) * dk + d] = vn[d];
      }
  }
  const float *Kh = a.Kc + (size_t)hk * a.hstride * dk, *Vh = a.Vc + (size_t)hk * a.hstride * dk;
  float qr[8];
#pragma unroll
  for (int i = 0; i < 8; i++) qr[i] = i < per ? q[lane + 32 * i] : 0.0f;
  for (int jb = j0; jb < j1; jb += 4 * kAttnWarps) {
    float kr[4][8];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int j = jb + wp + kAttnWarps * u;
      const float *row = j >= j1 ? nullptr : (own && j == nkv) ? kn : Kh + (size_t)j * dk;
#pragma unroll
      for (int i = 0; i < 8; i++) kr[u][i] = (row && i < per) ? row[lane + 32 * i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      float sv = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; i++) sv += qr[i] * kr[u][i];
      for (int o = 16; o; o >>= 1) sv += __shfl_xor_sync(0xffffffffu, sv, o);
      const int j = jb + wp + kAttnWarps * u;
      if (lane == 0 && j < j1) sc[j - j0] = sv * a.scale;
    }
  }
  __syncthreads();
  float m = -3.0e38f;
  for (int j = t; j < n; j += blockDim.x) m = fmaxf(m, sc[j]);
  m = block_max(m, red);
  float z = 0.0f;
  for (int j = t; j < n; j += blockDim.x) {
    const float e = expf(sc[j] - m);
    sc[j] = e;
    z += e;
  }
  z = block_sum(z, red);  // its barriers also publish sc
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; i++) acc[i] = 0.0f;
  for (int jb = j0; jb < j1; jb += 4 * kAttnWarps) {
    float vr[4][8];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int j = jb + wp + kAttnWarps * u;
      const float *row = j >= j1 ? nullptr : (own && j == nkv) ? vn : Vh + (size_t)j * dk;
#pragma unroll
      for (int i = 0; i < 8; i++) vr[u][i] = (row && i < per) ? row[lane + 32 * i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int j = jb + wp + kAttnWarps * u;
      const float e = j < j1 ? sc[j - j0] : 0.0f;
#pragma unroll
      for (int i = 0; i < 8; i++) acc[i] += e * vr[u][i];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; i++)
    if (i < per) part[wp * dk + lane + 32 * i] = acc[i];
  __syncthreads();
  for (int d = t; d < dk; d += blockDim.x) {
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; w++) sum += part[w * dk + d];
    a.po[((size_t)h * Sg + sp) * dk + d] = sum;
  }
  if (t == 0) {
    a.pm[h * Sg + sp] = m;
    a.pz[h * Sg + sp] = z;
  }
  __threadfence();
  __syncthreads();
  if (t == 0) last_split = atomicAdd(a.hcount + h, 1u) == (unsigned int)S - 1;
  __syncthreads();
  if (!last_split) return;
  // merge the head's S partials: weights exp(m_i - M), normalizer sum z_i exp(m_i - M)
  __threadfence();
  float M = -3.0e38f;
  for (int i = t; i < S; i += blockDim.x) M = fmaxf(M, __ldcg(a.pm + h * Sg + i));
  M = block_max(M, red);
  float Z = 0.0f;
  for (int i = t; i < S; i += blockDim.x) {
    const float w = expf(__ldcg(a.pm + h * Sg + i) - M);
    wts[i] = w;
    Z += __ldcg(a.pz + h * Sg + i) * w;
  }
  Z = block_sum(Z, red);
  float om = 0.0f;
  for (int d = t; d < dk; d += blockDim.x) {
    float o = 0.0f;
    for (int i = 0; i < S; i++) o += __ldcg(a.po + ((size_t)h * Sg + i) * dk + d) * wts[i];
    o /= Z;
    a.ao[h * dk + d] = o;
    om = fmaxf(om, fabsf(o));
  }
  om = block_max(om, red);
  __threadfence();
  if (t == 0) {
    a.hcount[h] = 0u;
    atomicMax(a.gmax, __float_as_uint(om));
    __threadfence();
    last_head = atomicAdd(a.count, 1u) == (unsigned int)a.H - 1;
  }
  __syncthreads();
  if (last_head) {
    __threadfence();
    const float s = glue::qscale(__uint_as_float(atomicAdd(a.gmax, 0u)));
    const int nq = a.H * dk;
    for (int i = t; i < nq; i += blockDim.x) a.ao8[i] = q8(__ldcg(a.ao + i), s);
    if (t == 0) {
      *a.sa = s;
      *a.gmax = 0u;
      *a.count = 0u;
    }
  }
}

cudaError_t launch_pdl(const void *kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, void **args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kern, args);
}

size_t up256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

// Workspace of one layer call, carved from one device allocation held by the context.
struct LayerWs {
  int8_t *xn8, *ao8, *xf8, *ac8;
  int32_t *Cq, *Ck, *Cv, *Co, *Cg, *Cu, *Cd;
  float *ao, *x1, *sc;  // sc: sx, sa, sf, sac
  float *pm, *pz, *po;  // attention split partials
  uint64_t *ll;         // persistent layer: the epoch-tagged words its CTAs exchange
  unsigned int *gmax, *count, *hcount;
  unsigned int *epoch, *sync;  // persistent layer: launch epoch, arrival counts
};

constexpr int kMaxHeads = 4096;
constexpr int kMaxGrid = 1024;  // CTAs of a persistent layer launch at most (one per SM)
constexpr size_t kCounterBytes = 256 + kMaxHeads * 4;

// Split-KV CTAs per head for attention over at most maxk keys: enough chunks of 32 keys to fill about one
// wave of the GPU's resident CTAs across the H heads.
static int attn_splits(int H, int maxk) {
  const int cap = std::max(1, std::min(kMaxSplit, 148 * (2048 / kAttnThreads) / H));
  return std::max(1, std::min(cap, (maxk + 31) / 32));
}
static int attn_kpc(int maxk, int Sg) { return std::max(32, (maxk + 32 * Sg - 1) / (32 * Sg) * 32); }
static size_t attn_smem(int dk, int kpc) { return (size_t)(3 * dk + kpc + kAttnWarps * dk + kMaxSplit) * 4; }

// Epoch-tagged words of the persistent layer: q, k, v, o, chunk maxima and sums, chunk rows, ao, head
// maxima, h, CTA maxima, the residual stream between layers.
static size_t ll_words(int D, int H, int Nq, int Nk, int F, int dk, int Sg) {
  return (size_t)Nq + 2 * (size_t)Nk + D + 2 * (size_t)H * Sg + (size_t)H * Sg * dk + Nq + H + F + kMaxGrid + D;
}

// The attention kernel's running maximum and CTA counters sit in a fixed region at the start of the
// allocation, zeroed once at allocation and left at zero by every launch (the last CTAs reset them),
// whatever the dimensions of the calls that share the workspace; so do the persistent layer's launch
// epoch (which only grows) and its arrival counts (left at zero). The first call on a context allocates
// the workspace, so it must precede any CUDA-graph capture.
static bool layer_ws(ork_npu *c, int D, int H, int Nq, int Nk, int F, int dk, int Sg, LayerWs *w) {
  const size_t parts[] = {up256(D),
                          up256(Nq),
                          up256(D),
                          up256(F),
                          up256((size_t)Nq * 4),
                          up256((size_t)Nk * 4),
                          up256((size_t)Nk * 4),
                          up256((size_t)D * 4),
                          up256((size_t)F * 4),
                          up256((size_t)F * 4),
                          up256((size_t)D * 4),
                          up256((size_t)Nq * 4),
                          up256((size_t)D * 4),
                          256,
                          up256((size_t)H * Sg * 4),
                          up256((size_t)H * Sg * 4),
                          up256((size_t)H * Sg * dk * 4),
                          up256(ll_words(D, H, Nq, Nk, F, dk, Sg) * 8)};
  constexpr int np = sizeof(parts) / sizeof(parts[0]);
  size_t total = kCounterBytes;
  for (size_t p : parts) total += p;
  if (c->capL < total) {
    if (c->dL) cudaFree(c->dL);
    c->dL = nullptr;
    c->capL = 0;
    if (cudaMalloc(&c->dL, total) != cudaSuccess) return false;
    if (cudaMemset(c->dL, 0, total) != cudaSuccess) return false;  // the counters start at zero
    c->capL = total;
  }
  w->gmax = (unsigned int *)c->dL;
  w->count = w->gmax + 1;
  w->epoch = w->gmax + 2;
  w->sync = w->gmax + 4;
  w->hcount = w->gmax + 64;
  uint8_t *p = (uint8_t *)c->dL + kCounterBytes;
  void **dst[np] = {(void **)&w->xn8, (void **)&w->ao8, (void **)&w->xf8, (void **)&w->ac8, (void **)&w->Cq,
                    (void **)&w->Ck,  (void **)&w->Cv,  (void **)&w->Co,  (void **)&w->Cg,  (void **)&w->Cu,
                    (void **)&w->Cd,  (void **)&w->ao,  (void **)&w->x1,  (void **)&w->sc,  (void **)&w->pm,
                    (void **)&w->pz,  (void **)&w->po,  (void **)&w->ll};
  for (int i = 0; i < np; i++) {
    *dst[i] = p;
    p += parts[i];
  }
  return true;
}

// Device copies of persistent-layer tables, one per distinct list of layer pointers, uploaded when first
// seen (outside CUDA-graph capture) and kept for the context's life.
struct LayerTabs {
  std::vector<std::pair<std::vector<FusedLayerW>, FusedLayerW *>> e;
};

void layer_tabs_free(ork_npu *c) {
  LayerTabs *t = (LayerTabs *)c->ltabs;
  if (!t) return;
  for (auto &p : t->e) cudaFree(p.second);
  delete t;
  c->ltabs = nullptr;
}

// True when this exact list of layer pointers already has a device table (its pointers were checked
// when it was first seen).
static bool layer_tab_seen(const ork_npu *c, const FusedLayerW *lw, int n) {
  const LayerTabs *t = (const LayerTabs *)c->ltabs;
  if (!t) return false;
  for (auto &p : t->e)
    if ((int)p.first.size() == n && !memcmp(p.first.data(), lw, sizeof(FusedLayerW) * n)) return true;
  return false;
}

static const FusedLayerW *layer_tab(ork_npu *c, const FusedLayerW *lw, int n) {
  if (!c->ltabs) c->ltabs = new (std::nothrow) LayerTabs;
  LayerTabs *t = (LayerTabs *)c->ltabs;
  if (!t) return nullptr;
  for (auto &p : t->e)
    if ((int)p.first.size() == n && !memcmp(p.first.data(), lw, sizeof(FusedLayerW) * n)) return p.second;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(c->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    fprintf(stderr, "[ork] ERROR ork_i8_mm_layer: a new list of layers during CUDA-graph capture; make one call "
                    "with these layers before capturing\n");
    return nullptr;
  }
  if (t->e.size() >= 4096) {  // bound the cache: drop everything (no graph may still use an old table...)
    fprintf(stderr, "[ork] ERROR ork_i8_mm_layer: more than 4096 distinct layer lists on one context\n");
    return nullptr;
  }
  FusedLayerW *d = nullptr;
  if (cudaMalloc(&d, sizeof(FusedLayerW) * n) != cudaSuccess) return nullptr;
  if (cudaMemcpy(d, lw, sizeof(FusedLayerW) * n, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(d);
    return nullptr;
  }
  t->e.emplace_back(std::vector<FusedLayerW>(lw, lw + n), d);
  return d;
}

// Enqueue n consecutive layers as one persistent launch (layer_fused.cu). W = the first layer's seven
// weights (dims and format are shared by all layers). Returns 0 when enqueued, -1 on an error, 1 when
// the persistent form does not apply (another format in the list, a plan that does not fit, or
// ORKB_LAYER_FUSED=0) and the caller must run the multi-launch form.
int fused_enqueue(ork_npu *c, const ork_layer_dims *d, const FusedLayerW *lw, int n, int fmt, ork_w *const *W,
                  const float *x, float *x_out, const ork_b200_layer_kv *kv) {
  const int D = (int)d->D, H = (int)d->H, Hkv = (int)d->Hkv, dk = (int)d->dk, F = (int)d->Nff;
  const int Nq = H * dk, Nk = Hkv * dk;
  const bool ext = kv && kv->append;
  const int maxk = (kv && kv->dpos) ? kv->hstride : (int)d->nkv + (ext ? 1 : 0);
  const int G = fused_grid(c->device);
  if (G < 1 || G > kMaxGrid) return 1;
  for (int i = 0; i < 7; i++)
    if (W[i]->fmt != fmt) return 1;
  if (c->tune.layer_fused == 0) return 1;  // the context's ORKB_LAYER_FUSED=0
  FusedArgs fa = {};
  fa.D = D, fa.H = H, fa.Hkv = Hkv, fa.dk = dk, fa.F = F;
  fa.Sg = fused_splits(H, maxk, G);
  fa.kpc = fused_kpc(maxk, fa.Sg);
  if (!fused_plan(&fa, fmt, G)) return 1;
  const int Sg = fa.Sg;
  LayerWs ws;
  if (!layer_ws(c, D, H, Nq, Nk, F, dk, Sg, &ws)) return -1;
  if (n == 1) {  // one layer: its pointers travel in the kernel parameters (any capture may use them)
    fa.lw = nullptr;
    fa.lw0 = *lw;
  } else {
    fa.lw = layer_tab(c, lw, n);
    if (!fa.lw) return -1;
  }
  fa.nl = n;
  fa.ext = ext ? 1 : 0;
  fa.x = x;
  fa.x_out = x_out;
  fa.nkv = (int)d->nkv;
  fa.pos = (int)d->pos;
  fa.hstride = (kv && kv->hstride > 0) ? kv->hstride : (int)d->nkv;
  fa.dpos = kv ? kv->dpos : nullptr;
  fa.scale = (float)d->attn_scale;
  fa.base = (float)d->rope_base;
  uint64_t *l = ws.ll;
  auto take = [&](size_t m) {
    uint64_t *r = l;
    l += m;
    return r;
  };
  fa.q = take(Nq), fa.k = take(Nk), fa.v = take(Nk), fa.o = take(D);
  fa.pm = take((size_t)H * Sg), fa.pz = take((size_t)H * Sg), fa.po = take((size_t)H * Sg * dk);
  fa.ao = take(Nq), fa.amax = take(H), fa.h = take(F), fa.hmax = take(kMaxGrid), fa.xl = take(D);
  fa.epoch = ws.epoch, fa.sync = ws.sync;
  const cudaError_t e = launch_layer_fused(fa, fmt, G, c->stream);
  if (e != cudaSuccess) {
    log_err("ork_i8_mm_layer (persistent)", e);
    return -1;
  }
  c->launches += 1;
  return 0;
}

// Enqueue one layer on the context's stream; every pointer is device memory. kv may be null (the
// reference's behaviour: caches read only, nkv keys).
int layer_enqueue(ork_npu *c, const ork_layer_dims *d, ork_w *const *W, const float *attn_norm, const float *q_norm,
                  const float *ffn_norm, const float *x, const float *Kc, const float *Vc, float *x_out,
                  const ork_b200_layer_kv *kv) {
  const int D = (int)d->D, H = (int)d->H, Hkv = (int)d->Hkv, dk = (int)d->dk, F = (int)d->Nff;
  const int Nq = H * dk, Nk = Hkv * dk;
  const bool ext = kv && kv->append;
  // keys attention may cover: the cache capacity when the position is read on the device
  const int maxk = (kv && kv->dpos) ? kv->hstride : (int)d->nkv + (ext ? 1 : 0);
  // the persistent one-launch layer (layer_fused.cu) when the seven weights share an int8-compute format
  // and its plan fits; ORKB_LAYER_FUSED=0 selects the multi-launch form
  FusedLayerW lw;
  for (int i = 0; i < 7; i++) lw.W[i] = (const uint8_t *)W[i]->d;
  lw.attn_norm = attn_norm, lw.q_norm = q_norm, lw.k_norm = kv ? kv->k_norm : nullptr, lw.ffn_norm = ffn_norm;
  lw.Kc = const_cast<float *>(Kc), lw.Vc = const_cast<float *>(Vc);
  const int fr = fused_enqueue(c, d, &lw, 1, W[0]->fmt, W, x, x_out, kv);
  if (fr != 1) return fr;  // 0 done, -1 error; 1: not eligible, run the multi-launch form
  const int Sg = attn_splits(H, maxk), kpc = attn_kpc(maxk, Sg);
  LayerWs ws;
  if (!layer_ws(c, D, H, Nq, Nk, F, dk, Sg, &ws)) return -1;
  {  // the glue kernels may use up to 200 KB of dynamic shared memory
    const void *k[] = {(const void *)norm_quant_kernel, (const void *)swiglu_quant_kernel,
                       (const void *)attention_kernel};
    for (const void *f : k)
      if (smem_attr(f, 200 * 1024) != cudaSuccess) return -1;
  }
  const bool pdl = c->pdl;
  cudaStream_t s = c->stream;
  int nl = 0;
  // projections reading the same activations: one batched decode launch when the weights share a format
  // and fit it, else one launch each through the ordinary route
  auto mm = [&](std::initializer_list<int> wi, const void *A, std::initializer_list<void *> Cs) -> bool {
    std::vector<ChainTask> t;
    bool batch = true;
    auto ci = Cs.begin();
    for (int i : wi) {
      ork_w *w = W[i];
      t.push_back(ChainTask{w->d, A, *ci++, 1, w->K, w->N, w->N, w->fmt});
      batch = batch && w->fmt == W[*wi.begin()]->fmt && batched_supports(w->fmt, 1, w->K);
    }
    if (batch) return launch_gemv_batched(t.data(), (int)t.size(), s, pdl, &nl) == cudaSuccess;
    auto cj = Cs.begin();
    for (int i : wi)
      if (launch(c, W[i], 1, A, *cj++)) return false;
    return true;
  };
  cudaError_t e;
  {  // 1: RMSNorm + quant of x
    const float *xx = x;
    const int32_t *no = nullptr;
    const float *nsa = nullptr;
    float *nx1 = nullptr;
    int n = D;
    void *args[] = {(void *)&xx, (void *)&no, (void *)&nsa, (void *)&nx1, (void *)&attn_norm, (void *)&n,
                    (void *)&ws.xn8, (void *)&ws.sc};
    e = launch_pdl((const void *)norm_quant_kernel, dim3(1), kGlueThreads, (size_t)D * 4, s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  // 2: q, k, v
  if (!mm({0, 1, 2}, ws.xn8, {ws.Cq, ws.Ck, ws.Cv})) return -1;
  {  // 3: attention
    AttnArgs a;
    a.Cq = ws.Cq;
    a.Ck = ws.Ck;
    a.Cv = ws.Cv;
    a.sx = ws.sc;
    a.q_norm = q_norm;
    a.k_norm = kv ? kv->k_norm : nullptr;
    a.Kc = Kc;
    a.Vc = Vc;
    a.Kw = ext ? const_cast<float *>(Kc) : nullptr;
    a.Vw = ext ? const_cast<float *>(Vc) : nullptr;
    a.H = H;
    a.Hkv = Hkv;
    a.dk = dk;
    a.nkv = (int)d->nkv;
    a.pos = (int)d->pos;
    a.hstride = (kv && kv->hstride > 0) ? kv->hstride : (int)d->nkv;
    a.dpos = kv ? kv->dpos : nullptr;
    a.kpc = kpc;
    a.scale = (float)d->attn_scale;
    a.base = (float)d->rope_base;
    a.pm = ws.pm;
    a.pz = ws.pz;
    a.po = ws.po;
    a.ao = ws.ao;
    a.gmax = ws.gmax;
    a.hcount = ws.hcount;
    a.count = ws.count;
    a.ao8 = ws.ao8;
    a.sa = ws.sc + 1;
    void *args[] = {(void *)&a};
    e = launch_pdl((const void *)attention_kernel, dim3(H, Sg), kAttnThreads, attn_smem(dk, kpc), s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  // 4: o
  if (!mm({3}, ws.ao8, {ws.Co})) return -1;
  {  // 5: x1 = x + Co / sa; RMSNorm + quant
    const float *xx = x;
    const int32_t *co = ws.Co;
    const float *sa = ws.sc + 1;
    float *x1 = ws.x1;
    int n = D;
    float *sf = ws.sc + 2;
    void *args[] = {(void *)&xx, (void *)&co, (void *)&sa, (void *)&x1, (void *)&ffn_norm, (void *)&n,
                    (void *)&ws.xf8, (void *)&sf};
    e = launch_pdl((const void *)norm_quant_kernel, dim3(1), kGlueThreads, (size_t)D * 4, s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  // 6: gate, up
  if (!mm({4, 5}, ws.xf8, {ws.Cg, ws.Cu})) return -1;
  {  // 7: SwiGLU + quant
    const float *sf = ws.sc + 2;
    float *sac = ws.sc + 3;
    int n = F;
    void *args[] = {(void *)&ws.Cg, (void *)&ws.Cu, (void *)&sf, (void *)&n, (void *)&ws.ac8, (void *)&sac};
    e = launch_pdl((const void *)swiglu_quant_kernel, dim3(1), kGlueThreads, (size_t)F * 4, s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  // 8: down
  if (!mm({6}, ws.ac8, {ws.Cd})) return -1;
  {  // 9: x_out = x1 + Cd / sac
    const float *x1 = ws.x1, *sac = ws.sc + 3;
    int n = D;
    void *args[] = {(void *)&x1, (void *)&ws.Cd, (void *)&sac, (void *)&n, (void *)&x_out};
    e = launch_pdl((const void *)residual_kernel, dim3((D + 255) / 256), 256, 0, s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  c->launches += (uint64_t)nl;
  return 0;
fail:
  log_err("ork_i8_mm_layer", e);
  return -1;
}

unsigned int layer_error_flag(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_layer_error, sizeof v);
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_layer_error, &z, sizeof z);
  }
  return v;
}

ORKB_ERR_WORD_SETTER(layer_set_err_word)

}  // namespace orkb

using namespace orkb;

namespace {

bool dims_ok(const ork_layer_dims *d, ork_w *const *W, const ork_b200_layer_kv *kv) {
  if (!d) return false;
  const long D = d->D, H = d->H, Hkv = d->Hkv, dk = d->dk, F = d->Nff;
  if (D < 32 || H < 1 || Hkv < 1 || H % Hkv || dk < 2 || dk % 2 || dk > 256 || d->dv != d->dk || F < 32) return false;
  if (D * 4 > 200 * 1024 || F * 4 > 200 * 1024) return false;
  // the caches' capacity must be given where the token is appended or the position is read on the device
  if (H > kMaxHeads || dk % 32 || (kv && (kv->dpos || kv->append) && kv->hstride <= 0)) return false;
  const long keys = (kv && kv->dpos) ? kv->hstride : (long)d->nkv + ((kv && kv->append) ? 1 : 0);
  if (keys < 1 || keys > (1 << 24)) return false;
  const int Sg = attn_splits((int)H, (int)keys);
  if (attn_smem((int)dk, attn_kpc((int)keys, Sg)) > 200 * 1024) return false;
  if (kv && kv->hstride > 0 && !kv->dpos && (long)d->nkv + (kv->append ? 1 : 0) > kv->hstride) return false;
  if (!(kv && kv->append) && d->nkv < 1) return false;
  const long Nq = H * dk, Nk = Hkv * dk;
  const long shape[7][2] = {{D, Nq}, {D, Nk}, {D, Nk}, {Nq, D}, {D, F}, {D, F}, {F, D}};
  for (int i = 0; i < 7; i++) {
    if (!W[i] || W[i]->dtype != DT_I8 || W[i]->K != shape[i][0] || W[i]->N != shape[i][1]) return false;
    if (!gemv_supports(W[i]->fmt, W[i]->K)) return false;
  }
  return true;
}

}  // namespace

extern "C" {

int ork_i8_mm_layer(ork_npu *c, const struct ork_layer_dims *d, ork_w *wq, ork_w *wk, ork_w *wv, ork_w *wo,
                    ork_w *wg, ork_w *wu, ork_w *wd, const float *attn_norm, const float *q_norm,
                    const float *ffn_norm, const float *x, const float *Kc, const float *Vc, float *x_out) {
  ork_w *W[7] = {wq, wk, wv, wo, wg, wu, wd};
  if (!c || !attn_norm || !q_norm || !ffn_norm || !x || !Kc || !Vc || !x_out || !dims_ok(d, W, nullptr)) return -3;
  if (async_in_flight(c, "ork_i8_mm_layer")) return -1;
  DeviceGuard dg(c->device);
  const size_t D = d->D, dk = d->dk, cache = (size_t)d->Hkv * d->nkv * dk;
  // host inputs are staged into one device block: x, norms, K and V caches, x_out
  const size_t parts[] = {D * 4, D * 4, dk * 4, D * 4, cache * 4, cache * 4, D * 4};
  const void *src[] = {x, attn_norm, q_norm, ffn_norm, Kc, Vc, nullptr};
  size_t off[7], total = 0;
  for (int i = 0; i < 7; i++) {
    off[i] = total;
    total += (parts[i] + 255) & ~(size_t)255;
  }
  if (!grow(&c->dS, &c->capS, total)) return -1;
  uint8_t *base = (uint8_t *)c->dS;
  const void *dp[7];
  for (int i = 0; i < 6; i++) {
    if (is_device_ptr(src[i], c->device)) {
      dp[i] = src[i];
    } else {
      dp[i] = base + off[i];
      if (cudaMemcpyAsync(base + off[i], src[i], parts[i], cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
        return -1;
    }
  }
  const bool out_dev = is_device_ptr(x_out, c->device);
  float *dout = out_dev ? x_out : (float *)(base + off[6]);
  if (layer_enqueue(c, d, W, (const float *)dp[1], (const float *)dp[2], (const float *)dp[3], (const float *)dp[0],
                    (const float *)dp[4], (const float *)dp[5], dout, nullptr))
    return -1;
  if (!out_dev && cudaMemcpyAsync(x_out, dout, D * 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) return -1;
  const cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) {
    log_err("ork_i8_mm_layer", e);
    return -1;
  }
  if (device_error()) return -1;
  return 0;
}

int ork_b200_i8_mm_layer_async(ork_npu *c, const struct ork_layer_dims *d, ork_w *wq, ork_w *wk, ork_w *wv, ork_w *wo,
                          ork_w *wg, ork_w *wu, ork_w *wd, const float *attn_norm, const float *q_norm,
                          const float *ffn_norm, const float *x, float *Kc, float *Vc, float *x_out,
                          const ork_b200_layer_kv *kv) {
  ork_w *W[7] = {wq, wk, wv, wo, wg, wu, wd};
  if (!c || !attn_norm || !q_norm || !ffn_norm || !x || !Kc || !Vc || !x_out || !dims_ok(d, W, kv)) return -3;
  DeviceGuard dg(c->device);
  if (!device_ptrs_ok(c, "ork_b200_i8_mm_layer_async",
                      {attn_norm, q_norm, ffn_norm, x, Kc, Vc, x_out, kv ? kv->k_norm : nullptr,
                       kv ? (const void *)kv->dpos : nullptr}))
    return -3;
  return layer_enqueue(c, d, W, attn_norm, q_norm, ffn_norm, x, Kc, Vc, x_out, kv);
}

int ork_b200_i8_mm_layers_async(ork_npu *c, const struct ork_layer_dims *d, int n, const ork_b200_layer_w *L,
                           const float *x, float *x_out, const ork_b200_layer_kv *kv) {
  if (!c || !L || !x || !x_out || n < 1 || n > 1024) return -3;
  for (int l = 0; l < n; l++) {
    const ork_b200_layer_w &y = L[l];
    ork_w *W[7] = {y.wq, y.wk, y.wv, y.wo, y.wg, y.wu, y.wd};
    if (!y.attn_norm || !y.q_norm || !y.ffn_norm || !y.Kc || !y.Vc || !dims_ok(d, W, kv)) return -3;
    if (y.wq->fmt != L[0].wq->fmt) return -3;
    for (int i = 1; i < 7; i++)
      if (W[i]->fmt != W[0]->fmt) return -3;
  }
  DeviceGuard dg(c->device);
  std::vector<FusedLayerW> tab(n);
  for (int l = 0; l < n; l++) {
    const ork_b200_layer_w &y = L[l];
    ork_w *W[7] = {y.wq, y.wk, y.wv, y.wo, y.wg, y.wu, y.wd};
    for (int i = 0; i < 7; i++) tab[l].W[i] = (const uint8_t *)W[i]->d;
    tab[l].attn_norm = y.attn_norm, tab[l].q_norm = y.q_norm, tab[l].k_norm = y.k_norm;
    tab[l].ffn_norm = y.ffn_norm, tab[l].Kc = y.Kc, tab[l].Vc = y.Vc;
  }
  // device pointers only: the per-layer ones are checked once per distinct list of layers
  if (!device_ptrs_ok(c, "ork_b200_i8_mm_layers_async", {x, x_out, kv ? (const void *)kv->dpos : nullptr}))
    return -3;
  if (!layer_tab_seen(c, tab.data(), n))
    for (int l = 0; l < n; l++)
      if (!device_ptrs_ok(c, "ork_b200_i8_mm_layers_async",
                          {L[l].attn_norm, L[l].q_norm, L[l].ffn_norm, L[l].k_norm, L[l].Kc, L[l].Vc}))
        return -3;
  ork_w *W0[7] = {L[0].wq, L[0].wk, L[0].wv, L[0].wo, L[0].wg, L[0].wu, L[0].wd};
  const int fr = fused_enqueue(c, d, tab.data(), n, W0[0]->fmt, W0, x, x_out, kv);
  if (fr != 1) return fr;
  // the multi-launch form, layer by layer, the residual stream through two context buffers
  const size_t xb = ((size_t)d->D * 4 + 255) & ~(size_t)255;
  if (n > 1 && !grow(&c->dX, &c->capX, 2 * xb)) return -1;
  const float *xi = x;
  for (int l = 0; l < n; l++) {
    const ork_b200_layer_w &y = L[l];
    ork_w *W[7] = {y.wq, y.wk, y.wv, y.wo, y.wg, y.wu, y.wd};
    float *xo = l == n - 1 ? x_out : (float *)((uint8_t *)c->dX + (l & 1) * xb);
    ork_b200_layer_kv k1 = kv ? *kv : ork_b200_layer_kv{nullptr, 0, 0, nullptr};
    k1.k_norm = y.k_norm;
    if (layer_enqueue(c, d, W, y.attn_norm, y.q_norm, y.ffn_norm, xi, y.Kc, y.Vc, xo, &k1)) return -1;
    xi = xo;
  }
  return 0;
}

}  // extern "C"
