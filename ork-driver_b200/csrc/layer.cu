// layer.cu -- the whole decode layer (ork_i8_mm_layer, ork-driver include/ork/chain.h:105-110) on B200.
//
// The reference runs one token (M = 1) through a Llama/Qwen-style layer with fp32 glue on its CPU and
// seven int8 matmuls on its NPU (src/npu/i8/chain.c:106-122, glue in src/spine_kernels.h). Here the glue
// runs in small fused kernels between the library's matmuls, every launch chained with programmatic
// dependent launch so the next matmul streams its weights while the glue runs:
//   1 norm_quant      RMSNorm(x) * attn_norm -> per-tensor int8 (s = 127 / max|.|)        1 CTA
//   2 matmul batch    q, k, v projections in one batched decode launch
//   3 attention       per query head: dequant, RMSNorm(q_norm), RoPE NeoX, softmax(q.K) V; the last
//                     head's CTA quantizes all heads' output (global max)                   H CTAs
//   4 matmul          o projection
//   5 norm_quant      x1 = x + Co / sa, RMSNorm(x1) * ffn_norm -> int8                     1 CTA
//   6 matmul batch    gate, up
//   7 swiglu_quant    silu(Cg / sf) * (Cu / sf) -> int8                                    1 CTA
//   8 matmul          down
//   9 residual        x_out = x1 + Cd / sac
// The glue uses the same formulas and operation order as the reference element by element; sums and
// maxima are tree reductions and expf/sinf/cosf/powf are CUDA's, so results agree with the reference to
// rounding (a quantization code can flip where a value sits on a rounding boundary).
// Decode extension (ork_i8_mm_layer_async in ork_b200.h): the token's k (dequantized, k-normed, rotated)
// and v are written into the caches at slot nkv and attention covers nkv + 1 keys; the position can be
// read from device memory so a captured graph replays across tokens.
#include <cuda_runtime.h>

#include <cstdio>
#include <vector>

#include "ork_b200.h"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"

namespace orkb {

namespace {

constexpr int kGlueThreads = 1024;
constexpr int kAttnThreads = 128;

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
  v = l < nw ? red[l] : 0.0f;
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ int8_t q8(float v, float s) {
  const int q = __float2int_rn(v * s);  // lrintf in the default rounding mode: nearest, ties to even
  return (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
}

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
  float ss = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (Co) {
      v = v + Co[i] / sa;
      x1[i] = v;
    }
    row[i] = v;
    ss += v * v;
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / n + 1e-6f);
  float mx = 1e-6f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float y = row[i] * r * g[i];
    row[i] = y;
    mx = fmaxf(mx, fabsf(y));
  }
  mx = block_max(mx, red);
  const float s = 127.0f / mx;
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
  float mx = 1e-6f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float gi = Cg[i] / sf, ui = Cu[i] / sf;
    const float a = (gi / (1.0f + expf(-gi))) * ui;
    row[i] = a;
    mx = fmaxf(mx, fabsf(a));
  }
  mx = block_max(mx, red);
  const float s = 127.0f / mx;
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

struct AttnArgs {
  const int32_t *Cq, *Ck, *Cv;
  const float *sx;
  const float *q_norm, *k_norm;
  const float *Kc, *Vc;  // caches [Hkv][hstride][dk]
  float *Kw, *Vw;        // extension: where the token's k / v are written (the caches), or null
  int H, Hkv, dk, nkv, pos, hstride;
  const int *dpos;  // extension: position (= cached tokens) read on the device, or null
  float scale, base;
  float *ao;           // [H][dk] fp32 attention output
  unsigned int *gmax;  // bits of the running max |ao| (non-negative floats order as their bits)
  unsigned int *count;
  int8_t *ao8;
  float *sa;
};

// RMSNorm (gain g) + RoPE NeoX of one head vector held in shared memory (dk values, dk <= blockDim)
__device__ void norm_rope(float *v, const float *g, int dk, int pos, float base, float *red) {
  const int t = threadIdx.x;
  float sq = 0.0f;
  for (int d = t; d < dk; d += blockDim.x) sq += v[d] * v[d];
  if (g) {
    sq = block_sum(sq, red);
    const float r = 1.0f / sqrtf(sq / dk + 1e-6f);
    for (int d = t; d < dk; d += blockDim.x) v[d] = v[d] * r * g[d];
    __syncthreads();
  }
  const int h = dk / 2;
  float a = 0.0f, b = 0.0f, c = 0.0f, s = 0.0f;
  if (t < h) {
    const float th = pos * powf(base, -2.0f * t / dk);
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

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ float sm[];  // q[dk], k[dk], v[dk], scores[nk]
  __shared__ float red[32];
  __shared__ bool last;
  pdl_start();
  pdl_wait();
  const int h = blockIdx.x, t = threadIdx.x, dk = a.dk;
  const int grp = a.H / a.Hkv, hk = h / grp;
  const bool ext = a.Kw != nullptr;
  const int pos = a.dpos ? *a.dpos : a.pos;
  const int nkv = a.dpos ? *a.dpos : a.nkv;
  const int nk = ext ? nkv + 1 : nkv;
  float *q = sm, *kn = sm + dk, *vn = sm + 2 * dk, *sc = sm + 3 * dk;
  const float sx = *a.sx;
  for (int d = t; d < dk; d += blockDim.x) q[d] = a.Cq[h * dk + d] / sx;
  __syncthreads();
  norm_rope(q, a.q_norm, dk, pos, a.base, red);
  if (ext) {  // the token's own k and v (every head of the group computes them; the first one stores them)
    for (int d = t; d < dk; d += blockDim.x) {
      kn[d] = a.Ck[hk * dk + d] / sx;
      vn[d] = a.Cv[hk * dk + d] / sx;
    }
    __syncthreads();
    norm_rope(kn, a.k_norm, dk, pos, a.base, red);
    if (h % grp == 0)
      for (int d = t; d < dk; d += blockDim.x) {
        a.Kw[((size_t)hk * a.hstride + nkv) * dk + d] = kn[d];
        a.Vw[((size_t)hk * a.hstride + nkv) * dk + d] = vn[d];
      }
  }
  const float *Kh = a.Kc + (size_t)hk * a.hstride * dk, *Vh = a.Vc + (size_t)hk * a.hstride * dk;
  // scores: one warp per key, lanes across dk
  const int lane = t & 31, wp = t >> 5, nw = blockDim.x >> 5;
  for (int j = wp; j < nk; j += nw) {
    const float *kr = (ext && j == nkv) ? kn : Kh + (size_t)j * dk;
    float s = 0.0f;
    for (int d = lane; d < dk; d += 32) s += q[d] * kr[d];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) sc[j] = s * a.scale;
  }
  __syncthreads();
  float mx = -1e30f;
  for (int j = t; j < nk; j += blockDim.x) mx = fmaxf(mx, sc[j]);
  mx = block_max(mx, red);
  float z = 0.0f;
  for (int j = t; j < nk; j += blockDim.x) {
    const float e = expf(sc[j] - mx);
    sc[j] = e;
    z += e;
  }
  z = block_sum(z, red);
  __syncthreads();
  float om = 0.0f;
  for (int d = t; d < dk; d += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < nk; j++) acc += sc[j] * ((ext && j == nkv) ? vn[d] : Vh[(size_t)j * dk + d]);
    const float o = acc / z;
    a.ao[h * dk + d] = o;
    om = fmaxf(om, fabsf(o));
  }
  om = block_max(om, red);
  // the last head's CTA quantizes every head's output with the global maximum
  if (t == 0) {
    atomicMax(a.gmax, __float_as_uint(om));
    __threadfence();
    last = atomicAdd(a.count, 1u) == (unsigned int)gridDim.x - 1;
  }
  __syncthreads();
  if (last) {
    __threadfence();
    const float m = fmaxf(1e-6f, __uint_as_float(atomicAdd(a.gmax, 0u)));
    const float s = 127.0f / m;
    const int n = a.H * dk;
    for (int i = t; i < n; i += blockDim.x) a.ao8[i] = q8(__ldcg(a.ao + i), s);
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
  unsigned int *gmax, *count;
};

// The attention kernel's running maximum and CTA counter sit in the first 256 bytes, a fixed place that
// is zeroed once at allocation and left at zero by every launch (the last CTA resets them), whatever the
// dimensions of the calls that share the workspace. The first call on a context allocates the workspace,
// so it must precede any CUDA-graph capture.
static bool layer_ws(ork_npu *c, int D, int Nq, int Nk, int F, LayerWs *w) {
  const size_t parts[] = {up256(D), up256(Nq), up256(D), up256(F), up256((size_t)Nq * 4), up256((size_t)Nk * 4),
                          up256((size_t)Nk * 4), up256((size_t)D * 4), up256((size_t)F * 4), up256((size_t)F * 4),
                          up256((size_t)D * 4), up256((size_t)Nq * 4), up256((size_t)D * 4), 256};
  size_t total = 256;
  for (size_t p : parts) total += p;
  if (c->capL < total) {
    if (c->dL) cudaFree(c->dL);
    c->dL = nullptr;
    c->capL = 0;
    if (cudaMalloc(&c->dL, total) != cudaSuccess) return false;
    if (cudaMemset(c->dL, 0, total) != cudaSuccess) return false;  // gmax / count start at zero
    c->capL = total;
  }
  w->gmax = (unsigned int *)c->dL;
  w->count = w->gmax + 1;
  uint8_t *p = (uint8_t *)c->dL + 256;
  void **dst[] = {(void **)&w->xn8, (void **)&w->ao8, (void **)&w->xf8, (void **)&w->ac8, (void **)&w->Cq,
                  (void **)&w->Ck,  (void **)&w->Cv,  (void **)&w->Co,  (void **)&w->Cg,  (void **)&w->Cu,
                  (void **)&w->Cd,  (void **)&w->ao,  (void **)&w->x1,  (void **)&w->sc};
  for (int i = 0; i < 14; i++) {
    *dst[i] = p;
    p += parts[i];
  }
  return true;
}

// Enqueue one layer on the context's stream; every pointer is device memory. kv may be null (the
// reference's behaviour: caches read only, nkv keys).
int layer_enqueue(ork_npu *c, const ork_layer_dims *d, ork_w *const *W, const float *attn_norm, const float *q_norm,
                  const float *ffn_norm, const float *x, const float *Kc, const float *Vc, float *x_out,
                  const ork_b200_layer_kv *kv) {
  const int D = (int)d->D, H = (int)d->H, Hkv = (int)d->Hkv, dk = (int)d->dk, F = (int)d->Nff;
  const int Nq = H * dk, Nk = Hkv * dk;
  LayerWs ws;
  if (!layer_ws(c, D, Nq, Nk, F, &ws)) return -1;
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
    e = launch_pdl((const void *)norm_quant_kernel, 1, kGlueThreads, (size_t)D * 4, s, pdl, args);
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
    const bool ext = kv && kv->append;
    a.Kw = ext ? const_cast<float *>(Kc) : nullptr;
    a.Vw = ext ? const_cast<float *>(Vc) : nullptr;
    a.H = H;
    a.Hkv = Hkv;
    a.dk = dk;
    a.nkv = (int)d->nkv;
    a.pos = (int)d->pos;
    a.hstride = (kv && kv->hstride > 0) ? kv->hstride : (int)d->nkv;
    a.dpos = kv ? kv->dpos : nullptr;
    const int maxk = (kv && kv->hstride > 0) ? kv->hstride : (int)d->nkv + 1;
    a.scale = (float)d->attn_scale;
    a.base = (float)d->rope_base;
    a.ao = ws.ao;
    a.gmax = ws.gmax;
    a.count = ws.count;
    a.ao8 = ws.ao8;
    a.sa = ws.sc + 1;
    void *args[] = {(void *)&a};
    e = launch_pdl((const void *)attention_kernel, H, kAttnThreads, (size_t)(3 * dk + maxk) * 4, s, pdl, args);
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
    e = launch_pdl((const void *)norm_quant_kernel, 1, kGlueThreads, (size_t)D * 4, s, pdl, args);
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
    e = launch_pdl((const void *)swiglu_quant_kernel, 1, kGlueThreads, (size_t)F * 4, s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  // 8: down
  if (!mm({6}, ws.ac8, {ws.Cd})) return -1;
  {  // 9: x_out = x1 + Cd / sac
    const float *x1 = ws.x1, *sac = ws.sc + 3;
    int n = D;
    void *args[] = {(void *)&x1, (void *)&ws.Cd, (void *)&sac, (void *)&n, (void *)&x_out};
    e = launch_pdl((const void *)residual_kernel, (D + 255) / 256, 256, 0, s, pdl, args);
    if (e != cudaSuccess) goto fail;
    nl++;
  }
  c->launches += (uint64_t)nl;
  return 0;
fail:
  log_err("ork_i8_mm_layer", e);
  return -1;
}

}  // namespace orkb

using namespace orkb;

namespace {

bool dims_ok(const ork_layer_dims *d, ork_w *const *W, const ork_b200_layer_kv *kv) {
  if (!d) return false;
  const long D = d->D, H = d->H, Hkv = d->Hkv, dk = d->dk, F = d->Nff;
  if (D < 32 || H < 1 || Hkv < 1 || H % Hkv || dk < 2 || dk % 2 || dk > 256 || d->dv != d->dk || F < 32) return false;
  if (D * 4 > 200 * 1024 || F * 4 > 200 * 1024) return false;
  const long keys = (kv && kv->hstride > 0) ? kv->hstride : (long)d->nkv + 1;
  if ((3 * dk + keys) * 4 > 200 * 1024) return false;
  if (kv && kv->append && kv->hstride > 0 && !kv->dpos && (long)d->nkv + 1 > kv->hstride) return false;
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

int ork_i8_mm_layer_async(ork_npu *c, const struct ork_layer_dims *d, ork_w *wq, ork_w *wk, ork_w *wv, ork_w *wo,
                          ork_w *wg, ork_w *wu, ork_w *wd, const float *attn_norm, const float *q_norm,
                          const float *ffn_norm, const float *x, float *Kc, float *Vc, float *x_out,
                          const ork_b200_layer_kv *kv) {
  ork_w *W[7] = {wq, wk, wv, wo, wg, wu, wd};
  if (!c || !attn_norm || !q_norm || !ffn_norm || !x || !Kc || !Vc || !x_out || !dims_ok(d, W, kv)) return -3;
  DeviceGuard dg(c->device);
  return layer_enqueue(c, d, W, attn_norm, q_norm, ffn_norm, x, Kc, Vc, x_out, kv);
}

}  // extern "C"
