// pack.cpp -- host-side pack-time code: per-channel quantizers, re-tiling to the resident layouts, and
// the O4N1 blob. Compiled with -ffp-contract=off so every float operation rounds exactly as ork-driver's
// scalar x86 build does; the int8 / int4 / NF4 codes (and hence the int32 results) are bit-identical to
// the reference's. Work is spread over channels on all host cores (ork-driver packs with all cores too,
// src/npu/core/sched.c:192), except stochastic rounding, whose single PRNG stream is sequential.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

#include "ork_internal.h"
#include "pack.h"

namespace orkb {

// src/npu.c:888-892 (ORKI_NF4_LEVELS): the 16 normalised NF4 levels.
static constexpr float kNf4Levels[16] = {
    -1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.39491748809814453f,
    -0.28444138169288635f, -0.18477343022823334f, -0.09105003625154495f, 0.0f,
    0.07958029955625534f, 0.16093020141124725f, 0.24611230194568634f, 0.33791524171829224f,
    0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f, 1.0f};

// src/npu/i4/quant.c:26: clip ratios of the imatrix scale search.
static const float kClipGrid[7] = {1.0f, 0.92f, 0.85f, 0.78f, 0.70f, 0.62f, 0.55f};

static int8_t nf4_code(int i) { return (int8_t)lrintf(kNf4Levels[i] * 127.0f); }

const int8_t kNf4Lut[16] = {nf4_code(0),  nf4_code(1),  nf4_code(2),  nf4_code(3), nf4_code(4),  nf4_code(5),
                            nf4_code(6),  nf4_code(7),  nf4_code(8),  nf4_code(9), nf4_code(10), nf4_code(11),
                            nf4_code(12), nf4_code(13), nf4_code(14), nf4_code(15)};

void parallel_for(int n, const std::function<void(int, int)> &fn) {
  int nt = (int)std::thread::hardware_concurrency();
  if (nt < 1) nt = 1;
  if (nt > n) nt = n;
  if (nt <= 1 || (size_t)n < 2) {
    if (n > 0) fn(0, n);
    return;
  }
  std::vector<std::thread> th;
  const int chunk = (n + nt - 1) / nt;
  for (int t = 0; t < nt; t++) {
    const int b = t * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    th.emplace_back([&fn, b, e] { fn(b, e); });
  }
  for (auto &x : th) x.join();
}

// src/npu.c:854-865 + src/npu/i8/pack.c:450-452.
void quant_i8_f32(int K, int N, const float *f32, int8_t *codes_nk, float *bscale) {
  parallel_for(N, [&](int b, int e) {
    for (int n = b; n < e; n++) {
      const float *fr = f32 + (size_t)n * K;
      float mx = 1e-9f;
      for (int k = 0; k < K; k++) {
        const float v = fabsf(fr[k]);
        if (v > mx) mx = v;
      }
      const float inv = 127.0f / mx;
      if (bscale) bscale[n] = mx / 127.0f;
      int8_t *dst = codes_nk + (size_t)n * K;
      for (int k = 0; k < K; k++) {
        const int q = (int)lrintf(fr[k] * inv);
        dst[k] = (int8_t)(q > 127 ? 127 : q < -127 ? -127 : q);
      }
    }
  });
}

static uint32_t xs32(uint32_t *s) {  // src/npu/internal.h:589
  uint32_t x = *s;
  x ^= x << 13;
  x ^= x >> 17;
  x ^= x << 5;
  *s = x;
  return x;
}

// The levels with a 16th entry that no value is below (+inf), for the branchless search in nf4_index;
// constant-initialised (constexpr), so a pack made during another unit's static initialisation sees it.
static constexpr float kNf4Search[16] = {
    kNf4Levels[0], kNf4Levels[1], kNf4Levels[2],  kNf4Levels[3],  kNf4Levels[4],  kNf4Levels[5],
    kNf4Levels[6], kNf4Levels[7], kNf4Levels[8],  kNf4Levels[9],  kNf4Levels[10], kNf4Levels[11],
    kNf4Levels[12], kNf4Levels[13], kNf4Levels[14], HUGE_VALF};

// src/npu/i4/quant.c:73-86: hi = first level >= wn (capped at 15), lo = hi-1; nearest with ties to hi,
// or stochastic (hi when t > u). The levels are increasing, so the first level >= wn is the number of
// levels below wn: a four-step binary search whose steps add 8 / 4 / 2 / 1 by comparison results instead
// of branching (random weights made the branches of a lower_bound mispredict about half the time). A NaN
// compares below nothing and lands on 0, as in the reference's scan.
static inline int nf4_index(float wn, int sr, uint32_t *seed) {
  if (wn > 1.0f) wn = 1.0f;
  else if (wn < -1.0f) wn = -1.0f;
  int hi = (kNf4Search[7] < wn) * 8;
  hi += (kNf4Search[hi + 3] < wn) * 4;
  hi += (kNf4Search[hi + 1] < wn) * 2;
  hi += (kNf4Search[hi] < wn) * 1;
  const int lo = hi > 0 ? hi - 1 : 0;
  if (lo == hi) return hi;
  const float t = (wn - kNf4Levels[lo]) / (kNf4Levels[hi] - kNf4Levels[lo]);
  if (sr) {
    const float u = (float)(xs32(seed) >> 8) * (1.0f / 16777216.0f);
    return (t > u) ? hi : lo;
  }
  return (t >= 0.5f) ? hi : lo;
}

// src/npu/i4/quant.c:130-151 (wq_err_chan): strictly sequential f32 accumulation.
static float wq_err(const float *fr, int K, float absmax, int nf4, const float *im) {
  float e = 0.0f;
  if (nf4) {
    const float sc = absmax / 127.0f, inv = absmax > 0 ? 1.0f / absmax : 0.0f;
    for (int k = 0; k < K; k++) {
      const int idx = nf4_index(fr[k] * inv, 0, nullptr);
      const float dq = (float)kNf4Lut[idx] * sc;
      const float d = fr[k] - dq;
      e += (im ? im[k] : 1.0f) * d * d;
    }
  } else {
    const float scale = absmax / 7.0f, inv = scale > 0 ? 1.0f / scale : 0.0f;
    for (int k = 0; k < K; k++) {
      int q = (int)lrintf(fr[k] * inv);
      if (q > 7) q = 7;
      else if (q < -7) q = -7;
      const float dq = (float)q * scale;
      const float d = fr[k] - dq;
      e += (im ? im[k] : 1.0f) * d * d;
    }
  }
  return e;
}

// src/npu/i4/quant.c:153-161 (orki_wq_best_absmax).
static float best_absmax(const float *fr, int K, float raw, int nf4, const float *im) {
  float best_abs = raw, best_e = wq_err(fr, K, raw, nf4, im);
  for (int g = 1; g < 7; g++) {
    const float cand = raw * kClipGrid[g];
    const float e = wq_err(fr, K, cand, nf4, im);
    if (e < best_e) {
      best_e = e;
      best_abs = cand;
    }
  }
  return best_abs;
}

// One channel of src/npu/i4/pack.c:60-80 / :839-850 (uniform: quant.c:28-40, NF4: quant.c:70-90).
static void i4a8_channel(const float *fr, int K, const float *im, int nf4, int sr, uint32_t *seed, uint8_t *nib,
                         float *bscale) {
  float mx = 1e-9f;
  for (int k = 0; k < K; k++) {
    const float v = fabsf(fr[k]);
    if (v > mx) mx = v;
  }
  if (im) mx = best_absmax(fr, K, mx, nf4, im);
  if (nf4) {
    *bscale = mx / 127.0f;
    const float inv = mx > 0 ? 1.0f / mx : 0.0f;
    for (int k = 0; k < K; k++) {
      const uint8_t v = (uint8_t)(nf4_index(fr[k] * inv, sr, seed) & 0xf);
      if (k & 1) nib[k >> 1] |= (uint8_t)(v << 4);
      else nib[k >> 1] = v;
    }
  } else {
    const float scale = mx / 7.0f;
    *bscale = scale;
    const float inv = scale > 0 ? 1.0f / scale : 0.0f;
    for (int k = 0; k < K; k++) {
      int q;
      if (sr) {
        const float u = (float)(xs32(seed) >> 8) * (1.0f / 16777216.0f);
        q = (int)floorf(fr[k] * inv + u);
      } else {
        q = (int)lrintf(fr[k] * inv);
      }
      if (q > 7) q = 7;
      else if (q < -7) q = -7;
      const uint8_t v = (uint8_t)(q & 0xf);
      if (k & 1) nib[k >> 1] |= (uint8_t)(v << 4);
      else nib[k >> 1] = v;
    }
  }
}

void quant_i4a8(int K, int N, const float *f32, const float *imatrix, int nf4, int sr, uint8_t *nib_nk,
                float *bscale) {
  if (sr) {  // one PRNG stream seeded 0x2545F491 across all channels in order (src/npu/i4/pack.c:32)
    uint32_t seed = 0x2545F491u;
    for (int n = 0; n < N; n++)
      i4a8_channel(f32 + (size_t)n * K, K, imatrix, nf4, 1, &seed, nib_nk + (size_t)n * (K / 2), bscale + n);
    return;
  }
  parallel_for(N, [&](int b, int e) {
    for (int n = b; n < e; n++)
      i4a8_channel(f32 + (size_t)n * K, K, imatrix, nf4, 0, nullptr, nib_nk + (size_t)n * (K / 2), bscale + n);
  });
}

// src/npu/i4/pack.c:850-858: qerr = sqrt(sum imp*(w-q)^2 / sum imp*w^2) in double, summed channel by
// channel and k by k in that order, q = code*bscale[n] with the code read back from the nibbles.
float i4a8_qerr(int K, int N, const float *f32, const float *imatrix, int nf4, const uint8_t *nib_nk,
                const float *bscale) {
  double qnum = 0.0, qden = 0.0;
  for (int n = 0; n < N; n++) {
    const float *fr = f32 + (size_t)n * K;
    const uint8_t *nb = nib_nk + (size_t)n * (K / 2);
    const float bs = bscale[n];
    for (int k = 0; k < K; k++) {
      const uint8_t ix = (k & 1) ? (nb[k >> 1] >> 4) : (nb[k >> 1] & 0xf);
      const int code = nf4 ? kNf4Lut[ix] : (ix >= 8 ? (int)ix - 16 : (int)ix);
      const double w = fr[k], q = (double)(float)code * bs, d = w - q;
      const double imp = imatrix ? imatrix[k] : 1.0;
      qnum += imp * d * d;
      qden += imp * w * w;
    }
  }
  return qden > 0.0 ? (float)std::sqrt(qnum / qden) : 0.0f;
}

void transpose_bytes(const void *src_kn, void *dst_nk, int K, int N, int esize) {
  const uint8_t *s = (const uint8_t *)src_kn;
  uint8_t *d = (uint8_t *)dst_nk;
  constexpr int T = 64;
  const int nblk = (N + T - 1) / T;
  parallel_for(nblk, [&](int b, int e) {
    for (int nb = b; nb < e; nb++) {
      const int n0 = nb * T, n1 = std::min(N, n0 + T);
      for (int k0 = 0; k0 < K; k0 += T) {
        const int k1 = std::min(K, k0 + T);
        for (int n = n0; n < n1; n++)
          for (int k = k0; k < k1; k++)
            memcpy(d + ((size_t)n * K + k) * esize, s + ((size_t)k * N + n) * esize, esize);
      }
    }
  });
}

// W4A4: B[K][N] int8 with int4 values -> nibbles [N][K/2], low nibble = even k, keeping the low 4 bits
// of each value as ork-driver's tiler does (src/npu/i4/pack.c:396-401, `B & 0xf`).
void pack_w4a4(const int8_t *B_kn, int K, int N, uint8_t *nib_nk) {
  parallel_for(N, [&](int b, int e) {
    for (int n = b; n < e; n++) {
      uint8_t *d = nib_nk + (size_t)n * (K / 2);
      for (int k = 0; k < K; k += 2) {
        const uint8_t lo = (uint8_t)B_kn[(size_t)k * N + n] & 0xf, hi = (uint8_t)B_kn[(size_t)(k + 1) * N + n] & 0xf;
        d[k >> 1] = (uint8_t)(lo | (hi << 4));
      }
    }
  });
}

// O4N1 header: src/npu/internal.h:584 (magic), :597 (struct layout), src/npu/i4/pack.c:91-103 (dump).
void o4n1_header(uint8_t *p, int K, int N, int quant_kind) {
  const uint32_t h[5] = {kO4N1Magic, kO4N1Version, (uint32_t)K, (uint32_t)N, (uint32_t)quant_kind};
  memcpy(p, h, sizeof h);
}

// src/npu/i4/pack.c:115-122: exact size, magic, version, K, N, and a known quant_kind.
bool o4n1_check(const void *blob, size_t n, int K, int N, int *quant_kind) {
  if (!blob || K <= 0 || N <= 0 || K % 32 || N % 32) return false;
  if (n != o4n1_bytes(K, N)) return false;
  uint32_t h[5];
  memcpy(h, blob, sizeof h);
  if (h[0] != kO4N1Magic || h[1] != kO4N1Version || (int32_t)h[2] != K || (int32_t)h[3] != N) return false;
  if (h[4] != 0 && h[4] != 1) return false;
  *quant_kind = (int)h[4];
  return true;
}

}  // namespace orkb
