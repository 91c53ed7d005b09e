// persist.cpp -- persisted tiled weights (.orkpack entries) and per-group-scaled weights.
//
// The one-page header, its stamp and the load-time refusal follow ork-driver src/npu/core/packhdr.c:
// same struct, magic, field order, zero padding, refusal order and codes. The caps id is built the same
// way (32-bit FNV-1a over the caps rule, the pack format version and the layout-deciding geometry, then
// the device id string) from THIS build's identity, so blobs tiled for another device are refused with
// ORK_PACKERR_CAPS instead of being read with the wrong layout. The payload after the header is the
// weight's resident layout (int8 / fp16 [N][K], W4A4 nibbles [N][K/2]).
//
// Grouped weights (ork-driver src/npu/i4/pack.c:686, src/npu/i4/pack.c:265, src/npu.c:1191) are the
// ordinary resident formats plus a group size; ork_i4_mm_run_grouped / ork_i8_mm_run_grouped run the
// grouped decode kernel (gemv.cu) that reproduces src/npu/core/buf.c:501-520 bit for bit.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "ork_b200.h"
#include "ork_internal.h"
#include "ork_npu.h"
#include "ork_structs.h"
#include "pack.h"

using namespace orkb;

namespace {

constexpr uint32_t kCapsRule = 1u;   // bump when the meaning of the resident layout changes
constexpr uint32_t kLayoutKMajor = 0x4B4D524Fu;  // resident rows are output channels, K contiguous
constexpr const char *kSocId = "b200";

uint32_t capid() {
  uint32_t h = 2166136261u;
  auto mix = [&](uint32_t v) {
    for (int b = 0; b < 4; b++) {
      h ^= (v >> (b * 8)) & 0xffu;
      h *= 16777619u;
    }
  };
  mix(kCapsRule);
  mix(ORK_PACK_FORMAT_VERSION);
  mix(kLayoutKMajor);
  mix(2u);  // nibble order: low nibble = even k
  for (const char *p = kSocId; *p; p++) {
    h ^= (unsigned char)*p;
    h *= 16777619u;
  }
  return h ? h : 1u;  // 0 is reserved for "unstamped"
}

void stamp(void *out, int dtype, int K, int N) {
  memset(out, 0, ORK_PACK_HDR_BYTES);  // the pad is zero: blobs are reproducible
  ork_pack_hdr *h = (ork_pack_hdr *)out;
  h->magic = ORK_PACK_MAGIC;
  h->fmt = ORK_PACK_FORMAT_VERSION;
  h->capid = capid();
  h->dtype = (uint32_t)dtype;
  h->K = K;
  h->N = N;
  h->hdr_bytes = ORK_PACK_HDR_BYTES;
  strncpy(h->soc, kSocId, sizeof h->soc - 1);
}

// 0, or the first refusal cause in the reference's order (unstamped, format, caps, header size, shape);
// each distinct cause is reported once per process.
int check(const void *blob, size_t n, int dtype, int K, int N) {
  static int said_unstamped = 0, said_fmt = 0, said_caps = 0;
  if (!blob || n < ORK_PACK_HDR_BYTES) return ORK_PACKERR_SHORT;
  ork_pack_hdr h;
  memcpy(&h, blob, sizeof h);
  if (h.magic != ORK_PACK_MAGIC) {
    if (!said_unstamped++)
      fprintf(stderr, "[ork] refusing an UNSTAMPED persisted weight (no pack header); rebuild the .orkpack\n");
    return ORK_PACKERR_UNSTAMPED;
  }
  if (h.fmt != ORK_PACK_FORMAT_VERSION) {
    if (!said_fmt++)
      fprintf(stderr, "[ork] refusing a persisted weight from pack format %u (this build is %u)\n", h.fmt,
              ORK_PACK_FORMAT_VERSION);
    return ORK_PACKERR_FORMAT;
  }
  if (h.capid != capid()) {
    char soc[17] = {0};
    memcpy(soc, h.soc, 16);
    if (!said_caps++)
      fprintf(stderr,
              "[ork] persisted weight rejected: it was written for device '%s' (caps id %08x) and this library "
              "is '%s' (caps id %08x), whose resident layout differs; dump the weight again with this library\n",
              soc, h.capid, kSocId, capid());
    return ORK_PACKERR_CAPS;
  }
  if (h.hdr_bytes != ORK_PACK_HDR_BYTES) return ORK_PACKERR_FORMAT;
  if ((int)h.dtype != dtype || h.K != K || h.N != N) return ORK_PACKERR_SHAPE;
  return 0;
}

size_t payload_bytes(int dtype, int K, int N) {
  return dtype == DT_F16 ? (size_t)K * N * 2 : dtype == DT_I4 ? (size_t)K * N / 2 : (size_t)K * N;
}

// nibbles [N][K/2] (low nibble = even k) -> int8 codes [N][K]: sign-extended, or through the NF4 table
void inflate(const uint8_t *nib, int K, int N, bool nf4, int8_t *out) {
  parallel_for(N, [&](int b, int e) {
    for (int n = b; n < e; n++) {
      const uint8_t *src = nib + (size_t)n * (K / 2);
      int8_t *dst = out + (size_t)n * K;
      for (int k = 0; k < K; k++) {
        const int q = (src[k >> 1] >> ((k & 1) * 4)) & 0xF;
        dst[k] = nf4 ? kNf4Lut[q] : (int8_t)(q >= 8 ? q - 16 : q);
      }
    }
  });
}

ork_w *load_payload(ork_npu *c, int K, int N, const void *blob, size_t n, int dtype, int fmt) {
  if (!c || check(blob, n, dtype, K, N)) return nullptr;
  if (n != ORK_PACK_HDR_BYTES + payload_bytes(dtype, K, N)) return nullptr;
  return new_weight(c, K, N, fmt, dtype, (const uint8_t *)blob + ORK_PACK_HDR_BYTES, payload_bytes(dtype, K, N));
}

int grouped_run(ork_npu *c, ork_w *w, int M, const int8_t *A, const float *aS, const float *bS, float *C,
                int want_dtype, bool async, const char *name) {
  if (!c || !w || !A || !aS || !bS || !C || M < 1) return -1;
  if (w->dtype != want_dtype || w->gsize < 1 || w->K % w->gsize) return -1;
  if (!grouped_supports(w->fmt, w->K, w->gsize)) {
    fprintf(stderr, "[ork] ERROR [%s]: group size %d is not supported for this weight format at K=%d\n", name,
            w->gsize, w->K);
    return -1;
  }
  const int Sk = w->K / w->gsize;
  const size_t abytes = (size_t)M * w->K, cbytes = (size_t)M * w->N * 4;
  const size_t asb = (size_t)M * Sk * 4, bsb = (size_t)Sk * w->N * 4;
  if (overlaps(A, abytes, C, cbytes)) {  // src/npu/i4/run.c:374
    fprintf(stderr, "[ork] ERROR [%s]: memory overlap detected! A [%p, +%zu) overlaps with C [%p, +%zu).\n", name,
            (const void *)A, abytes, (void *)C, cbytes);
    return -1;
  }
  if (!async && async_in_flight(c, name)) return -1;
  DeviceGuard dg(c->device);
  const void *dA = A;
  const float *daS = aS, *dbS = bS;
  float *dC = C;
  if (async) {
    if ((uintptr_t)A % 16 || (uintptr_t)C % 4 || (uintptr_t)aS % 4 || (uintptr_t)bS % 4) return -1;
    if (!device_ptrs_ok(c, name, {A, aS, bS, C})) return -1;
  } else {
    if (!(is_device_ptr(A, c->device) && (uintptr_t)A % 16 == 0)) {
      if (!grow(&c->dA, &c->capA, abytes)) return -1;
      if (cudaMemcpyAsync(c->dA, A, abytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
      dA = c->dA;
    }
    const bool sa_dev = is_device_ptr(aS, c->device), sb_dev = is_device_ptr(bS, c->device);
    if (!sa_dev || !sb_dev) {
      if (!grow(&c->dS, &c->capS, asb + bsb + 256)) return -1;
      uint8_t *p = (uint8_t *)c->dS;
      if (!sa_dev) {
        if (cudaMemcpyAsync(p, aS, asb, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
        daS = (const float *)p;
      }
      if (!sb_dev) {
        uint8_t *q = p + ((asb + 255) & ~(size_t)255);
        if (cudaMemcpyAsync(q, bS, bsb, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
        dbS = (const float *)q;
      }
    }
    if (!(is_device_ptr(C, c->device) && (uintptr_t)C % 4 == 0)) {
      if (!grow(&c->dC, &c->capC, cbytes)) return -1;
      dC = (float *)c->dC;
    }
  }
  GroupedArgs ga{w->d, dA, daS, dbS, dC, M, w->K, w->N, w->fmt, w->gsize};
  int nl = 0;
  cudaError_t e = launch_gemv_grouped(ga, c->stream, c->pdl, &nl);
  c->launches += (uint64_t)nl;
  if (e != cudaSuccess) {
    log_err(name, e);
    return -1;
  }
  if (async) return 0;
  if (dC != C && cudaMemcpyAsync(C, dC, cbytes, cudaMemcpyDefault, c->stream) != cudaSuccess) return -1;
  e = cudaStreamSynchronize(c->stream);
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

}  // namespace

extern "C" {

size_t ork_pack_hdr_bytes(void) { return ORK_PACK_HDR_BYTES; }

int ork_b200_pack_check(const void *blob, size_t n, int dtype, int K, int N) { return check(blob, n, dtype, K, N); }

uint32_t ork_b200_pack_capid(void) { return capid(); }

size_t ork_w_dump(const ork_w *w, void *out, size_t cap) {
  if (!w || !w->d) return 0;
  const size_t need = ORK_PACK_HDR_BYTES + payload_bytes(w->dtype, w->K, w->N);
  if (!out) return need;
  if (cap < need) return 0;
  uint8_t *p = (uint8_t *)out;
  stamp(p, w->dtype, w->K, w->N);
  DeviceGuard dg(w->ctx->device);
  const bool nib_store = w->dtype == DT_I8 && (w->fmt == FMT_U4 || w->fmt == FMT_NF4);
  if (nib_store) {  // int4 store of an int8-compute weight: its int8 codes, as the resident NPU tiles hold
    std::vector<uint8_t> nib(w->bytes);
    if (cudaMemcpy(nib.data(), w->d, w->bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return 0;
    inflate(nib.data(), w->K, w->N, w->fmt == FMT_NF4, (int8_t *)(p + ORK_PACK_HDR_BYTES));
  } else if (cudaMemcpy(p + ORK_PACK_HDR_BYTES, w->d, w->bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
    return 0;
  }
  return need;
}

size_t ork_i8_w_dump_cpu(ork_npu *c, int K, int N, const int8_t *B, void *out, size_t cap) {
  (void)c;  // host-only: the layout depends on nothing the context holds
  if (!B || K <= 0 || N <= 0 || K % 32 || N % 32) return 0;
  const size_t need = ORK_PACK_HDR_BYTES + (size_t)K * N;
  if (!out) return need;
  if (cap < need) return 0;
  stamp(out, DT_I8, K, N);
  transpose_bytes(B, (uint8_t *)out + ORK_PACK_HDR_BYTES, K, N, 1);
  return need;
}

size_t ork_i8_w_dump_bf_cpu(ork_npu *c, int K, int N, const int8_t *B, void *out, size_t cap) {
  (void)c, (void)K, (void)N, (void)B, (void)out, (void)cap;
  return 0;
}

size_t ork_i4_w_dump_cpu(ork_npu *c, int K, int N, const int8_t *B, void *out, size_t cap) {
  (void)c;
  if (!B || K <= 0 || N <= 0 || K % 32 || N % 64) return 0;
  const size_t need = ORK_PACK_HDR_BYTES + (size_t)K * N / 2;
  if (!out) return need;
  if (cap < need) return 0;
  stamp(out, DT_I4, K, N);
  pack_w4a4(B, K, N, (uint8_t *)out + ORK_PACK_HDR_BYTES);
  return need;
}

ork_w *ork_f16_mm_load(ork_npu *c, int K, int N, const void *blob, size_t n) {
  if (K <= 0 || N <= 0 || K % 32 || N % 16) return nullptr;
  return load_payload(c, K, N, blob, n, DT_F16, FMT_F16);
}

ork_w *ork_i8_mm_load(ork_npu *c, int K, int N, const void *blob, size_t n) {
  if (K <= 0 || N <= 0 || K % 32 || N % 32) return nullptr;
  return load_payload(c, K, N, blob, n, DT_I8, FMT_I8);
}

ork_w *ork_i4_mm_load(ork_npu *c, int K, int N, const void *blob, size_t n) {
  if (K <= 0 || N <= 0 || K % 32 || N % 64) return nullptr;
  return load_payload(c, K, N, blob, n, DT_I4, FMT_U4);
}

ork_w *ork_i4a8_mm_load_tiled(ork_npu *c, int K, int N, const void *blob, size_t n, int G) {
  if (!c || check(blob, n, DT_I4, K, N)) return nullptr;  // an ork_i4_w_dump_cpu blob (src/npu/i4/pack.c:267)
  if (K % 32 || N % 64 || n != ORK_PACK_HDR_BYTES + (size_t)K * N / 2) return nullptr;
  // the nibbles stay resident; as an int8-compute weight they are sign-extended uniform codes
  ork_w *w = new_weight(c, K, N, FMT_U4, DT_I8, (const uint8_t *)blob + ORK_PACK_HDR_BYTES, (size_t)K * N / 2);
  if (w) {
    w->quant_kind = ORK_QK_UNIFORM;
    w->gsize = (G > 0 && K % G == 0) ? G : 0;
  }
  return w;
}

ork_w *ork_i4_mm_pack_grouped(ork_npu *c, int K, int N, const int8_t *B, int G) {
  if (!c || !B || K <= 0 || N <= 0 || K % 32 || N % 64 || G <= 0 || G % 32 || K % G || G > 10752) return nullptr;
  std::vector<uint8_t> nib((size_t)K * N / 2);
  pack_w4a4(B, K, N, nib.data());
  ork_w *w = new_weight(c, K, N, FMT_U4, DT_I4, nib.data(), nib.size());
  if (w) w->gsize = G;
  return w;
}

int ork_w_set_group(ork_w *w, int G) {
  if (!w || (w->dtype != DT_I4 && w->dtype != DT_I8)) return -1;
  if (G > 0 && (w->K % G)) return -1;
  w->gsize = G > 0 ? G : 0;
  return 0;
}

int ork_i4_mm_run_grouped(ork_npu *c, ork_w *w, int M, const int8_t *A, const float *aScale, const float *bScale,
                          float *C) {
  return grouped_run(c, w, M, A, aScale, bScale, C, DT_I4, false, "ork_i4_mm_run_grouped");
}

int ork_i8_mm_run_grouped(ork_npu *c, ork_w *w, int M, const int8_t *A, const float *aScale, const float *bScale,
                          float *C) {
  return grouped_run(c, w, M, A, aScale, bScale, C, DT_I8, false, "ork_i8_mm_run_grouped");
}

int ork_b200_i4_mm_run_grouped_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, const float *daScale,
                                const float *dbScale, float *dC) {
  return grouped_run(c, w, M, dA, daScale, dbScale, dC, DT_I4, true, "ork_b200_i4_mm_run_grouped_async");
}

int ork_b200_i8_mm_run_grouped_async(ork_npu *c, ork_w *w, int M, const int8_t *dA, const float *daScale,
                                const float *dbScale, float *dC) {
  return grouped_run(c, w, M, dA, daScale, dbScale, dC, DT_I8, true, "ork_b200_i8_mm_run_grouped_async");
}

}  // extern "C"
