// nibble.cuh -- int4 weight expansion shared by the decode (gemv.cu) and tensor-core (gemm_sm100.cu)
// kernels: 8 nibbles (k = 8q .. 8q+7, low nibble of each byte = the even k) -> 8 int8 codes in k order,
// as two 32-bit words. Uniform codes are sign-extended (x | (x & 8) * 0x1E per byte); NF4 indices go
// through two 8-entry prmt tables (lut[8..15] and -lut[0..7], zero in the other half; prmt's
// sign-replicate selector bit picks the half), negated bytewise without carries. Exact: the results
// are the codes ork-driver's int4 inflation produces (src/npu/i4/pack.c:63-80, src/npu.c:888-892).
#pragma once
#include <stdint.h>

#include "ork_internal.h"

namespace orkb {

struct Nf4Tables {
  uint32_t neg0, neg1, pos0, pos1;
};

// prmt.b32 in its default mode, emitted directly: the selector's bit 3 (replicate the sign of the
// selected byte) is part of the NF4 lookup, and __byte_perm only honours the low 3 bits.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

template <int FMT>
__device__ __forceinline__ uint2 expand8(uint32_t w, const Nf4Tables &tb) {
  if constexpr (FMT == FMT_U4) {
    uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;  // k even / k odd, 0..15
    lo |= (lo & 0x08080808u) * 0x1Eu;                             // bit 3 set -> high nibble 0xF
    hi |= (hi & 0x08080808u) * 0x1Eu;
    return make_uint2(prmt(lo, hi, 0x5140), prmt(lo, hi, 0x7362));
  } else {
    const uint32_t x = w ^ 0x88888888u;
    const uint32_t p0 = prmt(tb.pos0, tb.pos1, x), p1 = prmt(tb.pos0, tb.pos1, x >> 16);
    const uint32_t n0 = prmt(tb.neg0, tb.neg1, w), n1 = prmt(tb.neg0, tb.neg1, w >> 16);
    // bytes of n are 0..127: (0x80 - n) ^ 0x80 == -n per byte, with no borrow between bytes
    return make_uint2(p0 | ((0x80808080u - n0) ^ 0x80808080u), p1 | ((0x80808080u - n1) ^ 0x80808080u));
  }
}

inline uint32_t pack4(int a, int b, int c, int d) {
  return (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) | ((uint32_t)(uint8_t)c << 16) |
         ((uint32_t)(uint8_t)d << 24);
}

// the NF4 tables of kNf4Lut for expand8<FMT_NF4>
inline Nf4Tables nf4_tables() {
  const int8_t *L = kNf4Lut;
  return Nf4Tables{pack4(-L[0], -L[1], -L[2], -L[3]), pack4(-L[4], -L[5], -L[6], -L[7]),
                   pack4(L[8], L[9], L[10], L[11]), pack4(L[12], L[13], L[14], L[15])};
}

}  // namespace orkb
