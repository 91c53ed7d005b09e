// glue.cuh -- the decode layer's element-wise glue formulas, shared by the multi-launch layer (layer.cu)
// and the persistent one (layer_fused.cu) so both compute the same values the same way. They follow
// ork-driver's CPU glue (src/spine_kernels.h: spine_rmsnorm, spine_quant, spine_silu_glu, spine_rope_neox)
// operation by operation; the files that include them compile with -fmad=false so no multiply-add is
// contracted where the reference rounds twice.
#pragma once
#include <stdint.h>

namespace orkb {
namespace glue {

// per-tensor int8 code of v at scale s (lrintf in the default rounding mode: nearest, ties to even;
// clamped to +-127)
__device__ __forceinline__ int8_t q8(float v, float s) {
  const int q = __float2int_rn(v * s);
  return (int8_t)(q > 127 ? 127 : (q < -127 ? -127 : q));
}

// scale of a per-tensor quantization whose largest magnitude is mx (the reference floors it at 1e-6)
__device__ __forceinline__ float qscale(float mx) { return 127.0f / fmaxf(1e-6f, mx); }

// RMSNorm reciprocal of a row of n values whose squares sum to ss
__device__ __forceinline__ float rms_recip(float ss, int n) { return 1.0f / sqrtf(ss / n + 1e-6f); }

// SwiGLU of one gate / up pair already dequantized
__device__ __forceinline__ float silu_mul(float gi, float ui) { return (gi / (1.0f + expf(-gi))) * ui; }

// RoPE NeoX angle of pair i (of dk / 2) at position pos
__device__ __forceinline__ float rope_angle(int pos, float base, int i, int dk) {
  return pos * powf(base, -2.0f * i / dk);
}

}  // namespace glue
}  // namespace orkb
