// pack.h -- host pack-time helpers (pack.cpp).
#pragma once
#include <functional>
#include <stddef.h>
#include <stdint.h>

namespace orkb {

constexpr uint32_t kO4N1Magic = 0x4F344E31u;  // 'O','4','N','1' (ork-driver src/npu/internal.h:584)
constexpr uint32_t kO4N1Version = 1u;         // == ork_pack_format_version()
constexpr size_t kO4N1Header = 20;            // {u32 magic, u32 version, i32 K, i32 N, u32 quant_kind}

inline size_t o4n1_bytes(int K, int N) { return kO4N1Header + (size_t)N * 4 + (size_t)K * N / 2; }

void parallel_for(int n, const std::function<void(int, int)> &fn);
void quant_i8_f32(int K, int N, const float *f32, int8_t *codes_nk, float *bscale);
void quant_i4a8(int K, int N, const float *f32, const float *imatrix, int nf4, int sr, uint8_t *nib_nk,
                float *bscale);
float i4a8_qerr(int K, int N, const float *f32, const float *imatrix, int nf4, const uint8_t *nib_nk,
                const float *bscale);
void transpose_bytes(const void *src_kn, void *dst_nk, int K, int N, int esize);
void pack_w4a4(const int8_t *B_kn, int K, int N, uint8_t *nib_nk);
void o4n1_header(uint8_t *p, int K, int N, int quant_kind);
bool o4n1_check(const void *blob, size_t n, int K, int N, int *quant_kind);

}  // namespace orkb
