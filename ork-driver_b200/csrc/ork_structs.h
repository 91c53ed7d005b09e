// ork_structs.h -- the context and weight objects behind the opaque handles of include/ork_npu.h
// (shared by the C ABI translation units; not installed).
#pragma once
#include <cuda_runtime.h>

#include <stddef.h>
#include <stdint.h>

#include "ork_internal.h"

struct ork_npu {
  int device = 0;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  void *dA = nullptr;
  size_t capA = 0;
  void *dC = nullptr;
  size_t capC = 0;
  bool pdl = true;
  int force_route = -1;
  uint64_t launches = 0;
};

struct ork_w {
  ork_npu *ctx = nullptr;
  int K = 0, N = 0;
  int fmt = orkb::FMT_I8;
  int dtype = orkb::DT_I8;
  int quant_kind = 0;
  bool int4_store = false;  // an ork_i4a8 weight: carries bscale and dumps as O4N1
  void *d = nullptr;
  size_t bytes = 0;
  float *bscale = nullptr;
};

namespace orkb {
// 0 = CUDA-core GEMV, 1 = tcgen05 GEMM, -1 = no kernel for this weight and M.
int route_for(const ork_npu *c, const ork_w *w, int M);
// Sticky device-side error flags (a bounded wait that expired); cleared when read.
bool device_error();
}  // namespace orkb
