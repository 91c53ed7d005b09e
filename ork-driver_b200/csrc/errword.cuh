// errword.cuh -- one word of mapped, pinned host memory per device that every kernel's error path sets
// besides its own module's flag, so a synchronising call checks for device-side errors with one host
// memory read instead of a copy of every module's flag (which cost ~60 us per call). Each translation
// unit that includes this has its own device pointer to the word, set by its setter once per device.
#pragma once
#include <cuda_runtime.h>

namespace orkb {
namespace {

__device__ unsigned int *g_err_word = nullptr;

__device__ __forceinline__ void err_word_set() {
  unsigned int *w = g_err_word;
  if (w) *(volatile unsigned int *)w = 1u;
}

}  // namespace
}  // namespace orkb

// defines `void name(unsigned int *device_ptr)` (namespace orkb) that points this unit's kernels at the word
#define ORKB_ERR_WORD_SETTER(name)                                              \
  cudaError_t name(unsigned int *device_ptr) {                                  \
    return cudaMemcpyToSymbol(g_err_word, &device_ptr, sizeof device_ptr);      \
  }
