// device_prims.cuh — device-wide exclusive scan and stable LSD radix sort
// used by the VCSR builder.  Written for this library (no CUB), plain CUDA.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "common.h"

namespace vcsr {

// Stream-ordered device scratch; every allocation is released together.
struct Scratch {
  cudaStream_t st;
  void *ptrs[64];
  int n = 0;
  explicit Scratch(cudaStream_t s) : st(s) {}
  ~Scratch() {
    for (int i = 0; i < n; ++i) cudaFreeAsync(ptrs[i], st);
  }
  template <class T>
  vcsr_status get(T **out, int64_t count) {
    if (n == 64) return fail(VCSR_ERR_ALLOC, "scratch table full");
    size_t bytes = sizeof(T) * (size_t)(count > 0 ? count : 1);
    cudaError_t e = cudaMallocAsync((void **)out, bytes, st);
    if (e != cudaSuccess)
      return fail(VCSR_ERR_ALLOC, "device scratch of %zu bytes: %s", bytes,
                  cudaGetErrorString(e));
    ptrs[n++] = *out;
    return VCSR_OK;
  }
};

// out[i] = sum of in[0..i) for i < n; *total (device) = sum of all n.
// T is int or long long.  in and out may not alias.
template <class T>
vcsr_status scan_exclusive(const T *in, T *out, int64_t n, T *total,
                           Scratch &sc);

// Stable sort of (keys, vals) by the low `bits` bits of keys, ascending.
// Results land in keys_out / vals_out; the inputs are left untouched.
vcsr_status radix_sort_pairs(const uint32_t *keys_in, const int *vals_in,
                             uint32_t *keys_out, int *vals_out, int64_t n,
                             int bits, Scratch &sc);

}  // namespace vcsr
