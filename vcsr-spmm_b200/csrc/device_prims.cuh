// device_prims.cuh — device-wide exclusive scan and stable LSD radix sort
// used by the VCSR builder.  Written for this library (no CUB), plain CUDA.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "common.h"

namespace vcsr {

// Stream-ordered device scratch; every allocation is released together (or
// earlier with release()).
struct Scratch {
  cudaStream_t st;
  std::vector<void *> ptrs;
  explicit Scratch(cudaStream_t s) : st(s) {}
  ~Scratch() {
    for (void *p : ptrs) cudaFreeAsync(p, st);
  }
  template <class T>
  vcsr_status get(T **out, int64_t count) {
    size_t bytes = sizeof(T) * (size_t)(count > 0 ? count : 1);
    cudaError_t e = cudaMallocAsync((void **)out, bytes, st);
    if (e != cudaSuccess)
      return fail(VCSR_ERR_ALLOC, "device scratch of %zu bytes: %s", bytes,
                  cudaGetErrorString(e));
    ptrs.push_back(*out);
    return VCSR_OK;
  }
  // frees one allocation now (stream-ordered)
  void release(void *p) {
    for (size_t i = 0; i < ptrs.size(); ++i)
      if (ptrs[i] == p) {
        cudaFreeAsync(p, st);
        ptrs.erase(ptrs.begin() + (long)i);
        return;
      }
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
