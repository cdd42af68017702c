// common.h — error plumbing shared by every translation unit of the library.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <exception>
#include <new>
#include <stdexcept>
#include <string>

#include "vcsr_spmm.h"

namespace vcsr {

// Record a failure in the thread-local message and return its status.
vcsr_status fail(vcsr_status s, const char *fmt, ...)
    __attribute__((format(printf, 2, 3)));
void clear_error();

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Runs an entry point's body and turns a C++ exception of the host code into
// a status, so that none crosses the C ABI: a host allocation that fails
// inside a standard container (std::bad_alloc, or std::length_error for a
// size no container can hold) is VCSR_ERR_ALLOC like a failed malloc.
template <class F>
vcsr_status no_throw(F &&body) {
  try {
    return body();
  } catch (const std::bad_alloc &) {
    return fail(VCSR_ERR_ALLOC, "out of host memory");
  } catch (const std::length_error &) {
    return fail(VCSR_ERR_ALLOC, "out of host memory (size beyond a container's limit)");
  } catch (const std::exception &e) {
    return fail(VCSR_ERR_INVALID, "host exception: %s", e.what());
  }
}

}  // namespace vcsr

#define VCSR_TRY(expr)                        \
  do {                                        \
    vcsr_status _st = (expr);                 \
    if (_st != VCSR_OK) return _st;           \
  } while (0)

#ifdef __CUDACC__
#define VCSR_CUDA(expr)                                                       \
  do {                                                                        \
    cudaError_t _e = (expr);                                                  \
    if (_e != cudaSuccess)                                                    \
      return vcsr::fail(VCSR_ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__,    \
                        #expr, cudaGetErrorString(_e));                       \
  } while (0)
#endif
