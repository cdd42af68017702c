// common.h — error plumbing shared by every translation unit of the library.
#pragma once
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "vcsr_spmm.h"

namespace vcsr {

// Record a failure in the thread-local message and return its status.
vcsr_status fail(vcsr_status s, const char *fmt, ...)
    __attribute__((format(printf, 2, 3)));
void clear_error();

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

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
