// host_transfer.h — row lists and row copies of the host-buffer entry point
// (host_transfer.cu).
#pragma once
#include <cuda_runtime.h>

#include "common.h"

struct vcsr_plan;

namespace vcsr {

// Builds, once per plan, the ascending device lists of the B rows the
// product reads (touched columns) and of the C rows that hold an entry, and
// the host ranges of the empty C rows.  Synchronises `st`.
vcsr_status host_transfer_lists(vcsr_plan *p, cudaStream_t st);

// dst[r][o0 .. o0+w) = src[r][o0 .. o0+w) for r in rows[0..n), rows of `ld`
// floats; ld, o0 and w multiples of 4, src and dst 16-byte aligned.  Either
// side may be mapped page-locked host memory (its device address).  At most
// blocks_max blocks of 256 threads.
vcsr_status copy_rows(const float *src, float *dst, int ld, const int *rows, int n, int o0,
                      int w, int blocks_max, cudaStream_t st);

}  // namespace vcsr
