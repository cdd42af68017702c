// panel_gpu.h — the plan's layout built on the GPU (panel_gpu_build.cu).
//
// The reference builds its VCSR on the host (include/vcsr.hpp:25-109: per-
// segment lists, std::sort of every row per segment).  Here every step of the
// engine's own layout runs as device kernels over the CSR in HBM: validation,
// the per-row sort when rows are unsorted, the dense 16x16 TF32 panel split,
// the vector height, the union of each vector's rows with its row masks, the
// nnz-balanced units and split parts, the batches and long units, and the row
// panels of the host pipeline.  The layout is bit-identical to the host
// builder's (panel_build.cpp, kept for that comparison).
#pragma once
#include <cuda_runtime.h>

#include "common.h"
#include "plan_impl.h"

namespace vcsr {

// Checks a device CSR (row_ptr from 0 to nnz and non-decreasing, columns in
// [0, N)) and returns in *out a device CSR whose rows are sorted by column,
// stably: `d` itself when it already is (*owned = false), else a private
// sorted copy (*owned = true; free with vcsr_csr_free(out, VCSR_DEVICE)).
vcsr_status device_sorted_csr(const vcsr_csr &d, vcsr_csr *out, bool *owned, cudaStream_t st);

// Builds p's device layout from a validated device CSR with sorted rows
// (the layout fields of vcsr_plan: vector panels, units, batches, long
// units, split bookkeeping, row panels, and with VCSR_PLAN_TF32_PANELS the
// dense panels and their residual).  p->M/N/nnz/params are set by the caller.
vcsr_status build_plan_layout_device(vcsr_plan *p, const vcsr_csr &d, int sms,
                                     cudaStream_t st);

// p->d_long_col: the long units (whole-warp units and split parts) ordered by
// the first union column they read, ties in vector order.  Warps that run at
// the same time then read B rows of nearby columns, so the parts of the
// longest rows (narrow column spans) share B rows in L2.  Measured on B200,
// R-MAT 2^22 at O = 256: 6.52 -> 6.15 ms per product; power-law O=64 106.5 ->
// 108.5 us.  Results are unchanged: split parts are summed in part order
// whatever order they run in.
vcsr_status order_long_by_column(vcsr_plan *p, cudaStream_t st);

}  // namespace vcsr
