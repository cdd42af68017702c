// seg_tc.h — the tensor-core segment kernel's launch interface (spmm_seg_tc.cu).
#pragma once
#include <cstddef>

#include <cuda_runtime.h>

#include "common.h"

namespace vcsr {

// Rows of a piece: a piece is at most this many consecutive columns of A
// (B rows), a multiple of 8 (one K = 8 MMA step per 8 rows).
constexpr int kSegPieceRows = 32;

// The segment layout on the device.  Row block k (0 <= k < n_rb) starts at
// row rb_row[k] (a multiple of 16) and owns pieces pp[k] .. pp[k+1]-1.  Piece
// q = {c0, L, koff, 0}: B rows c0 .. c0+L-1 (L a multiple of 8, at most
// kSegPieceRows; rows past N read as zeros) against the row block's values
// in those columns, stored from a + 16*koff as L x 16 FP32 values in the
// tensor core's K-major core-matrix order
//   value(row n, column c0 + k) at (k / 4) * 64 + (n / 8) * 32 + (n % 8) * 4 + k % 4
// (zero where the row has no entry; duplicates summed in CSR order).
// rp/col/val: the whole CSR, for recomputing any output the split product
// leaves non-finite exactly as the CSR sum does.
struct SegView {
  int n_rb = 0;
  const int *rb_row = nullptr;
  const int *pp = nullptr;
  const int4 *pieces = nullptr;
  const float *a = nullptr;
  const int *rp = nullptr, *col = nullptr;
  const float *val = nullptr;
  int M = 0, N = 0, O = 0, ldb = 0, ldc = 0, n_ochunks = 0;
  int accumulate = 0;  // C += product (a residual was written first), else C = product
  int slab3d = 0;      // B's tensor map is 3-D (set by the launcher)
  const float *B = nullptr;
  float *C = nullptr;
  // first failure: wait site | block index << 4; 0 when none (shared with
  // the TF32 panel kernel's error word and describe_tc_error)
  int *err = nullptr;
};

size_t seg_smem_bytes();

// C (+)= the segment product on `st`.  Needs O and ldb multiples of 4 and a
// 16-byte aligned B.
vcsr_status launch_seg_tc(const SegView &V, const float *B, int N, int ldb, float *C, int ldc,
                          int O, cudaStream_t st, int *launches);

}  // namespace vcsr
