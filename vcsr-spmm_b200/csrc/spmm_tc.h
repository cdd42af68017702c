// spmm_tc.h — the tcgen05 TF32 dense-panel kernel's launch interface.
#pragma once
#include <cstddef>

#include <cuda.h>
#include <cuda_runtime.h>

#include "common.h"

namespace vcsr {

// Dense 16x16 panels of A on the device.  Row block k (0 <= k < n_rb) starts
// at row rb_row[k] and owns blocks rb_ptr[k] .. rb_ptr[k+1]-1 (at least one);
// block b covers columns 16*blk_col[b] .. +15 and its 256 values sit at
// blk_val + 256*b in the K-major core-matrix order
//   value(row n, column k) at ((k / 4) * 2 + n / 8) * 32 + (n % 8) * 4 + k % 4,
// rounded to TF32.
struct TcView {
  int n_rb = 0;
  const int *rb_row = nullptr;
  const int *rb_ptr = nullptr;
  const int *blk_col = nullptr;
  const float *blk_val = nullptr;
  int M = 0, O = 0, ldc = 0, n_ochunks = 0;
  // B's tensor map is 3-D (32 floats, rows, 32-float chunks): one copy per
  // slab instead of four (set by the launcher when O is a multiple of 32)
  int slab3d = 0;
  float *C = nullptr;
  // first failure: wait site (1 stage full, 2 stage empty, 3 accumulator
  // full, 4 accumulator free) | block index << 4; 0 when none
  int *err = nullptr;
  // test hook: block 0 withholds its first accumulator-ready signal, and the
  // epilogue's wait for it gives up after a short bounded poll
  int inject = 0;
};

size_t tc_smem_bytes();

// cuTensorMapEncodeTiled, found once through the runtime's driver entry
// point (the library does not link the driver library).
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);
vcsr_status tensor_map_encoder(EncodeTiledFn *out);

// Text for a nonzero error word.
void describe_tc_error(int word, char *buf, size_t n);

// C[rows of the panels] += panels * B, on `st` (C must already hold the
// other entries' product).  Needs O and ldb multiples of 4, B 16-byte aligned.
vcsr_status launch_tc_panels(const TcView &V, const float *B, int N, int ldb, float *C,
                             int ldc, int O, cudaStream_t st, int *launches);

}  // namespace vcsr
