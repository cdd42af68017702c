// spmm_kernels.h — internal launch interface of the SpMM kernels.
#pragma once
#include <cuda_runtime.h>

#include "common.h"

namespace vcsr {

// Device view of a vector-panel layout (panel.h) or, with row_ptr set and
// R = 1, of a plain CSR (one unit per row, never split).
struct PanelDevView {
  const int *ucol = nullptr;
  const float *uval = nullptr;
  // R > 1: per union column, bit r set when row r of the vector holds the
  // entry (the others are padding zeros).  Read only when a padded sum came
  // out NaN and the rows are recomputed over their own entries.
  const unsigned *umask = nullptr;
  const int4 *units = nullptr;    // {vector, begin, end, split slot or -1}
  const int *row_ptr = nullptr;   // CSR mode only
  int n_units = 0;
  const int4 *batches = nullptr;  // {v0, v1, first union column, end}: consecutive
  int n_batches = 0;              // short vectors walked by one sub-warp each
  const int *vec_ptr = nullptr;   // union offsets of the vectors (num_vectors + 1)
  const int *long_idx = nullptr;  // units walked by a whole warp
  int n_long = 0;
  const int2 *parts = nullptr;    // per split slot: {split vector, part}
  const int2 *svecs = nullptr;    // per split vector: {first slot, nparts}
  float *partials = nullptr;      // split slots x R x pstride floats
  int *counters = nullptr;        // split vectors x counter_stride tickets
  int pstride = 0;                // = the plan's max_O
  int counter_stride = 0;         // >= O-tiles of any launch shape
  int n_split_units = 0;
  int M = 0;
  int R = 1;
  int accumulate = 0;  // C += A * B instead of C = A * B
};

// Element type of B: FP32 as stored, or 16-bit values widened to FP32 as they
// are loaded (exactly), the sums being FP32 either way.
enum class BType { kF32, kBF16, kF16 };

struct LaunchShape {
  int VW;        // floats per access: 4 (128-bit) or 1
  int NV;        // accesses per lane per O-tile
  int lshift;    // log2 of lanes per sub-warp
  int W;         // O columns per tile
  int n_otiles;  // tiles over O
};

LaunchShape pick_shape(int O, int R, bool vec4);

// Launches the long-unit kernel (on `side`, forked from and joined back to
// `st` with the two events, when there is short work too) and the short-work
// kernel (on `st`).  side may be null: then both run on `st`.  B holds FP32
// values, or BF16 ones with bf16 = true (widened to FP32 as they are loaded;
// not for the plain-CSR rowptr form).  reserve_sms: the grids are sized for
// that many fewer SMs, so that every block can be resident beside kernels
// that hold blocks on that many SMs (the host entry point's copy kernels).
vcsr_status launch_panel_spmm(const PanelDevView &P, bool rowptr,
                              const void *B, int ldb, float *C, int ldc, int O,
                              cudaStream_t st, int *launches, cudaStream_t side,
                              cudaEvent_t fork, cudaEvent_t join,
                              BType bt = BType::kF32, int reserve_sms = 0);

}  // namespace vcsr
