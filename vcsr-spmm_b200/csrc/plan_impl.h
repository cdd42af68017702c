// plan_impl.h — the plan object shared by the plan's translation units
// (plan.cu: build and run; plan_io.cu: save and load).
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <utility>
#include <vector>

#include "common.h"

struct vcsr_plan {
  int M = 0, N = 0, nnz = 0;
  vcsr_plan_params params{};
  int device = 0;
  // vector panels on the device
  int R = 1;
  int num_vectors = 0;
  int64_t num_union = 0;
  int chunk = 0;
  int n_units = 0, n_split_units = 0, n_split_vectors = 0;
  int *d_ucol = nullptr;
  float *d_uval = nullptr;
  unsigned *d_umask = nullptr;  // R > 1: which rows of a vector hold each union entry
  int4 *d_units = nullptr;
  int4 *d_batches = nullptr;
  int *d_long = nullptr, *d_vec_ptr = nullptr;
  int n_batches = 0, n_long = 0;
  // the long units ordered by their first union column (launches over the
  // whole matrix; d_long keeps vector order for the row panels)
  int *d_long_col = nullptr;
  int2 *d_parts = nullptr;
  int2 *d_svecs = nullptr;
  float *d_partials = nullptr;
  int *d_counters = nullptr;
  int pstride = 0, counter_stride = 0;
  int64_t panel_bytes = 0;
  // optional segment-major VCSR (include/vcsr.hpp:12-23 layout)
  bool has_ref = false;
  vcsr_vcsr ref{};
  // dense 16x16 panels on the tcgen05 TF32 path (VCSR_PLAN_TF32_PANELS)
  int *d_rb_row = nullptr, *d_rb_ptr = nullptr, *d_blk_col = nullptr, *d_err = nullptr;
  float *d_blk_val = nullptr;
  int n_panel_rb = 0, n_panel_blocks = 0;
  // tensor-core segments (VCSR_PLAN_TC_SEGMENTS, seg_tc.h): row blocks with
  // pieces, the pieces, their dense tiles, and the whole CSR for recomputing
  // non-finite outputs; seg_only: no residual, the segment kernel writes C
  int *d_seg_rb_row = nullptr, *d_seg_pp = nullptr, *d_seg_rp = nullptr, *d_seg_col = nullptr;
  int4 *d_seg_pieces = nullptr;
  float *d_seg_a = nullptr, *d_seg_val = nullptr;
  int n_seg_rb = 0, n_seg_pieces = 0, seg_rows = 0, seg_min_run = 0;
  bool seg_only = false;
  // test hook (vcsr_plan_test_withhold_signal): the next TF32 panel launch
  // withholds one barrier signal; one-shot
  mutable std::atomic<int> tc_inject{0};
  int64_t panel_nnz = 0;
  // side stream and events for running long units beside short ones
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  // host-buffer entry point: staging buffers, the download stream and one
  // event per column chunk
  float *d_stage_B = nullptr, *d_stage_C = nullptr;
  cudaStream_t down = nullptr, comp = nullptr;
  std::vector<cudaEvent_t> chunk_done;
  // row panels for the host entry point's row pipeline: vectors
  // [v0, v1) = batches [b0, b1) + long units [l0, l1); the panel's rows read
  // B rows up to col_max
  struct RowPanel {
    int row0, row1, b0, b1, l0, l1, col_max;
  };
  std::vector<RowPanel> rpanels;
  size_t stage_B = 0, stage_C = 0;
  // rows the host entry point moves with page-locked buffers
  // (host_transfer.h): touched B rows, C rows holding an entry, and the
  // ranges [r0, r1) of empty C rows that host threads zero
  bool xfer_built = false;
  int *d_xcols = nullptr, *d_xrows = nullptr;
  int n_xcols = 0, n_xrows = 0;
  std::vector<std::pair<int, int>> empty_rows;
  double build_ms = 0;
};

namespace vcsr {

// Device copy of a host vector (at least one element is allocated), enqueued
// on `st`; adds the bytes to *bytes.
template <class T>
vcsr_status upload(T **dst, const std::vector<T> &src, cudaStream_t st,
                   int64_t *bytes) {
  const size_t n = src.size() ? src.size() : 1;
  VCSR_CUDA(cudaMalloc((void **)dst, sizeof(T) * n));
  if (!src.empty())
    VCSR_CUDA(cudaMemcpyAsync(*dst, src.data(), sizeof(T) * src.size(),
                              cudaMemcpyHostToDevice, st));
  if (bytes) *bytes += (int64_t)(sizeof(T) * n);
  return VCSR_OK;
}

// Frees everything the plan owns on the device (not the object itself).
void plan_release(vcsr_plan *p);

// The device state that follows from the uploaded layout: the side stream
// and events (long units beside short ones) and the split-row scratch.
vcsr_status plan_finish(vcsr_plan *p, cudaStream_t st);

}  // namespace vcsr
