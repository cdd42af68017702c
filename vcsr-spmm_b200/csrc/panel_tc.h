// panel_tc.h — host-side split of A into dense 16x16 TF32 panels and a
// residual CSR (layout of the panels: spmm_tc.h).
#pragma once
#include <vector>

#include "vcsr_spmm.h"

namespace vcsr {

struct TcHost {
  std::vector<int> rb_row;     // first row of each row block with panels
  std::vector<int> rb_ptr;     // block offsets per such row block (+1)
  std::vector<int> blk_col;    // block column of each panel
  std::vector<float> blk_val;  // 256 TF32 values per panel, core-matrix order
};

// A block is a panel when at least `min_nnz` of its 256 positions hold
// entries; the entries of the other blocks go to the residual CSR
// (r_rp, r_col, r_val), in their CSR order.
vcsr_status split_dense_panels(const vcsr_csr &csr, int min_nnz, TcHost *tc,
                               std::vector<int> &r_rp, std::vector<int> &r_col,
                               std::vector<float> &r_val);

}  // namespace vcsr
