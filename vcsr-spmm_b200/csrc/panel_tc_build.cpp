// panel_tc_build.cpp — split A into dense 16x16 panels (for the tcgen05 TF32
// kernel, spmm_tc.cu) and a residual CSR (for the FP32 row-stationary
// kernel).  A block is a panel when at least `min_nnz` of its 256 positions
// hold entries; duplicate entries inside a panel are summed in CSR order.
#include <algorithm>
#include <cstring>
#include <vector>

#include <omp.h>

#include "common.h"
#include "panel_tc.h"

namespace vcsr {

namespace {

// Round to TF32 (10 explicit mantissa bits), nearest-even; the tensor core
// reads only those bits.
float round_tf32(float x) {
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) != 0x7f800000u) {
    u += 0xFFFu + ((u >> 13) & 1u);
    u &= ~0x1FFFu;
  }
  float y;
  std::memcpy(&y, &u, 4);
  return y;
}

}  // namespace

vcsr_status split_dense_panels(const vcsr_csr &csr, int min_nnz, TcHost *tc,
                               std::vector<int> &r_rp, std::vector<int> &r_col,
                               std::vector<float> &r_val) {
  const int M = csr.M;
  const int nrb = (int)ceil_div(M, 16);
  std::vector<std::vector<int>> dense(nrb);  // sorted dense block columns
  std::vector<int64_t> rcount((size_t)M + 1, 0);
#pragma omp parallel
  {
    std::vector<int> bcs;
#pragma omp for schedule(dynamic, 8)
    for (int i = 0; i < nrb; ++i) {
      const int r0 = 16 * i, r1 = std::min(M, r0 + 16);
      bcs.clear();
      for (int p = csr.row_ptr[r0]; p < csr.row_ptr[r1]; ++p) bcs.push_back(csr.col[p] >> 4);
      std::sort(bcs.begin(), bcs.end());
      auto &d = dense[i];
      for (size_t a = 0; a < bcs.size();) {
        size_t b = a;
        while (b < bcs.size() && bcs[b] == bcs[a]) ++b;
        if ((int)(b - a) >= min_nnz) d.push_back(bcs[a]);
        a = b;
      }
      for (int r = r0; r < r1; ++r) {
        int64_t c = 0;
        for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p)
          if (!std::binary_search(d.begin(), d.end(), csr.col[p] >> 4)) ++c;
        rcount[r + 1] = c;
      }
    }
  }
  r_rp.assign((size_t)M + 1, 0);
  for (int r = 0; r < M; ++r) rcount[r + 1] += rcount[r];
  for (int r = 0; r <= M; ++r) r_rp[r] = (int)rcount[r];
  r_col.assign((size_t)rcount[M], 0);
  r_val.assign((size_t)rcount[M], 0.f);
  tc->rb_row.clear();
  tc->rb_ptr.assign(1, 0);
  tc->blk_col.clear();
  std::vector<int> first(nrb, -1);  // first block index of each row block with panels
  for (int i = 0; i < nrb; ++i) {
    if (dense[i].empty()) continue;
    first[i] = (int)tc->blk_col.size();
    tc->rb_row.push_back(16 * i);
    for (int j : dense[i]) tc->blk_col.push_back(j);
    tc->rb_ptr.push_back((int)tc->blk_col.size());
  }
  tc->blk_val.assign(tc->blk_col.size() * 256, 0.f);
#pragma omp parallel for schedule(dynamic, 8)
  for (int i = 0; i < nrb; ++i) {
    const int r0 = 16 * i, r1 = std::min(M, r0 + 16);
    const auto &d = dense[i];
    for (int r = r0; r < r1; ++r) {
      int o = r_rp[r];
      for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) {
        const int c = csr.col[p];
        auto it = std::lower_bound(d.begin(), d.end(), c >> 4);
        if (it == d.end() || *it != (c >> 4)) {
          r_col[o] = c;
          r_val[o] = csr.val[p];
          ++o;
          continue;
        }
        const int b = first[i] + (int)(it - d.begin());
        const int n = r - r0, k = c & 15;
        tc->blk_val[(size_t)b * 256 + ((k / 4) * 2 + n / 8) * 32 + (n % 8) * 4 + (k % 4)] +=
            csr.val[p];
      }
    }
  }
  for (float &v : tc->blk_val) v = round_tf32(v);
  return VCSR_OK;
}

}  // namespace vcsr
