// ref_shim.cpp — C entry points over the reference's own header-only host
// path, compiled from the reference tree (include/mmio.hpp, include/csr.hpp,
// include/vcsr.hpp) by oracle/Makefile into oracle/_ref/libvcsr_ref.so.
//
// TEST INFRASTRUCTURE ONLY: used by tests/golden/make_golden.py to record the
// reference's outputs and by tests that pin the oracle against them.  The
// reference sources are included from where they lie; nothing is copied.
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "mmio.hpp"
#include "csr.hpp"
#include "vcsr.hpp"

static thread_local std::string g_err;

template <class T>
static T *dup(const std::vector<T> &v) {
  T *p = (T *)std::malloc(sizeof(T) * (v.size() ? v.size() : 1));
  if (!v.empty()) std::memcpy(p, v.data(), sizeof(T) * v.size());
  return p;
}

extern "C" {

const char *ref_last_error(void) { return g_err.c_str(); }
void ref_free(void *p) { std::free(p); }

// read_matrix_market_coo (include/mmio.hpp:22)
int ref_read_mtx(const char *path, int *M, int *N, int *nnz, int **rows,
                 int **cols, float **vals) {
  try {
    COO c = read_matrix_market_coo(path);
    *M = c.M; *N = c.N; *nnz = (int)c.vals.size();
    *rows = dup(c.rows); *cols = dup(c.cols); *vals = dup(c.vals);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 4;
  }
}

// coo_to_csr (include/csr.hpp:16)
int ref_coo_to_csr(int M, int N, int nnz, const int *rows, const int *cols,
                   const float *vals, int **row_ptr, int **col, float **val) {
  try {
    COO c; c.M = M; c.N = N;
    c.rows.assign(rows, rows + nnz);
    c.cols.assign(cols, cols + nnz);
    c.vals.assign(vals, vals + nnz);
    CSR r = coo_to_csr(c);
    *row_ptr = dup(r.row_ptr); *col = dup(r.col); *val = dup(r.val);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 8;
  }
}

// csr_to_vcsr_spmm (include/vcsr.hpp:25)
int ref_csr_to_vcsr(int M, int N, const int *row_ptr, const int *col,
                    const float *val, int segw, int bundle, int *num_groups,
                    long long *num_slots, int **group_ptr, int **group_depth,
                    int **group_seg_base, int **group_rows, int **lcol,
                    float **vals) {
  try {
    CSR c; c.M = M; c.N = N; c.nnz = row_ptr[M];
    c.row_ptr.assign(row_ptr, row_ptr + M + 1);
    c.col.assign(col, col + c.nnz);
    c.val.assign(val, val + c.nnz);
    VCSRSpMM v = csr_to_vcsr_spmm(c, segw, bundle);
    *num_groups = (int)v.group_depth.size();
    *num_slots = (long long)v.lcol.size();
    *group_ptr = dup(v.group_ptr); *group_depth = dup(v.group_depth);
    *group_seg_base = dup(v.group_seg_base); *group_rows = dup(v.group_rows);
    *lcol = dup(v.lcol); *vals = dup(v.val);
    return 0;
  } catch (const std::exception &e) {
    g_err = e.what();
    return 1;
  }
}

}  // extern "C"
