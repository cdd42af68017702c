// ref_kernels_shim.cu — C entry points over the reference's GPU launchers in
// src/kernels.cu (csr_spmm_kernel, vcsr_spmm_kernel, the cuSPARSE wrapper),
// compiled for sm_100a from the reference tree by oracle/Makefile into
// oracle/_ref/libvcsr_ref_kernels.so.
//
// TEST INFRASTRUCTURE ONLY: a GPU test runs run_csr_spmm_gpu to pin the
// oracle's CSR semantics against the reference's own kernel, and the kernels
// can be timed as "reference rebuilt for sm_100a" peers.  They are never the
// measured product path.
#include "kernels.cu"

extern "C" {

// run_csr_spmm_gpu (src/kernels.cu:107)
int ref_gpu_csr_spmm(int M, const int *d_rowptr, const int *d_col,
                     const float *d_val, const float *dB, int O, float *dC,
                     void *stream, float *ms) {
  float t = 0.f;
  run_csr_spmm_gpu(M, d_rowptr, d_col, d_val, dB, O, dC, (cudaStream_t)stream,
                   t);
  *ms = t;
  return (int)cudaGetLastError();
}

// run_vcsr_spmm_gpu (src/kernels.cu:120).  The caller must give B at least
// ceil(N/segw)*segw rows: the reference kernel reads whole segments of B.
int ref_gpu_vcsr_spmm(int M, int N, int segw, int bundle, int num_groups,
                      const int *group_ptr, const int *group_depth,
                      const int *group_seg_base, const int *group_rows,
                      long long num_slots, const int *lcol, const float *val,
                      const float *dB, int O, int tileK, float *dC,
                      void *stream, float *ms) {
  VCSRSpMM v;
  v.M = M; v.N = N; v.segw = segw; v.bundle = bundle;
  v.group_ptr.assign(group_ptr, group_ptr + num_groups + 1);
  v.group_depth.assign(group_depth, group_depth + num_groups);
  v.group_seg_base.assign(group_seg_base, group_seg_base + num_groups);
  v.group_rows.assign(group_rows, group_rows + (size_t)num_groups * bundle);
  v.lcol.assign(lcol, lcol + num_slots);
  v.val.assign(val, val + num_slots);
  float t = 0.f;
  run_vcsr_spmm_gpu(v, dB, O, tileK, dC, (cudaStream_t)stream, t);
  *ms = t;
  return (int)cudaGetLastError();
}

// run_cusparse_spmm (src/kernels.cu:170)
float ref_gpu_cusparse_spmm(int M, int N, int nnz, const int *d_rowptr,
                            const int *d_col, const float *d_val,
                            const float *dB, int O, float *dC) {
  return run_cusparse_spmm(M, N, nnz, d_rowptr, d_col, d_val, dB, O, dC);
}

}  // extern "C"
