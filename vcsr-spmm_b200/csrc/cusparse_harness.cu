// cusparse_harness.cu — the vendor baseline, set up once and run many times.
//
// Replaces run_cusparse_spmm (src/kernels.cu:170-235), which made a handle, a
// stream, the descriptors and the buffer on every call and ran
// CUSPARSE_SPMM_ALG_DEFAULT without preprocessing.  Here those are made once
// in vcsr_cusparse_create (with cusparseSpMM_preprocess where the algorithm
// has one), so vcsr_cusparse_run times only cusparseSpMM.
#include <cuda_runtime.h>
#include <cusparse.h>

#include "common.h"

using vcsr::fail;

struct vcsr_cusparse {
  cusparseHandle_t h = nullptr;
  cusparseSpMatDescr_t A = nullptr;
  cusparseDnMatDescr_t B = nullptr, C = nullptr;
  void *buf = nullptr;
  cusparseSpMMAlg_t alg = CUSPARSE_SPMM_ALG_DEFAULT;
  float alpha = 1.f, beta = 0.f;
};

#define VCSR_CUSP(expr)                                                      \
  do {                                                                       \
    cusparseStatus_t _s = (expr);                                            \
    if (_s != CUSPARSE_STATUS_SUCCESS) {                                     \
      vcsr_cusparse_destroy(x);                                              \
      return fail(VCSR_ERR_CUDA, "%s: %s", #expr, cusparseGetErrorString(_s)); \
    }                                                                        \
  } while (0)

extern "C" {

void vcsr_cusparse_destroy(vcsr_cusparse *x) {
  if (!x) return;
  if (x->A) cusparseDestroySpMat(x->A);
  if (x->B) cusparseDestroyDnMat(x->B);
  if (x->C) cusparseDestroyDnMat(x->C);
  if (x->h) cusparseDestroy(x->h);
  cudaFree(x->buf);
  delete x;
}

vcsr_status vcsr_cusparse_create(int M, int N, int nnz, const int *d_row_ptr,
                                 const int *d_col, const float *d_val,
                                 const float *dB, int O, float *dC, int alg,
                                 vcsr_stream_t stream, vcsr_cusparse **out) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!out) return fail(VCSR_ERR_INVALID, "null out");
    *out = nullptr;
    if (M <= 0 || N <= 0 || O <= 0 || nnz < 0)
      return fail(VCSR_ERR_INVALID, "cuSPARSE harness needs M, N, O > 0");
    static const cusparseSpMMAlg_t algs[] = {
        CUSPARSE_SPMM_ALG_DEFAULT, CUSPARSE_SPMM_CSR_ALG1, CUSPARSE_SPMM_CSR_ALG2,
        CUSPARSE_SPMM_CSR_ALG3};
    if (alg < 0 || alg > 3) return fail(VCSR_ERR_INVALID, "alg must be 0..3");
    vcsr_cusparse *x = new vcsr_cusparse();
    x->alg = algs[alg];
    VCSR_CUSP(cusparseCreate(&x->h));
    VCSR_CUSP(cusparseSetStream(x->h, (cudaStream_t)stream));
    VCSR_CUSP(cusparseCreateCsr(&x->A, M, N, nnz, (void *)d_row_ptr, (void *)d_col,
                                (void *)d_val, CUSPARSE_INDEX_32I,
                                CUSPARSE_INDEX_32I, CUSPARSE_INDEX_BASE_ZERO,
                                CUDA_R_32F));
    VCSR_CUSP(cusparseCreateDnMat(&x->B, N, O, O, (void *)dB, CUDA_R_32F,
                                  CUSPARSE_ORDER_ROW));
    VCSR_CUSP(cusparseCreateDnMat(&x->C, M, O, O, (void *)dC, CUDA_R_32F,
                                  CUSPARSE_ORDER_ROW));
    size_t bytes = 0;
    VCSR_CUSP(cusparseSpMM_bufferSize(x->h, CUSPARSE_OPERATION_NON_TRANSPOSE,
                                      CUSPARSE_OPERATION_NON_TRANSPOSE, &x->alpha,
                                      x->A, x->B, &x->beta, x->C, CUDA_R_32F,
                                      x->alg, &bytes));
    if (bytes) {
      cudaError_t e = cudaMalloc(&x->buf, bytes);
      if (e != cudaSuccess) {
        vcsr_cusparse_destroy(x);
        return fail(VCSR_ERR_ALLOC, "cuSPARSE buffer: %s", cudaGetErrorString(e));
      }
    }
    if (x->alg == CUSPARSE_SPMM_CSR_ALG3) {
      VCSR_CUSP(cusparseSpMM_preprocess(x->h, CUSPARSE_OPERATION_NON_TRANSPOSE,
                                        CUSPARSE_OPERATION_NON_TRANSPOSE,
                                        &x->alpha, x->A, x->B, &x->beta, x->C,
                                        CUDA_R_32F, x->alg, x->buf));
    }
    *out = x;
    return VCSR_OK;
  });
}

vcsr_status vcsr_cusparse_run(vcsr_cusparse *x, vcsr_stream_t stream) {
  vcsr::clear_error();
  if (!x) return fail(VCSR_ERR_INVALID, "null handle");
  cusparseStatus_t s = cusparseSetStream(x->h, (cudaStream_t)stream);
  if (s == CUSPARSE_STATUS_SUCCESS)
    s = cusparseSpMM(x->h, CUSPARSE_OPERATION_NON_TRANSPOSE,
                     CUSPARSE_OPERATION_NON_TRANSPOSE, &x->alpha, x->A, x->B,
                     &x->beta, x->C, CUDA_R_32F, x->alg, x->buf);
  if (s != CUSPARSE_STATUS_SUCCESS)
    return fail(VCSR_ERR_CUDA, "cusparseSpMM: %s", cusparseGetErrorString(s));
  return VCSR_OK;
}

}  // extern "C"
