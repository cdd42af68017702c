// memory.cu — device copies and frees of the ABI containers, and the dense
// generator (host and device fills give identical bits: rng.h).
#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>

#include "common.h"
#include "rng.h"

using vcsr::fail;

namespace {

__global__ void fill_uniform_kernel(float *out, int64_t rows, int64_t cols,
                                    int64_t ld, uint64_t key, float lo,
                                    float hi) {
  const int64_t total = rows * cols;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    out[r * ld + c] = vcsr::uniform_f(vcsr::rnd(key, (uint64_t)i), lo, hi);
  }
}

template <class T>
vcsr_status dev_copy(T **dst, const T *src, int64_t n, cudaStream_t st) {
  *dst = nullptr;
  size_t bytes = sizeof(T) * (size_t)(n > 0 ? n : 1);
  VCSR_CUDA(cudaMalloc((void **)dst, bytes));
  if (n > 0)
    VCSR_CUDA(cudaMemcpyAsync(*dst, src, sizeof(T) * (size_t)n,
                              cudaMemcpyHostToDevice, st));
  return VCSR_OK;
}

template <class T>
vcsr_status host_copy(T **dst, const T *src, int64_t n) {
  *dst = (T *)malloc(sizeof(T) * (size_t)(n > 0 ? n : 1));
  if (!*dst) return fail(VCSR_ERR_ALLOC, "out of host memory");
  if (n > 0)
    VCSR_CUDA(cudaMemcpy(*dst, src, sizeof(T) * (size_t)n, cudaMemcpyDeviceToHost));
  return VCSR_OK;
}

}  // namespace

extern "C" {

vcsr_status vcsr_gen_dense(float *out, int64_t rows, int64_t cols, int64_t ld,
                           uint64_t seed, float lo, float hi, int where,
                           vcsr_stream_t stream) {
  vcsr::clear_error();
  if (!out || rows < 0 || cols < 0 || ld < cols)
    return fail(VCSR_ERR_INVALID, "bad dense fill arguments");
  const uint64_t key = vcsr::stream_key(seed, 0xB0B0ull);
  if (where == VCSR_HOST) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
      for (int64_t c = 0; c < cols; ++c)
        out[r * ld + c] =
            vcsr::uniform_f(vcsr::rnd(key, (uint64_t)(r * cols + c)), lo, hi);
    return VCSR_OK;
  }
  if (rows * cols == 0) return VCSR_OK;
  int dev = 0, sms = 148;
  VCSR_CUDA(cudaGetDevice(&dev));
  VCSR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int64_t blocks = vcsr::ceil_div(rows * cols, 256);
  if (blocks > (int64_t)sms * 32) blocks = (int64_t)sms * 32;
  fill_uniform_kernel<<<(int)blocks, 256, 0, (cudaStream_t)stream>>>(
      out, rows, cols, ld, key, lo, hi);
  VCSR_CUDA(cudaGetLastError());
  return VCSR_OK;
}

vcsr_status vcsr_csr_to_device(const vcsr_csr *h, vcsr_csr *d,
                               vcsr_stream_t stream) {
  vcsr::clear_error();
  if (!h || !d) return fail(VCSR_ERR_INVALID, "null argument");
  std::memset(d, 0, sizeof *d);
  cudaStream_t st = (cudaStream_t)stream;
  VCSR_TRY(dev_copy(&d->row_ptr, h->row_ptr, (int64_t)h->M + 1, st));
  VCSR_TRY(dev_copy(&d->col, h->col, (int64_t)h->nnz, st));
  VCSR_TRY(dev_copy(&d->val, h->val, (int64_t)h->nnz, st));
  d->M = h->M; d->N = h->N; d->nnz = h->nnz;
  return VCSR_OK;
}

void vcsr_csr_free(vcsr_csr *csr, int where) {
  if (!csr) return;
  if (where == VCSR_DEVICE) {
    cudaFree(csr->row_ptr); cudaFree(csr->col); cudaFree(csr->val);
  } else {
    free(csr->row_ptr); free(csr->col); free(csr->val);
  }
  std::memset(csr, 0, sizeof *csr);
}

void vcsr_vcsr_free(vcsr_vcsr *v, int where) {
  if (!v) return;
  void *ptrs[] = {v->group_ptr, v->group_depth, v->group_seg_base,
                  v->group_rows, v->lcol, v->val, v->segment_group_start};
  for (void *p : ptrs) {
    if (where == VCSR_DEVICE) cudaFree(p); else free(p);
  }
  std::memset(v, 0, sizeof *v);
}

vcsr_status vcsr_vcsr_to_host(const vcsr_vcsr *dv, vcsr_vcsr *hv) {
  vcsr::clear_error();
  if (!dv || !hv) return fail(VCSR_ERR_INVALID, "null argument");
  std::memset(hv, 0, sizeof *hv);
  *hv = *dv;
  hv->group_ptr = hv->group_depth = hv->group_seg_base = hv->group_rows =
      hv->lcol = hv->segment_group_start = nullptr;
  hv->val = nullptr;
  const int64_t G = dv->num_groups, P = dv->num_slots, S = dv->num_segments;
  vcsr_status st;
  if ((st = host_copy(&hv->group_ptr, dv->group_ptr, G + 1)) ||
      (st = host_copy(&hv->group_depth, dv->group_depth, G)) ||
      (st = host_copy(&hv->group_seg_base, dv->group_seg_base, G)) ||
      (st = host_copy(&hv->group_rows, dv->group_rows, G * dv->bundle)) ||
      (st = host_copy(&hv->lcol, dv->lcol, P)) ||
      (st = host_copy(&hv->val, dv->val, P)) ||
      (st = host_copy(&hv->segment_group_start, dv->segment_group_start, S + 1))) {
    vcsr_vcsr_free(hv, VCSR_HOST);
    return st;
  }
  return VCSR_OK;
}

}  // extern "C"
