// host_transfer.cu — the rows the host-buffer entry point has to move.
//
// A product reads only the B rows whose column some entry of A holds, and
// writes non-zero values only into the C rows that hold an entry.  On graph
// matrices that is about half of each (R-MAT 2^22: 48% of the columns are
// touched, 52% of the rows are empty), so vcsr_spmm_host moves just those
// rows across PCIe when the caller's buffers are page-locked: a copy kernel
// reads the touched B rows straight from the mapped host buffer and another
// writes the non-empty C rows straight into it, while host threads zero the
// empty C rows.  This file builds the two row lists once per plan (from the
// panel layout in HBM) and provides the copy kernel.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "common.h"
#include "device_prims.cuh"
#include "host_transfer.h"
#include "plan_impl.h"

namespace vcsr {
namespace {

__global__ void mark_cols_kernel(const int *__restrict__ ucol, int64_t n, int N,
                                 int *__restrict__ flag) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int c = ucol[i];
    if (c >= 0 && c < N) flag[c] = 1;
  }
}

// Row r of vector v holds an entry when some union entry of v has bit r of
// its row mask set (R = 1: the vector is not empty).
__global__ void mark_rows_kernel(const int *__restrict__ vec_ptr,
                                 const unsigned *__restrict__ umask, int R, int nvec,
                                 int M, int *__restrict__ flag) {
  for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += gridDim.x * blockDim.x) {
    const int b = vec_ptr[v], e = vec_ptr[v + 1];
    unsigned m = 0;
    if (R == 1) {
      m = e > b ? 1u : 0u;
    } else {
      for (int j = b; j < e; ++j) m |= umask[j];
    }
    for (int r = 0; r < R; ++r) {
      const int row = v * R + r;
      if (row < M) flag[row] = (m >> r) & 1u;
    }
  }
}

__global__ void compact_kernel(const int *__restrict__ flag, const int *__restrict__ pos,
                               int n, int *__restrict__ out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    if (flag[i]) out[pos[i]] = i;
}

// dst[r * ld + o4 + c] = src[r * ld + o4 + c] (float4 units) for every row r
// of rows[0..n) and c < w4.  Four loads are issued before their stores so
// that many reads of the mapped host buffer are in flight per thread.
__global__ void __launch_bounds__(256) copy_rows_kernel(const float4 *__restrict__ src,
                                                         float4 *__restrict__ dst, int64_t ld4,
                                                         const int *__restrict__ rows,
                                                         int n, int o4, int w4) {
  constexpr int U = 4;
  const int64_t total = (int64_t)n * w4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t e0 = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e0 < total;
       e0 += stride * U) {
    float4 v[U];
    int64_t at[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t e = e0 + u * stride;
      at[u] = -1;
      if (e < total) {
        const int64_t i = e / w4;
        at[u] = (int64_t)rows[i] * ld4 + o4 + (e - i * w4);
        v[u] = src[at[u]];
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (at[u] >= 0) dst[at[u]] = v[u];
  }
}

// Device list of the indices i < n with flag[i] != 0, ascending.
vcsr_status compact(const int *flag, int n, int **out, int *count, Scratch &sc,
                    cudaStream_t st) {
  int *pos = nullptr, *total = nullptr;
  VCSR_TRY(sc.get(&pos, n));
  VCSR_TRY(sc.get(&total, 1));
  VCSR_TRY(scan_exclusive<int>(flag, pos, n, total, sc));
  int h = 0;
  VCSR_CUDA(cudaMemcpyAsync(&h, total, sizeof(int), cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  VCSR_CUDA(cudaMalloc(out, sizeof(int) * (size_t)(h > 0 ? h : 1)));
  if (n > 0) compact_kernel<<<std::min((n + 255) / 256, 4096), 256, 0, st>>>(flag, pos, n, *out);
  VCSR_CUDA(cudaGetLastError());
  *count = h;
  return VCSR_OK;
}

}  // namespace

vcsr_status host_transfer_lists(vcsr_plan *p, cudaStream_t st) {
  if (p->xfer_built) return VCSR_OK;
  Scratch sc(st);
  int *cflag = nullptr, *rflag = nullptr;
  VCSR_TRY(sc.get(&cflag, p->N));
  VCSR_TRY(sc.get(&rflag, p->M));
  if (p->N > 0) VCSR_CUDA(cudaMemsetAsync(cflag, 0, sizeof(int) * (size_t)p->N, st));
  if (p->M > 0) VCSR_CUDA(cudaMemsetAsync(rflag, 0, sizeof(int) * (size_t)p->M, st));
  if (p->num_union > 0)
    mark_cols_kernel<<<(int)std::min<int64_t>((p->num_union + 255) / 256, 8192), 256, 0, st>>>(
        p->d_ucol, p->num_union, p->N, cflag);
  if (p->num_vectors > 0)
    mark_rows_kernel<<<std::min((p->num_vectors + 255) / 256, 8192), 256, 0, st>>>(
        p->d_vec_ptr, p->d_umask, p->R, p->num_vectors, p->M, rflag);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(compact(cflag, p->N, &p->d_xcols, &p->n_xcols, sc, st));
  VCSR_TRY(compact(rflag, p->M, &p->d_xrows, &p->n_xrows, sc, st));
  // the empty rows as host ranges [r0, r1)
  std::vector<int> h(p->M > 0 ? p->M : 1);
  if (p->M > 0)
    VCSR_CUDA(cudaMemcpyAsync(h.data(), rflag, sizeof(int) * (size_t)p->M,
                              cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  p->empty_rows.clear();
  for (int r = 0; r < p->M;) {
    if (h[r]) {
      ++r;
      continue;
    }
    int e = r;
    while (e < p->M && !h[e]) ++e;
    p->empty_rows.push_back({r, e});
    r = e;
  }
  p->xfer_built = true;
  return VCSR_OK;
}

vcsr_status copy_rows(const float *src, float *dst, int ld, const int *rows, int n, int o0,
                      int w, int blocks_max, cudaStream_t st) {
  if (n <= 0 || w <= 0) return VCSR_OK;
  const int64_t total4 = (int64_t)n * (w / 4);
  const int64_t want = (total4 + 255) / 256;
  const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>(want, blocks_max));
  copy_rows_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4 *>(src),
                                           reinterpret_cast<float4 *>(dst), ld / 4, rows, n,
                                           o0 / 4, w / 4);
  VCSR_CUDA(cudaGetLastError());
  return VCSR_OK;
}

}  // namespace vcsr
