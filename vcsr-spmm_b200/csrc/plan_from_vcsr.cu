// plan_from_vcsr.cu — the engine's plan for the matrix a reference-format
// VCSRSpMM holds (include/vcsr.hpp:12-23).  The reference's launcher,
// run_vcsr_spmm_gpu (src/kernels.cu:120-167), is handed that format; the
// drop-in C++ launcher turns it back into CSR entries on the GPU and runs the
// engine's layout and kernels instead of the segment-major kernel.
//   1. per group: depth >= 0, group_ptr[g+1] - group_ptr[g] == depth * bundle,
//      group_ptr[0] == 0 and group_ptr[G] == num_slots, seg_base in [0, N);
//   2. per slot: its group (binary search in group_ptr), its lane
//      (slot - group_ptr[g]) % bundle and row group_rows[g * bundle + lane];
//      the slot is an entry when row >= 0 and lcol >= 0 -- the reference
//      pads depth with lcol = -1 / val = 0 (vcsr.hpp:82-97) and the last group
//      of a segment with rows -1 -- at column seg_base + lcol;
//   3. an exclusive scan of the entry flags compacts (row, column, value);
//   4. a stable radix sort by row gives CSR order (the entries of a row in
//      slot order: segment, then depth); row_ptr[r] = the first sorted entry
//      whose row is >= r;
//   5. vcsr_plan_create on that device CSR (it sorts each row by column).
#include <cuda_runtime.h>

#include <climits>

#include "common.h"
#include "device_prims.cuh"

using vcsr::fail;

namespace vcsr {
namespace {

constexpr int kThreads = 256;

int grid_of(int64_t n) {
  const int64_t b = ceil_div(n > 0 ? n : 1, kThreads);
  return (int)(b > 148 * 64 ? 148 * 64 : b);
}

// bit 0: group_ptr inconsistent with depth * bundle or the slot count,
// bit 1: a segment base outside [0, N)
__global__ void check_groups_kernel(int G, int bundle, int N, int64_t num_slots,
                                    const int *__restrict__ group_ptr,
                                    const int *__restrict__ depth,
                                    const int *__restrict__ seg_base, int *bad) {
  int flags = 0;
  for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < G; g += gridDim.x * blockDim.x) {
    const int d = depth[g];
    const int64_t span = (int64_t)group_ptr[g + 1] - group_ptr[g];
    if (d < 0 || span != (int64_t)d * bundle) flags |= 1;
    if (g == 0 && group_ptr[0] != 0) flags |= 1;
    if (g == G - 1 && (int64_t)group_ptr[G] != num_slots) flags |= 1;
    if (seg_base[g] < 0 || seg_base[g] >= N) flags |= 2;
  }
  if (flags) atomicOr(bad, flags);
}

// the group holding slot s: the last g with group_ptr[g] <= s
__device__ __forceinline__ int group_of(const int *group_ptr, int G, int s) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (group_ptr[mid] <= s) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// entry flags per slot; bit 2: a row outside [-1, M), bit 3: an lcol
// outside [-1, segw) or a column past N
__global__ void flag_slots_kernel(int P, int G, int bundle, int segw, int M, int N,
                                  const int *__restrict__ group_ptr,
                                  const int *__restrict__ seg_base,
                                  const int *__restrict__ group_rows,
                                  const int *__restrict__ lcol, int *flag, int *bad) {
  int flags = 0;
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < P; s += gridDim.x * blockDim.x) {
    const int g = group_of(group_ptr, G, s);
    const int lane = (s - group_ptr[g]) % bundle;
    const int row = group_rows[(int64_t)g * bundle + lane];
    const int lc = lcol[s];
    if (row < -1 || row >= M) flags |= 4;
    if (lc < -1 || lc >= segw || (lc >= 0 && (int64_t)seg_base[g] + lc >= N)) flags |= 8;
    flag[s] = (row >= 0 && lc >= 0) ? 1 : 0;
  }
  if (flags) atomicOr(bad, flags);
}

__global__ void compact_kernel(int P, int G, int bundle, const int *__restrict__ group_ptr,
                               const int *__restrict__ seg_base,
                               const int *__restrict__ group_rows,
                               const int *__restrict__ lcol, const float *__restrict__ val,
                               const int *__restrict__ flag, const int *__restrict__ idx,
                               uint32_t *key, int *ord, int *col, float *v) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < P; s += gridDim.x * blockDim.x) {
    if (!flag[s]) continue;
    const int g = group_of(group_ptr, G, s);
    const int lane = (s - group_ptr[g]) % bundle;
    const int i = idx[s];
    key[i] = (uint32_t)group_rows[(int64_t)g * bundle + lane];
    ord[i] = i;
    col[i] = seg_base[g] + lcol[s];
    v[i] = val[s];
  }
}

__global__ void gather_kernel(int nnz, const int *__restrict__ perm,
                              const int *__restrict__ col_in, const float *__restrict__ val_in,
                              int *col_out, float *val_out) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nnz; i += gridDim.x * blockDim.x) {
    const int j = perm[i];
    col_out[i] = col_in[j];
    val_out[i] = val_in[j];
  }
}

// row_ptr[r] = number of sorted entries whose row is < r, for r in [0, M]
__global__ void row_ptr_kernel(int M, int nnz, const uint32_t *__restrict__ rows, int *row_ptr) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r <= M; r += gridDim.x * blockDim.x) {
    int lo = 0, hi = nnz;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((int)rows[mid] < r) lo = mid + 1; else hi = mid;
    }
    row_ptr[r] = lo;
  }
}

int bits_of(uint32_t v) {
  int b = 0;
  while (b < 32 && (v >> b)) ++b;
  return b > 0 ? b : 1;
}

template <class T>
vcsr_status to_device(const T *src, int64_t n, int where, T **dst, Scratch &sc) {
  if (where == VCSR_DEVICE || n == 0) {
    *dst = const_cast<T *>(src);
    return VCSR_OK;
  }
  VCSR_TRY(sc.get(dst, n));
  VCSR_CUDA(cudaMemcpyAsync(*dst, src, sizeof(T) * (size_t)n, cudaMemcpyHostToDevice, sc.st));
  return VCSR_OK;
}

}  // namespace
}  // namespace vcsr

extern "C" vcsr_status vcsr_plan_from_vcsr(const vcsr_vcsr *v, int where,
                                           const vcsr_plan_params *params, vcsr_plan **out,
                                           vcsr_stream_t stream) {
  using namespace vcsr;
  return no_throw([&]() -> vcsr_status {
    clear_error();
    if (!v || !params || !out) return fail(VCSR_ERR_INVALID, "null argument");
    *out = nullptr;
    if (where != VCSR_HOST && where != VCSR_DEVICE)
      return fail(VCSR_ERR_INVALID, "where must be VCSR_HOST or VCSR_DEVICE");
    if (v->M < 0 || v->N < 0 || v->num_groups < 0 || v->num_slots < 0)
      return fail(VCSR_ERR_INVALID, "negative size in the VCSR");
    if (v->segw <= 0 || v->bundle <= 0) return fail(VCSR_ERR_INVALID, "segw and bundle must be > 0");
    if (v->num_slots > INT_MAX)
      return fail(VCSR_ERR_UNSUPPORTED, "%lld slots exceed 32-bit entry indices",
                  (long long)v->num_slots);
    const int G = v->num_groups, P = (int)v->num_slots, M = v->M, N = v->N;
    if ((int64_t)G * v->bundle > INT_MAX)
      return fail(VCSR_ERR_UNSUPPORTED, "group_rows of %lld entries exceed 32-bit indices",
                  (long long)G * v->bundle);
    if (G > 0 && (!v->group_ptr || !v->group_depth || !v->group_seg_base || !v->group_rows))
      return fail(VCSR_ERR_INVALID, "null group array");
    if (P > 0 && (!v->lcol || !v->val)) return fail(VCSR_ERR_INVALID, "null slot array");
    if (G == 0 && P > 0) return fail(VCSR_ERR_INVALID, "%d slots but no groups", P);
    cudaStream_t st = (cudaStream_t)stream;
    Scratch sc(st);
    const int *gp = nullptr, *gd = nullptr, *gs = nullptr, *gr = nullptr, *lc = nullptr;
    const float *gv = nullptr;
    VCSR_TRY(to_device(v->group_ptr, G > 0 ? (int64_t)G + 1 : 0, where, const_cast<int **>(&gp), sc));
    VCSR_TRY(to_device(v->group_depth, G, where, const_cast<int **>(&gd), sc));
    VCSR_TRY(to_device(v->group_seg_base, G, where, const_cast<int **>(&gs), sc));
    VCSR_TRY(to_device(v->group_rows, (int64_t)G * v->bundle, where, const_cast<int **>(&gr), sc));
    VCSR_TRY(to_device(v->lcol, P, where, const_cast<int **>(&lc), sc));
    VCSR_TRY(to_device(v->val, P, where, const_cast<float **>(&gv), sc));
    int *bad = nullptr, *flag = nullptr, *idx = nullptr, *count = nullptr;
    VCSR_TRY(sc.get(&bad, 1));
    VCSR_TRY(sc.get(&count, 1));
    VCSR_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), st));
    int h[2] = {0, 0};
    if (G > 0) {
      check_groups_kernel<<<grid_of(G), kThreads, 0, st>>>(G, v->bundle, N, v->num_slots, gp, gd,
                                                           gs, bad);
      VCSR_CUDA(cudaGetLastError());
      VCSR_CUDA(cudaMemcpyAsync(h, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      if (h[0] & 1)
        return fail(VCSR_ERR_INVALID, "group_ptr does not match group_depth * bundle and the"
                                      " slot count");
      if (h[0] & 2) return fail(VCSR_ERR_INVALID, "a group_seg_base is outside [0, N)");
    }
    int nnz = 0;
    vcsr_csr dev{M, N, 0, nullptr, nullptr, nullptr};
    int *row_ptr = nullptr, *col = nullptr;
    float *val = nullptr;
    VCSR_TRY(sc.get(&row_ptr, (int64_t)M + 1));
    if (P > 0) {
      VCSR_TRY(sc.get(&flag, P));
      VCSR_TRY(sc.get(&idx, P));
      flag_slots_kernel<<<grid_of(P), kThreads, 0, st>>>(P, G, v->bundle, v->segw, M, N, gp, gs,
                                                         gr, lc, flag, bad);
      VCSR_CUDA(cudaGetLastError());
      VCSR_TRY(scan_exclusive<int>(flag, idx, P, count, sc));
      VCSR_CUDA(cudaMemcpyAsync(h, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaMemcpyAsync(h + 1, count, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      if (h[0] & 4) return fail(VCSR_ERR_RANGE, "a group_rows entry is outside [-1, M)");
      if (h[0] & 8) return fail(VCSR_ERR_RANGE, "an lcol is outside [-1, segw) or past column N");
      nnz = h[1];
    }
    if (nnz > 0) {
      uint32_t *key = nullptr, *key_sorted = nullptr;
      int *ord = nullptr, *perm = nullptr, *col_c = nullptr;
      float *val_c = nullptr;
      VCSR_TRY(sc.get(&key, nnz));
      VCSR_TRY(sc.get(&key_sorted, nnz));
      VCSR_TRY(sc.get(&ord, nnz));
      VCSR_TRY(sc.get(&perm, nnz));
      VCSR_TRY(sc.get(&col_c, nnz));
      VCSR_TRY(sc.get(&val_c, nnz));
      VCSR_TRY(sc.get(&col, nnz));
      VCSR_TRY(sc.get(&val, nnz));
      compact_kernel<<<grid_of(P), kThreads, 0, st>>>(P, G, v->bundle, gp, gs, gr, lc, gv, flag,
                                                      idx, key, ord, col_c, val_c);
      VCSR_CUDA(cudaGetLastError());
      VCSR_TRY(radix_sort_pairs(key, ord, key_sorted, perm, nnz, bits_of((uint32_t)M), sc));
      gather_kernel<<<grid_of(nnz), kThreads, 0, st>>>(nnz, perm, col_c, val_c, col, val);
      VCSR_CUDA(cudaGetLastError());
      row_ptr_kernel<<<grid_of((int64_t)M + 1), kThreads, 0, st>>>(M, nnz, key_sorted, row_ptr);
    } else {
      VCSR_CUDA(cudaMemsetAsync(row_ptr, 0, sizeof(int) * ((size_t)M + 1), st));
    }
    VCSR_CUDA(cudaGetLastError());
    dev.nnz = nnz;
    dev.row_ptr = row_ptr;
    dev.col = col;
    dev.val = val;
    // the plan is built from (and no longer needs) this CSR; the scratch is
    // freed in stream order after it
    return vcsr_plan_create(&dev, VCSR_DEVICE, params, out, stream);
  });
}
