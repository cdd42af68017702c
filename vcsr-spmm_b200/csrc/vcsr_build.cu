// vcsr_build.cu — GPU construction of the segment-major VCSR
// (include/vcsr.hpp:12-23 layout) from a device CSR, replacing the host
// builder csr_to_vcsr_spmm (include/vcsr.hpp:25-109).
//
// The reference walks S*M (segment,row) lists on one host thread.  Here only
// the non-empty (row, segment) pairs exist ("entries", at most nnz):
//   1. head flags: entry p starts a pair when it opens its row or its column
//      segment differs from entry p-1 (rows are sorted by column);
//   2. exclusive scan of the flags numbers the pairs; each pair records row,
//      segment, first entry and count;
//   3. stable radix sort by segment gives each segment's rows ascending;
//      stable radix sort by (segment, count descending) gives the packing
//      order of vcsr.hpp:56-59 with ties by row ascending;
//   4. groups: segment s has ceil(nz_s / bundle) groups (later groups of the
//      reference have depth 0 and are skipped, vcsr.hpp:70); depth = count of
//      the group's first row; group_ptr = scan of depth * bundle;
//   5. the last group of a segment is filled with the smallest rows that have
//      no entry in the segment (the reference takes rows of count 0 in
//      whatever order std::sort left them), lanes past row M-1 get -1;
//   6. one warp per group writes group_rows and the depth-major slots
//      (slot = group_ptr[g] + d*bundle + lane, vcsr.hpp:82-97).
#include <cuda_runtime.h>

#include <cstring>

#include "common.h"
#include "device_prims.cuh"

using vcsr::fail;

namespace vcsr {
namespace {

__device__ __forceinline__ int row_of(const int *row_ptr, int M, int p) {
  // last row r with row_ptr[r] <= p (rows may be empty)
  int lo = 0, hi = M - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (row_ptr[mid] <= p) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// bit 0: row_ptr not monotone / wrong ends, bit 1: column outside [0, N),
// bit 2: a row not sorted by column
__global__ void validate_kernel(const int *row_ptr, const int *col, int M, int N,
                                int nnz, int *bad) {
  int flags = 0;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r <= M;
       r += gridDim.x * blockDim.x) {
    if (r == 0 && row_ptr[0] != 0) flags |= 1;
    if (r == M && row_ptr[M] != nnz) flags |= 1;
    if (r < M && row_ptr[r + 1] < row_ptr[r]) flags |= 1;
  }
  if (!flags) {
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < nnz;
         p += gridDim.x * blockDim.x) {
      const int c = col[p];
      if (c < 0 || c >= N) flags |= 2;
    }
  }
  if (flags) atomicOr(bad, flags);
}

__global__ void sorted_kernel(const int *row_ptr, const int *col, int M,
                              int *bad) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < M;
       r += gridDim.x * blockDim.x)
    for (int p = row_ptr[r] + 1; p < row_ptr[r + 1]; ++p)
      if (col[p] < col[p - 1]) {
        atomicOr(bad, 4);
        break;
      }
}

__global__ void head_kernel(const int *row_ptr, const int *col, int M, int nnz,
                            int segw, int *head) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < nnz;
       p += gridDim.x * blockDim.x) {
    const int r = row_of(row_ptr, M, p);
    head[p] = (p == row_ptr[r] || col[p] / segw != col[p - 1] / segw) ? 1 : 0;
  }
}

__global__ void pairs_kernel(const int *row_ptr, const int *col, int M, int nnz,
                             int segw, const int *head, const int *idx,
                             int *pr_row, int *pr_seg, int *pr_start) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < nnz;
       p += gridDim.x * blockDim.x) {
    if (!head[p]) continue;
    const int e = idx[p];
    pr_row[e] = row_of(row_ptr, M, p);
    pr_seg[e] = col[p] / segw;
    pr_start[e] = p;
  }
}

__global__ void count_kernel(const int *pr_start, int E, int nnz, int *pr_cnt,
                             int *maxc) {
  int local = 0;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E;
       e += gridDim.x * blockDim.x) {
    const int c = (e + 1 < E ? pr_start[e + 1] : nnz) - pr_start[e];
    pr_cnt[e] = c;
    local = max(local, c);
  }
  for (int o = 16; o; o >>= 1) local = max(local, __shfl_xor_sync(0xffffffffu, local, o));
  if ((threadIdx.x & 31) == 0) atomicMax(maxc, local);
}

__global__ void keys_kernel(const int *pr_seg, const int *pr_cnt, int E,
                            int cbits, int maxc, uint32_t *k_seg,
                            uint32_t *k_pack, int *iota, int *seg_count) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E;
       e += gridDim.x * blockDim.x) {
    const uint32_t s = (uint32_t)pr_seg[e];
    k_seg[e] = s;
    k_pack[e] = (s << cbits) | (uint32_t)(maxc - pr_cnt[e]);
    iota[e] = e;
    atomicAdd(seg_count + s, 1);
  }
}

__global__ void ngroups_kernel(const int *seg_count, int S, int bundle,
                               int *ng) {
  for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < S;
       s += gridDim.x * blockDim.x)
    ng[s] = (seg_count[s] + bundle - 1) / bundle;
}

// per group: its segment, depth and slot count
__global__ void group_meta_kernel(const int *seg_first, const int *seg_count,
                                  const int *g_first, const int *ng, int S,
                                  int bundle, int segw, const int *pack_order,
                                  const int *pr_cnt, int *g_seg, int *g_depth,
                                  int *g_seg_base, long long *g_slots) {
  // one warp per segment, lanes over its groups
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < S; s += warps) {
    const int n = ng[s], g0 = g_first[s], f = seg_first[s];
    for (int k = lane; k < n; k += 32) {
      const int depth = pr_cnt[pack_order[f + k * bundle]];
      g_seg[g0 + k] = s;
      g_depth[g0 + k] = depth;
      g_seg_base[g0 + k] = s * segw;
      g_slots[g0 + k] = (long long)depth * bundle;
    }
  }
}

// Rows with no entry in segment s, ascending: the first `need` of them go to
// lanes nz_s .. of the segment's last group.  One warp per segment walks the
// segment's rows (ascending) 32 at a time and takes the gaps.
__global__ void pad_rows_kernel(const int *seg_first, const int *seg_count,
                                const int *g_first, const int *ng, int S, int M,
                                int bundle, const int *by_seg, const int *pr_row,
                                int *group_rows) {
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  const unsigned lt = (1u << lane) - 1u;
  for (int s = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; s < S; s += warps) {
    const int nz = seg_count[s], n = ng[s];
    if (n == 0) continue;
    const long long last_end = (long long)n * bundle;
    const int need = (int)((last_end < M ? last_end : M) - nz);
    if (need <= 0) continue;
    int *out = group_rows + (long long)(g_first[s] + n - 1) * bundle +
               (nz - (n - 1) * bundle);
    const int f = seg_first[s];
    int found = 0, prev = -1;
    for (int i0 = 0; found < need; i0 += 32) {
      const int i = i0 + lane;
      // members past the end act as a sentinel row M
      const int r = i < nz ? pr_row[by_seg[f + i]] : M;
      int p = __shfl_up_sync(0xffffffffu, r, 1);
      if (lane == 0) p = prev;
      const int gap = (i <= nz) ? r - p - 1 : 0;
      int incl = gap;
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = incl - gap;
      for (int t = 0; t < gap && found + excl + t < need; ++t)
        out[found + excl + t] = p + 1 + t;
      found += __shfl_sync(0xffffffffu, incl, 31);
      prev = __shfl_sync(0xffffffffu, r, 31);
      if (__any_sync(0xffffffffu, i >= nz)) break;
    }
    (void)lt;
  }
}

__global__ void pack_kernel(const int *g_seg, const int *g_depth,
                            const int *group_ptr, const int *seg_first,
                            const int *seg_count, const int *g_first, int G,
                            int M, int bundle, int segw, const int *pack_order,
                            const int *pr_row, const int *pr_cnt,
                            const int *pr_start, const int *col,
                            const float *val, int *group_rows, int *lcol,
                            float *sval) {
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; g < G; g += warps) {
    const int s = g_seg[g];
    const int k = g - g_first[s];
    const int nz = seg_count[s], f = seg_first[s];
    const int depth = g_depth[g];
    const long long gp = group_ptr[g];
    const int sbase = s * segw;
    for (int l = lane; l < bundle; l += 32) {
      const long long pos = (long long)k * bundle + l;
      int cnt = 0, start = 0;
      if (pos < nz) {
        const int e = pack_order[f + pos];
        group_rows[(long long)g * bundle + l] = pr_row[e];
        cnt = pr_cnt[e];
        start = pr_start[e];
      } else if (pos >= M) {
        group_rows[(long long)g * bundle + l] = -1;
      }  // else: a count-0 row already placed by pad_rows_kernel
      for (int d = 0; d < depth; ++d) {
        const long long slot = gp + (long long)d * bundle + l;
        if (d < cnt) {
          lcol[slot] = col[start + d] - sbase;
          sval[slot] = val[start + d];
        } else {
          lcol[slot] = -1;
          sval[slot] = 0.f;
        }
      }
    }
  }
}

__global__ void narrow_kernel(const long long *in, int *out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (int)in[i];
}

int grid_for(int64_t n, int threads = 256) {
  int64_t b = ceil_div(n > 0 ? n : 1, threads);
  return (int)(b > 148 * 64 ? 148 * 64 : b);
}

int bits_for(uint32_t v) {
  int b = 0;
  while (b < 32 && (v >> b)) ++b;
  return b;
}

}  // namespace
}  // namespace vcsr

extern "C" vcsr_status vcsr_build_vcsr(const vcsr_csr *d, int segw, int bundle,
                                       vcsr_vcsr *out, vcsr_stream_t stream) {
  return vcsr::no_throw([&]() -> vcsr_status {
    using namespace vcsr;
    clear_error();
    if (!d || !out) return fail(VCSR_ERR_INVALID, "null argument");
    std::memset(out, 0, sizeof *out);
    if (bundle <= 0) return fail(VCSR_ERR_INVALID, "bundle must be >0");
    if (segw <= 0) return fail(VCSR_ERR_INVALID, "segw must be >0");
    if (d->M < 0 || d->N < 0 || d->nnz < 0) return fail(VCSR_ERR_INVALID, "negative size");
    cudaStream_t st = (cudaStream_t)stream;
    const int M = d->M, N = d->N, nnz = d->nnz;
    const int S = (int)ceil_div(N, segw);
    Scratch sc(st);
    out->M = M; out->N = N; out->segw = segw; out->bundle = bundle;
    out->num_segments = S;
    auto alloc_out = [&](int64_t G, int64_t P) -> vcsr_status {
      VCSR_CUDA(cudaMalloc(&out->group_ptr, sizeof(int) * (size_t)(G + 1)));
      VCSR_CUDA(cudaMalloc(&out->group_depth, sizeof(int) * (size_t)(G > 0 ? G : 1)));
      VCSR_CUDA(cudaMalloc(&out->group_seg_base, sizeof(int) * (size_t)(G > 0 ? G : 1)));
      VCSR_CUDA(cudaMalloc(&out->group_rows,
                           sizeof(int) * (size_t)(G * bundle > 0 ? G * bundle : 1)));
      VCSR_CUDA(cudaMalloc(&out->lcol, sizeof(int) * (size_t)(P > 0 ? P : 1)));
      VCSR_CUDA(cudaMalloc(&out->val, sizeof(float) * (size_t)(P > 0 ? P : 1)));
      VCSR_CUDA(cudaMalloc(&out->segment_group_start, sizeof(int) * ((size_t)S + 1)));
      return VCSR_OK;
    };
    if (nnz == 0 || M == 0) {
      vcsr_status s = alloc_out(0, 0);
      if (s == VCSR_OK) {
        cudaError_t e = cudaMemsetAsync(out->group_ptr, 0, sizeof(int), st);
        if (e == cudaSuccess)
          e = cudaMemsetAsync(out->segment_group_start, 0, sizeof(int) * ((size_t)S + 1), st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) s = fail(VCSR_ERR_CUDA, "%s", cudaGetErrorString(e));
      }
      if (s != VCSR_OK) vcsr_vcsr_free(out, VCSR_DEVICE);
      return s;
    }
    vcsr_status s;
    auto body = [&]() -> vcsr_status {
      int *bad;
      VCSR_TRY(sc.get(&bad, 1));
      VCSR_CUDA(cudaMemsetAsync(bad, 0, sizeof(int), st));
      validate_kernel<<<grid_for((int64_t)nnz + M + 1), 256, 0, st>>>(d->row_ptr, d->col,
                                                                     M, N, nnz, bad);
      VCSR_CUDA(cudaGetLastError());
      int hbad = 0;
      VCSR_CUDA(cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      if (hbad & 1) return fail(VCSR_ERR_INVALID, "row_ptr is not a valid CSR row pointer");
      if (hbad & 2) return fail(VCSR_ERR_RANGE, "a column index lies outside [0, N)");
      sorted_kernel<<<grid_for(M), 256, 0, st>>>(d->row_ptr, d->col, M, bad);
      VCSR_CUDA(cudaGetLastError());
      VCSR_CUDA(cudaMemcpyAsync(&hbad, bad, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      if (hbad & 4)
        return fail(VCSR_ERR_INVALID, "CSR rows must be sorted by column (coo_to_csr order)");
      int *head, *idx, *dE;
      VCSR_TRY(sc.get(&head, nnz));
      VCSR_TRY(sc.get(&idx, nnz));
      VCSR_TRY(sc.get(&dE, 2));
      head_kernel<<<grid_for(nnz), 256, 0, st>>>(d->row_ptr, d->col, M, nnz, segw, head);
      VCSR_CUDA(cudaGetLastError());
      VCSR_TRY(scan_exclusive<int>(head, idx, nnz, dE, sc));
      int E = 0;
      VCSR_CUDA(cudaMemcpyAsync(&E, dE, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      int *pr_row, *pr_seg, *pr_start, *pr_cnt, *maxc;
      VCSR_TRY(sc.get(&pr_row, E));
      VCSR_TRY(sc.get(&pr_seg, E));
      VCSR_TRY(sc.get(&pr_start, E));
      VCSR_TRY(sc.get(&pr_cnt, E));
      VCSR_TRY(sc.get(&maxc, 1));
      pairs_kernel<<<grid_for(nnz), 256, 0, st>>>(d->row_ptr, d->col, M, nnz, segw,
                                                  head, idx, pr_row, pr_seg, pr_start);
      VCSR_CUDA(cudaGetLastError());
      VCSR_CUDA(cudaMemsetAsync(maxc, 0, sizeof(int), st));
      count_kernel<<<grid_for(E), 256, 0, st>>>(pr_start, E, nnz, pr_cnt, maxc);
      VCSR_CUDA(cudaGetLastError());
      int hmaxc = 0;
      VCSR_CUDA(cudaMemcpyAsync(&hmaxc, maxc, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      const int sbits = bits_for((uint32_t)(S > 0 ? S - 1 : 0));
      const int cbits = bits_for((uint32_t)hmaxc);
      if (sbits + cbits > 32)
        return fail(VCSR_ERR_UNSUPPORTED, "segment/count keys exceed 32 bits");
      uint32_t *k_seg, *k_pack, *k_tmp;
      int *iota, *seg_count, *by_seg, *pack_order;
      VCSR_TRY(sc.get(&k_seg, E));
      VCSR_TRY(sc.get(&k_pack, E));
      VCSR_TRY(sc.get(&k_tmp, E));
      VCSR_TRY(sc.get(&iota, E));
      VCSR_TRY(sc.get(&seg_count, S));
      VCSR_TRY(sc.get(&by_seg, E));
      VCSR_TRY(sc.get(&pack_order, E));
      VCSR_CUDA(cudaMemsetAsync(seg_count, 0, sizeof(int) * (size_t)S, st));
      keys_kernel<<<grid_for(E), 256, 0, st>>>(pr_seg, pr_cnt, E, cbits, hmaxc, k_seg,
                                               k_pack, iota, seg_count);
      VCSR_CUDA(cudaGetLastError());
      VCSR_TRY(radix_sort_pairs(k_seg, iota, k_tmp, by_seg, E, sbits, sc));
      VCSR_TRY(radix_sort_pairs(k_pack, iota, k_tmp, pack_order, E, sbits + cbits, sc));
      int *seg_first, *ng, *g_first, *dG;
      VCSR_TRY(sc.get(&seg_first, S));
      VCSR_TRY(sc.get(&ng, S));
      VCSR_TRY(sc.get(&g_first, (int64_t)S + 1));
      VCSR_TRY(sc.get(&dG, 1));
      VCSR_TRY(scan_exclusive<int>(seg_count, seg_first, S, nullptr, sc));
      ngroups_kernel<<<grid_for(S), 256, 0, st>>>(seg_count, S, bundle, ng);
      VCSR_CUDA(cudaGetLastError());
      VCSR_TRY(scan_exclusive<int>(ng, g_first, S, dG, sc));
      int G = 0;
      VCSR_CUDA(cudaMemcpyAsync(&G, dG, sizeof(int), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      if ((int64_t)G * bundle > INT32_MAX)
        return fail(VCSR_ERR_UNSUPPORTED, "G*bundle exceeds 32-bit indexing");
      int *g_seg, *g_depth_tmp;
      long long *g_slots, *g_ptr64, *dP;
      VCSR_TRY(sc.get(&g_seg, G));
      VCSR_TRY(sc.get(&g_depth_tmp, G));
      VCSR_TRY(sc.get(&g_slots, G));
      VCSR_TRY(sc.get(&g_ptr64, (int64_t)G + 1));
      VCSR_TRY(sc.get(&dP, 1));
      // group metadata into the outputs once sizes are known: depth first
      int *g_seg_base_tmp;
      VCSR_TRY(sc.get(&g_seg_base_tmp, G));
      group_meta_kernel<<<grid_for((int64_t)S * 32), 256, 0, st>>>(
          seg_first, seg_count, g_first, ng, S, bundle, segw, pack_order, pr_cnt, g_seg,
          g_depth_tmp, g_seg_base_tmp, g_slots);
      VCSR_CUDA(cudaGetLastError());
      VCSR_TRY(scan_exclusive<long long>(g_slots, g_ptr64, G, dP, sc));
      long long P = 0;
      VCSR_CUDA(cudaMemcpyAsync(&P, dP, sizeof(long long), cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      if (P > INT32_MAX) return fail(VCSR_ERR_UNSUPPORTED, "VCSR exceeds 32-bit slot indexing");
      VCSR_TRY(alloc_out(G, P));
      out->num_groups = G;
      out->num_slots = P;
      if (G > 0) {
        narrow_kernel<<<grid_for(G), 256, 0, st>>>(g_ptr64, out->group_ptr, G);
        VCSR_CUDA(cudaGetLastError());
        VCSR_CUDA(cudaMemcpyAsync(out->group_depth, g_depth_tmp, sizeof(int) * (size_t)G,
                                  cudaMemcpyDeviceToDevice, st));
        VCSR_CUDA(cudaMemcpyAsync(out->group_seg_base, g_seg_base_tmp,
                                  sizeof(int) * (size_t)G, cudaMemcpyDeviceToDevice, st));
      }
      const int Pi = (int)P;
      VCSR_CUDA(cudaMemcpyAsync(out->group_ptr + G, &Pi, sizeof(int),
                                cudaMemcpyHostToDevice, st));
      VCSR_CUDA(cudaMemcpyAsync(out->segment_group_start, g_first,
                                sizeof(int) * (size_t)S, cudaMemcpyDeviceToDevice, st));
      VCSR_CUDA(cudaMemcpyAsync(out->segment_group_start + S, &G, sizeof(int),
                                cudaMemcpyHostToDevice, st));
      pad_rows_kernel<<<grid_for((int64_t)S * 32), 256, 0, st>>>(
          seg_first, seg_count, g_first, ng, S, M, bundle, by_seg, pr_row,
          out->group_rows);
      VCSR_CUDA(cudaGetLastError());
      pack_kernel<<<grid_for((int64_t)G * 32), 256, 0, st>>>(
          g_seg, out->group_depth, out->group_ptr, seg_first, seg_count, g_first, G, M,
          bundle, segw, pack_order, pr_row, pr_cnt, pr_start, d->col, d->val,
          out->group_rows, out->lcol, out->val);
      VCSR_CUDA(cudaGetLastError());
      VCSR_CUDA(cudaStreamSynchronize(st));  // host-side Pi/G copies end here
      return VCSR_OK;
    };
    s = body();
    if (s != VCSR_OK) {
      cudaStreamSynchronize(st);
      vcsr_vcsr_free(out, VCSR_DEVICE);
    }
    return s;
  });
}
