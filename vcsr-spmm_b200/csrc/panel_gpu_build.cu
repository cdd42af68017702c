// panel_gpu_build.cu — the plan's layout built on the GPU (see panel_gpu.h).
//
// Every pass is a grid-stride kernel over rows, entries, vectors or units,
// glued by the library's device scan and stable radix sort
// (device_prims.cu); the host only reads back a handful of totals (the
// validation flags, the union size, the number of units) to size the next
// allocation.  The rules are the host builder's (panel_build.cpp,
// panel_tc_build.cpp, plan.cu), restated for data-parallel execution:
//  * union of a vector = its rows' (column, occurrence) keys, ascending; an
//    entry is the union's representative of its key when no earlier row of
//    the vector holds the key, and the key's union position is the number of
//    representatives with smaller keys (per row a binary search and a
//    difference of the representative prefix sum);
//  * vector height: the largest R <= 8 whose sampled vectors are >= 60%
//    dense, over the same 4,096 sampled 16-row windows;
//  * dense TF32 panels: per 16-row block a 16-lane merge of the rows' block
//    columns, a panel where a block column holds >= min_nnz entries.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "common.h"
#include "device_prims.cuh"
#include "panel_gpu.h"
#include "seg_tc.h"

namespace vcsr {
namespace {

constexpr int kThreads = 256;
constexpr int kLongUnit = 128;      // units of >= this many union columns: a whole warp
constexpr int kMaxBatchVecs = 64;   // vectors per batch at most (staged vec_ptr window)

// Grid of a grid-stride loop over n items.
unsigned grid_for(int64_t n, int per = kThreads) {
  const int64_t g = (n + per - 1) / per;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 32));
}

#define GRID_STRIDE(i, n)                                                          \
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)(n); \
       i += (int64_t)gridDim.x * blockDim.x)

// First index in [lo, hi) with a[index] >= x (hi if none).
__device__ __forceinline__ int lower_idx(const int *__restrict__ a, int lo, int hi, int x) {
  while (lo < hi) {
    const int m = lo + ((hi - lo) >> 1);
    if (a[m] < x) lo = m + 1; else hi = m;
  }
  return lo;
}
// First index in [lo, hi) with a[index] > x (hi if none).
__device__ __forceinline__ int upper_idx(const int *__restrict__ a, int lo, int hi, int x) {
  while (lo < hi) {
    const int m = lo + ((hi - lo) >> 1);
    if (a[m] <= x) lo = m + 1; else hi = m;
  }
  return lo;
}

template <class T>
vcsr_status dmalloc(T **p, int64_t n) {
  VCSR_CUDA(cudaMalloc((void **)p, sizeof(T) * (size_t)(n > 0 ? n : 1)));
  return VCSR_OK;
}

// The plan's device bytes, counted as the upload path counts them (at least
// one element per array), so that a plan reports the same size however it
// was built or loaded.
void acct(vcsr_plan *p, size_t elem, int64_t n) {
  p->panel_bytes += (int64_t)(elem * (size_t)(n > 0 ? n : 1));
}

template <class T>
vcsr_status read1(T *host, const T *dev, cudaStream_t st) {
  VCSR_CUDA(cudaMemcpyAsync(host, dev, sizeof(T), cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  return VCSR_OK;
}

// ------------------------------------------------------------ validation
// flags: 1 row_ptr, 2 column range, 4 unsorted row; first[0..2] the first
// offending row, entry and entry.
__global__ void check_rowptr_kernel(const int *__restrict__ rp, int M, int nnz, int *flags,
                                    int *first) {
  GRID_STRIDE(r, (int64_t)M + 1) {
    const int x = rp[r];
    bool bad = x < 0 || x > nnz;
    if (r == 0) bad = bad || x != 0;
    else bad = bad || x < rp[r - 1];
    if (r == M) bad = bad || x != nnz;
    if (bad) {
      atomicOr(flags, 1);
      atomicMin(first, (int)r);
    }
  }
}

// row_of[p] = the row of entry p (a warp per row).
__global__ void row_of_kernel(const int *__restrict__ rp, int M, int *row_of) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = w0; r < M; r += nw)
    for (int p = rp[r] + lane; p < rp[r + 1]; p += 32) row_of[p] = (int)r;
}

__global__ void check_cols_kernel(const int *__restrict__ col, const int *__restrict__ row_of,
                                  int nnz, int N, int *flags, int *first) {
  GRID_STRIDE(p, nnz) {
    const int c = col[p];
    if (c < 0 || c >= N) {
      atomicOr(flags, 2);
      atomicMin(first + 1, (int)p);
    } else if (p > 0 && row_of[p - 1] == row_of[p] && col[p - 1] > c) {
      atomicOr(flags, 4);
      atomicMin(first + 2, (int)p);
    }
  }
}

__global__ void iota_kernel(int *a, int64_t n) {
  GRID_STRIDE(i, n) a[i] = (int)i;
}

template <class T>
__global__ void gather_kernel(const T *__restrict__ src, const int *__restrict__ idx, T *dst,
                              int64_t n) {
  GRID_STRIDE(i, n) dst[i] = src[idx[i]];
}

int bits_for(int64_t max_value) {
  int b = 1;
  while (b < 32 && ((int64_t)1 << b) <= max_value) ++b;
  return b;
}

}  // namespace

vcsr_status device_sorted_csr(const vcsr_csr &d, vcsr_csr *out, bool *owned, cudaStream_t st) {
  *owned = false;
  *out = d;
  const int M = d.M, nnz = d.nnz;
  Scratch sc(st);
  int *flags = nullptr;  // [0] flags, [1..3] first offenders
  VCSR_TRY(sc.get(&flags, 4));
  const int init[4] = {0, INT32_MAX, INT32_MAX, INT32_MAX};
  VCSR_CUDA(cudaMemcpyAsync(flags, init, sizeof init, cudaMemcpyHostToDevice, st));
  check_rowptr_kernel<<<grid_for((int64_t)M + 1), kThreads, 0, st>>>(d.row_ptr, M, nnz, flags,
                                                                      flags + 1);
  VCSR_CUDA(cudaGetLastError());
  int h[4];
  VCSR_CUDA(cudaMemcpyAsync(h, flags, sizeof h, cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  if (h[0] & 1) {
    if (h[1] == 0 || h[1] == M)
      return fail(VCSR_ERR_INVALID, "row_ptr must start at 0 and end at nnz");
    return fail(VCSR_ERR_INVALID, "row_ptr decreases at row %d", h[1] - 1);
  }
  if (nnz == 0) return VCSR_OK;
  int *row_of = nullptr;
  VCSR_TRY(sc.get(&row_of, nnz));
  row_of_kernel<<<grid_for((int64_t)M * 32), kThreads, 0, st>>>(d.row_ptr, M, row_of);
  VCSR_CUDA(cudaGetLastError());
  check_cols_kernel<<<grid_for(nnz), kThreads, 0, st>>>(d.col, row_of, nnz, d.N, flags,
                                                         flags + 1);
  VCSR_CUDA(cudaGetLastError());
  VCSR_CUDA(cudaMemcpyAsync(h, flags, sizeof h, cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  if (h[0] & 2) {
    int c = 0;
    VCSR_TRY(read1(&c, d.col + h[2], st));
    return fail(VCSR_ERR_RANGE, "column %d of entry %d outside [0, %d)", c, h[2], d.N);
  }
  if (!(h[0] & 4)) return VCSR_OK;
  // Unsorted rows: a stable sort by column, then a stable sort by row, keeps
  // equal (row, column) entries in their input order -- a stable per-row sort.
  int *idx = nullptr, *perm = nullptr, *rowk = nullptr, *perm2 = nullptr;
  uint32_t *keys = nullptr;
  VCSR_TRY(sc.get(&idx, nnz));
  VCSR_TRY(sc.get(&perm, nnz));
  VCSR_TRY(sc.get(&keys, nnz));
  VCSR_TRY(sc.get(&rowk, nnz));
  VCSR_TRY(sc.get(&perm2, nnz));
  iota_kernel<<<grid_for(nnz), kThreads, 0, st>>>(idx, nnz);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(radix_sort_pairs(reinterpret_cast<const uint32_t *>(d.col), idx, keys, perm, nnz,
                            bits_for(d.N - 1), sc));
  gather_kernel<int><<<grid_for(nnz), kThreads, 0, st>>>(row_of, perm, rowk, nnz);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(radix_sort_pairs(reinterpret_cast<const uint32_t *>(rowk), perm, keys, perm2, nnz,
                            bits_for(M - 1), sc));
  vcsr_csr s = d;
  s.row_ptr = nullptr; s.col = nullptr; s.val = nullptr;
  cudaError_t e = cudaMalloc(&s.row_ptr, sizeof(int) * ((size_t)M + 1));
  if (e == cudaSuccess) e = cudaMalloc(&s.col, sizeof(int) * (size_t)nnz);
  if (e == cudaSuccess) e = cudaMalloc(&s.val, sizeof(float) * (size_t)nnz);
  if (e != cudaSuccess) {
    vcsr_csr_free(&s, VCSR_DEVICE);
    return fail(VCSR_ERR_CUDA, "sorted CSR copy: %s", cudaGetErrorString(e));
  }
  *owned = true;
  *out = s;
  VCSR_CUDA(cudaMemcpyAsync(s.row_ptr, d.row_ptr, sizeof(int) * ((size_t)M + 1),
                            cudaMemcpyDeviceToDevice, st));
  gather_kernel<int><<<grid_for(nnz), kThreads, 0, st>>>(d.col, perm2, s.col, nnz);
  gather_kernel<float><<<grid_for(nnz), kThreads, 0, st>>>(d.val, perm2, s.val, nnz);
  VCSR_CUDA(cudaGetLastError());
  return VCSR_OK;
}

namespace {

// ------------------------------------------------- dense TF32 panels
// Row block i (rows 16i .. 16i+15): lane l < 16 walks row 16i + l; the warp
// takes the smallest block column any lane is at, the lanes count their
// entries in it, and the block column is a panel when the count reaches
// min_nnz.  Pass 0 counts the panels of each row block, pass 1 writes their
// block columns (ascending) from first[i] on.
__global__ void dense_blocks_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                                    int M, int min_nnz, int pass, int *ndense,
                                    const int *__restrict__ first, int *blk_col) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int nrb = (M + 15) / 16;
  for (int64_t i = w0; i < nrb; i += nw) {
    const int r = (int)(16 * i) + lane;
    const bool own = lane < 16 && r < M;
    int p = own ? rp[r] : 0;
    const int e = own ? rp[r + 1] : 0;
    int found = 0;
    const int base = pass ? first[i] : 0;
    for (;;) {
      const int bc = p < e ? (col[p] >> 4) : INT32_MAX;
      const int m = __reduce_min_sync(0xffffffffu, bc);
      if (m == INT32_MAX) break;
      int c = 0;
      while (p < e && (col[p] >> 4) == m) {
        ++p;
        ++c;
      }
      const int tot = (int)__reduce_add_sync(0xffffffffu, (unsigned)c);
      if (tot >= min_nnz) {
        if (pass == 1 && lane == 0) blk_col[base + found] = m;
        ++found;
      }
    }
    if (pass == 0 && lane == 0) ndense[i] = found;
  }
}

// Round to TF32 (10 explicit mantissa bits), nearest-even; Inf and NaN kept.
__device__ __forceinline__ float round_tf32_dev(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) != 0x7f800000u) {
    u += 0xFFFu + ((u >> 13) & 1u);
    u &= ~0x1FFFu;
  }
  return __uint_as_float(u);
}

// Per entry: its panel (if its block column is one of its row block's) or
// the residual.  A panel entry that starts its run of equal columns writes
// the run's sum (0 + v1 + v2 ..., CSR order) rounded to TF32 at its place in
// the block's core-matrix order.
__global__ void split_entries_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                                     const float *__restrict__ val,
                                     const int *__restrict__ row_of, int nnz,
                                     const int *__restrict__ ndense,
                                     const int *__restrict__ first,
                                     const int *__restrict__ blk_col, int *resid,
                                     float *blk_val) {
  GRID_STRIDE(p, nnz) {
    const int r = row_of[p], i = r >> 4;
    const int c = col[p], bc = c >> 4;
    const int b0 = first[i], b1 = b0 + ndense[i];
    const int b = lower_idx(blk_col, b0, b1, bc);
    const bool dense = b < b1 && blk_col[b] == bc;
    resid[p] = dense ? 0 : 1;
    if (dense && (p == rp[r] || col[p - 1] != c)) {
      float s = 0.f;
      for (int q = (int)p; q < rp[r + 1] && col[q] == c; ++q) s += val[q];
      const int n = r & 15, k = c & 15;
      blk_val[(size_t)b * 256 + ((k / 4) * 2 + n / 8) * 32 + (n % 8) * 4 + (k % 4)] =
          round_tf32_dev(s);
    }
  }
}

// Residual CSR: row r starts at RF[rp[r]], entry p goes to RF[p].
__global__ void residual_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                                const float *__restrict__ val, const int *__restrict__ resid,
                                const int *__restrict__ RF, int M, int nnz, int *r_rp,
                                int *r_col, float *r_val) {
  GRID_STRIDE(r, (int64_t)M + 1) r_rp[r] = RF[rp[r]];
  GRID_STRIDE(p, nnz) {
    if (resid[p]) {
      r_col[RF[p]] = col[p];
      r_val[RF[p]] = val[p];
    }
  }
}

// Row blocks holding panels: rb_row / rb_ptr, compacted in order.
__global__ void row_blocks_kernel(const int *__restrict__ ndense, const int *__restrict__ first,
                                  const int *__restrict__ RBI, int nrb, int n_blk,
                                  int *rb_row, int *rb_ptr) {
  GRID_STRIDE(i, nrb) {
    if (ndense[i] > 0) {
      rb_row[RBI[i]] = (int)(16 * i);
      rb_ptr[RBI[i]] = first[i];
    }
    if (i == nrb - 1) rb_ptr[RBI[i] + (ndense[i] > 0 ? 1 : 0)] = n_blk;
  }
}

__global__ void positive_flags_kernel(const int *__restrict__ a, int64_t n, int *flags) {
  GRID_STRIDE(i, n) flags[i] = a[i] > 0 ? 1 : 0;
}

// ------------------------------------------------- vector height
// The sampled windows: window of sample s = s * windows / samples (16 rows
// from row 16 * window); cnt[s] = its entries.
__global__ void sample_counts_kernel(const int *__restrict__ rp, int M, int64_t windows,
                                     int samples, int *cnt) {
  GRID_STRIDE(s, samples) {
    const int64_t w = s * windows / samples;
    const int r0 = (int)(w * 16), r1 = min(M, r0 + 16);
    cnt[s] = rp[r1] - rp[r0];
  }
}

// acc[0] = entries of the sampled windows, acc[1 + j] = the sum of the union
// sizes of their vectors at R = 2, 4, 8, 16 (vectors aligned to the window,
// which starts at a multiple of 16 rows).  An entry counts towards its
// vector's union when no earlier row of the vector holds its (column,
// occurrence) key.  One thread per sampled entry (off = exclusive prefix of
// the windows' entries), so a window of long rows spreads over many blocks.
__global__ void sample_unions_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                                     int M, int64_t windows, int samples,
                                     const int *__restrict__ off, int total,
                                     unsigned long long *acc) {
  __shared__ unsigned long long part[5][kThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  unsigned long long loc[5] = {0, 0, 0, 0, 0};  // entries, R = 2, 4, 8, 16
  GRID_STRIDE(i, total) {
    int lo = 0, hi = samples;  // the sample holding entry i: last s with off[s] <= i
    while (hi - lo > 1) {
      const int m = (lo + hi) >> 1;
      if (off[m] <= i) lo = m; else hi = m;
    }
    const int64_t w = (int64_t)lo * windows / samples;
    const int r0 = (int)(w * 16);
    const int p = rp[r0] + (int)(i - off[lo]);
    int r = r0;
    while (rp[r + 1] <= p) ++r;
    const int c = col[p];
    const int occ = p - lower_idx(col, rp[r], p, c);
    unsigned present = 0;
    for (int rr = r0; rr < r; ++rr) {
      const int b = rp[rr], e = rp[rr + 1];
      const int l0 = lower_idx(col, b, e, c);
      const int h0 = upper_idx(col, l0, e, c);
      if (h0 - l0 > occ) present |= 1u << (rr - r0);
    }
    loc[0] += 1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int R = 2 << j;
      const int vs = ((r - r0) / R) * R;
      const unsigned mask = ((1u << (r - r0)) - 1u) & ~((1u << vs) - 1u);
      if (!(present & mask)) loc[1 + j] += 1;
    }
  }
#pragma unroll
  for (int j = 0; j < 5; ++j) {
    unsigned long long x = loc[j];
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) part[j][warp] = x;
  }
  __syncthreads();
  if (threadIdx.x < 5) {
    unsigned long long t = 0;
    for (int q = 0; q < kThreads / 32; ++q) t += part[threadIdx.x][q];
    if (t) atomicAdd(acc + threadIdx.x, t);
  }
}

// ------------------------------------------------- vector panels, R > 1
// Key of entry p = (its column c, its occurrence: how many earlier entries
// of its row have column c).  flag[p] = 1 when no earlier row of p's vector
// holds the key: p represents the key in the vector's union.
__global__ void first_flag_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                                  const int *__restrict__ row_of, int nnz, int R, int *flag) {
  GRID_STRIDE(p, nnz) {
    const int r = row_of[p], vs = (r / R) * R, c = col[p];
    const int occ = (int)p - lower_idx(col, rp[r], (int)p, c);
    bool first = true;
    for (int rr = vs; rr < r && first; ++rr) {
      const int e = rp[rr + 1];
      const int lo = lower_idx(col, rp[rr], e, c);
      if (upper_idx(col, lo, e, c) - lo > occ) first = false;
    }
    flag[p] = first ? 1 : 0;
  }
}

// vec_ptr[v] = representatives before vector v's first entry (F is the
// exclusive prefix sum of the flags, F[nnz] their total).
__global__ void vec_ptr_kernel(const int *__restrict__ rp, const int *__restrict__ F, int M,
                               int R, int V, int *vec_ptr) {
  GRID_STRIDE(v, (int64_t)V + 1) vec_ptr[v] = F[rp[min((int64_t)M, v * R)]];
}

// Entry p lands at union position u = vec_ptr[v] + (representatives of the
// vector with a smaller key): per row of the vector, the entries with a
// smaller key are a prefix of the row (a binary search), and the
// representatives among them a difference of F.
__global__ void place_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                             const float *__restrict__ val, const int *__restrict__ row_of,
                             const int *__restrict__ F, int M, int nnz, int R, int *ucol,
                             float *uval, unsigned *umask) {
  GRID_STRIDE(p, nnz) {
    const int r = row_of[p], vs = (r / R) * R, ve = min(M, vs + R), c = col[p];
    const int occ = (int)p - lower_idx(col, rp[r], (int)p, c);
    int rank = 0;
    for (int rr = vs; rr < ve; ++rr) {
      const int b = rp[rr], e = rp[rr + 1];
      int q;
      if (rr == r) {
        q = (int)p;
      } else {
        const int lo = lower_idx(col, b, e, c);
        q = lo + min(occ, upper_idx(col, lo, e, c) - lo);
      }
      rank += F[q] - F[b];
    }
    const int u = F[rp[vs]] + rank;
    uval[(size_t)u * R + (r - vs)] = val[p];
    atomicOr(umask + u, 1u << (r - vs));
    if (F[p + 1] != F[p]) ucol[u] = c;
  }
}

// ------------------------------------------------- units
// A vector of n union columns is one unit when n <= chunk, else
// ceil(n / chunk) parts of ceil(n / parts) columns (a split vector).
__global__ void vec_parts_kernel(const int *__restrict__ vec_ptr, int V, int chunk,
                                 int *nparts, int *split, int *split_parts) {
  GRID_STRIDE(v, V) {
    const int n = vec_ptr[v + 1] - vec_ptr[v];
    const int np = n > chunk ? (n + chunk - 1) / chunk : 1;
    nparts[v] = np;
    split[v] = np > 1 ? 1 : 0;
    split_parts[v] = np > 1 ? np : 0;
  }
}

__global__ void fill_units_kernel(const int *__restrict__ vec_ptr, int V,
                                  const int *__restrict__ nparts, const int *__restrict__ uoff,
                                  const int *__restrict__ svi, const int *__restrict__ poff,
                                  int4 *units, int2 *parts, int2 *svecs) {
  GRID_STRIDE(v, V) {
    const int b = vec_ptr[v], e = vec_ptr[v + 1], np = nparts[v], u0 = uoff[v];
    if (np == 1) {
      units[u0] = make_int4((int)v, b, e, -1);
      continue;
    }
    const int sv = svi[v], first = poff[v], per = (e - b + np - 1) / np;
    svecs[sv] = make_int2(first, np);
    for (int q = 0; q < np; ++q) {
      const int pb = b + q * per, pe = min(e, pb + per);
      units[u0 + q] = make_int4((int)v, pb, pe, first + q);
      parts[first + q] = make_int2(sv, q);
    }
  }
}

// Split parts and units of >= kLongUnit columns are walked by a whole warp
// ("long"); the others are short.
__global__ void classify_units_kernel(const int4 *__restrict__ units, int n_units, int *is_long,
                                      int *is_short, int *short_len) {
  GRID_STRIDE(u, n_units) {
    const int4 U = units[u];
    const int len = U.z - U.y;
    const bool lg = U.w >= 0 || len >= kLongUnit;
    is_long[u] = lg ? 1 : 0;
    is_short[u] = lg ? 0 : 1;
    short_len[u] = lg ? 0 : len;
  }
}

// Batches of consecutive short units (one vector each), walked by one
// sub-warp: a batch starts at a short unit that follows a long unit (or is
// the first), at every 64th short unit, and where the short units' running
// column count crosses a multiple of batch_cols; with R > 2 every short
// unit is a batch of its own.  Long units are listed in order.
__global__ void batch_start_kernel(int n_units, int R, int batch_cols,
                                   const int *__restrict__ is_long, const int *__restrict__ lidx,
                                   const int *__restrict__ kidx, const int *__restrict__ C,
                                   int *long_idx, int *bstart) {
  GRID_STRIDE(u, n_units) {
    if (is_long[u]) {
      long_idx[lidx[u]] = (int)u;
      bstart[u] = 0;
      continue;
    }
    const int k = kidx[u];
    const bool st = R > 2 || u == 0 || is_long[u - 1] || (k % kMaxBatchVecs) == 0 ||
                    C[u] / batch_cols != C[u - 1] / batch_cols;
    bstart[u] = st ? 1 : 0;
  }
}

// batch = {first vector, one past the last, first union column, end column}
__global__ void fill_batches_kernel(const int4 *__restrict__ units, int n_units,
                                    const int *__restrict__ is_long,
                                    const int *__restrict__ bstart,
                                    const int *__restrict__ bidx, int *batches) {
  GRID_STRIDE(u, n_units) {
    if (is_long[u]) continue;
    const int4 U = units[u];
    const int id = bstart[u] ? bidx[u] : bidx[u] - 1;
    if (bstart[u]) {
      batches[4 * id + 0] = U.x;
      batches[4 * id + 2] = U.y;
    }
    if (u + 1 == n_units || is_long[u + 1] || bstart[u + 1]) {
      batches[4 * id + 1] = U.x + 1;
      batches[4 * id + 3] = U.z;
    }
  }
}

// ------------------------------------------------- row panels
__global__ void row_cut_kernel(const int *__restrict__ rp, int M, const long long *targets,
                               int n, int *rows) {
  GRID_STRIDE(j, n) {
    int lo = 0, hi = M + 1;  // first row index with rp >= target
    while (lo < hi) {
      const int m = lo + ((hi - lo) >> 1);
      if ((long long)rp[m] < targets[j]) lo = m + 1; else hi = m;
    }
    rows[j] = lo;
  }
}

// col_max[j] = the highest column any row of panel j reads (rows sorted:
// each row's last entry), -1 for none.
__global__ void panel_colmax_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                                    int M, const int *__restrict__ bounds, int n, int *col_max) {
  // whole warps run the loop (rows past M count as empty), so that a warp
  // whose rows share a panel reduces before its one atomic
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t Mw = ((int64_t)M + 31) & ~(int64_t)31;
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < Mw; r += stride) {
    int v = -1, j = 0;
    if (r < M) {
      const int e = rp[r + 1];
      if (e > rp[r]) v = col[e - 1];
      while (j + 1 < n && r >= bounds[j + 1]) ++j;
    }
    const int j0 = __shfl_sync(0xffffffffu, j, 0);
    if (__all_sync(0xffffffffu, j == j0)) {
      const int m = __reduce_max_sync(0xffffffffu, v);
      if ((threadIdx.x & 31) == 0 && m >= 0) atomicMax(col_max + j0, m);
    } else if (v >= 0) {
      atomicMax(col_max + j, v);
    }
  }
}

__global__ void unit_vec_kernel(const int4 *__restrict__ units, const int *__restrict__ idx,
                                int n, int *out) {
  GRID_STRIDE(i, n) out[i] = units[idx[i]].x;
}

__global__ void batch_v0_kernel(const int *__restrict__ batches, int n, int *out) {
  GRID_STRIDE(i, n) out[i] = batches[4 * i];
}

// ------------------------------------------------- tensor-core segments
// The 16-row union of vector v (R = 16 panels: ucol ascending, a duplicate
// entry repeating its column) cut into runs of consecutive columns.  Pass 0
// counts the runs shorter than 8 columns (*short_runs).  Pass 1 counts, per
// vector, the runs of at least min_run columns, their pieces (at most
// kSegPieceRows rows, a multiple of 8) and the pieces' rows.  Pass 2 writes
// the runs {c0, length}, the pieces {c0, L, koff} and the dense tiles (values
// of a column added in union order, which is CSR order for duplicates).
__global__ void seg_runs_kernel(const int *__restrict__ vec_ptr, const int *__restrict__ ucol,
                                const float *__restrict__ uval,
                                const unsigned *__restrict__ umask, int V, int min_run,
                                int pass, int *short_runs, int *nruns, int *npieces, int *nrows,
                                const int *__restrict__ run_off,
                                const int *__restrict__ piece_off,
                                const int *__restrict__ row_off, int2 *runs, int4 *pieces,
                                float *a) {
  GRID_STRIDE(v, V) {
    const int b = vec_ptr[v], e = vec_ptr[v + 1];
    int nr = 0, np = 0, nk = 0, ns = 0;
    int j = b;
    while (j < e) {
      // the run starting at union entry j: columns c0 .. c1-1, entries j .. j1-1
      const int c0 = ucol[j];
      int c1 = c0 + 1, j1 = j + 1;
      while (j1 < e && (ucol[j1] == c1 - 1 || ucol[j1] == c1)) {
        if (ucol[j1] == c1) ++c1;
        ++j1;
      }
      const int len = c1 - c0;
      if (len < 8) ++ns;
      if (len >= min_run) {
        const int pieces_here = (len + kSegPieceRows - 1) / kSegPieceRows;
        if (pass == 2) {
          const int kbase = row_off[v] + nk;
          runs[run_off[v] + nr] = make_int2(c0, len);
          for (int q = 0; q < pieces_here; ++q) {
            const int rest = len - q * kSegPieceRows;
            const int L = min(kSegPieceRows, (rest + 7) & ~7);
            pieces[piece_off[v] + np + q] = make_int4(c0 + q * kSegPieceRows, L,
                                                      kbase + q * kSegPieceRows, 0);
          }
          for (int jj = j; jj < j1; ++jj) {
            const int k = ucol[jj] - c0, q = k / kSegPieceRows, kk = k % kSegPieceRows;
            float *tile = a + (size_t)(kbase + q * kSegPieceRows) * 16;
            const unsigned m = umask[jj];
            for (int n = 0; n < 16; ++n)
              if ((m >> n) & 1u)
                tile[(kk / 4) * 64 + (n / 8) * 32 + (n % 8) * 4 + (kk % 4)] +=
                    uval[(size_t)jj * 16 + n];
          }
        }
        for (int q = 0; q < pieces_here; ++q) {
          const int rest = len - q * kSegPieceRows;
          nk += min(kSegPieceRows, (rest + 7) & ~7);
        }
        np += pieces_here;
        ++nr;
      }
      j = j1;
    }
    if (pass == 0 && ns) atomicAdd(short_runs, ns);
    if (pass == 1) {
      nruns[v] = nr;
      npieces[v] = np;
      nrows[v] = nk;
    }
  }
}

// Entries outside every tensor-core run of their row block: the residual.
__global__ void seg_residual_flags_kernel(const int *__restrict__ col,
                                          const int *__restrict__ row_of, int nnz,
                                          const int *__restrict__ run_off,
                                          const int2 *__restrict__ runs, int *resid) {
  GRID_STRIDE(p, nnz) {
    const int v = row_of[p] >> 4, c = col[p];
    int lo = run_off[v], hi = run_off[v + 1];
    while (lo < hi) {  // first run starting after c
      const int m = lo + ((hi - lo) >> 1);
      if (runs[m].x <= c) lo = m + 1; else hi = m;
    }
    const bool in = lo > run_off[v] && c < runs[lo - 1].x + runs[lo - 1].y;
    resid[p] = in ? 0 : 1;
  }
}

// Row blocks holding pieces, compacted in order.
__global__ void seg_row_blocks_kernel(const int *__restrict__ npieces,
                                      const int *__restrict__ piece_off,
                                      const int *__restrict__ rbi, int V, int n_pieces,
                                      int *rb_row, int *pp) {
  GRID_STRIDE(v, V) {
    if (npieces[v] > 0) {
      rb_row[rbi[v]] = (int)(16 * v);
      pp[rbi[v]] = piece_off[v];
    }
    if (v == V - 1) pp[rbi[v] + (npieces[v] > 0 ? 1 : 0)] = n_pieces;
  }
}

// The largest R <= 8 whose sampled vectors are at least 60% dense (the host
// builder's choose_vec_rows, panel_build.cpp, on the same samples).
vcsr_status choose_vec_rows_device(const vcsr_csr &w, int sms, Scratch &sc, int *R_out) {
  const int64_t windows = ((int64_t)w.M + 15) / 16;
  const int samples = (int)std::min<int64_t>(windows, 4096);
  *R_out = 1;
  if (samples == 0) return VCSR_OK;
  unsigned long long *acc = nullptr;
  int *cnt = nullptr, *off = nullptr;
  VCSR_TRY(sc.get(&acc, 5));
  VCSR_TRY(sc.get(&cnt, samples));
  VCSR_TRY(sc.get(&off, (int64_t)samples + 1));
  VCSR_CUDA(cudaMemsetAsync(acc, 0, 5 * sizeof(unsigned long long), sc.st));
  sample_counts_kernel<<<grid_for(samples), kThreads, 0, sc.st>>>(w.row_ptr, w.M, windows,
                                                                   samples, cnt);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(scan_exclusive<int>(cnt, off, samples, off + samples, sc));
  int total = 0;
  VCSR_TRY(read1(&total, off + samples, sc.st));
  sample_unions_kernel<<<grid_for(total), kThreads, 0, sc.st>>>(
      w.row_ptr, w.col, w.M, windows, samples, off, total, acc);
  VCSR_CUDA(cudaGetLastError());
  unsigned long long h[5];
  VCSR_CUDA(cudaMemcpyAsync(h, acc, sizeof h, cudaMemcpyDeviceToHost, sc.st));
  VCSR_CUDA(cudaStreamSynchronize(sc.st));
  const double nnz_s = (double)h[0];
  const int cands[3] = {2, 4, 8};
  for (int j = 0; j < 3; ++j) {
    const double un = (double)h[1 + j];
    const double dens = un > 0 ? nnz_s / (un * cands[j]) : 0.0;
    if (dens >= 0.6) *R_out = cands[j];
  }
  return VCSR_OK;
}

}  // namespace

__global__ void long_first_col_kernel(const int4 *__restrict__ units,
                                      const int *__restrict__ lidx,
                                      const int *__restrict__ ucol, int n, uint32_t *keys,
                                      int *vals) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int u = lidx[i];
    keys[i] = (uint32_t)ucol[units[u].y];
    vals[i] = u;
  }
}

vcsr_status order_long_by_column(vcsr_plan *p, cudaStream_t st) {
  const int n = p->n_long;
  if (n <= 1 || p->d_long_col) return VCSR_OK;
  Scratch sc(st);
  uint32_t *kin = nullptr, *kout = nullptr;
  int *vin = nullptr;
  VCSR_TRY(sc.get(&kin, n));
  VCSR_TRY(sc.get(&kout, n));
  VCSR_TRY(sc.get(&vin, n));
  VCSR_TRY(dmalloc(&p->d_long_col, n));
  long_first_col_kernel<<<grid_for(n), kThreads, 0, st>>>(p->d_units, p->d_long, p->d_ucol, n,
                                                          kin, vin);
  VCSR_CUDA(cudaGetLastError());
  int bits = 1;
  while (bits < 32 && (1LL << bits) < (long long)p->N) ++bits;
  VCSR_TRY(radix_sort_pairs(kin, vin, kout, p->d_long_col, n, bits, sc));
  acct(p, 4, n);
  VCSR_CUDA(cudaStreamSynchronize(st));  // the scratch dies here
  return VCSR_OK;
}

vcsr_status build_plan_layout_device(vcsr_plan *p, const vcsr_csr &d, int sms,
                                     cudaStream_t st) {
  const vcsr_plan_params &params = p->params;
  const int M = d.M;
  Scratch sc(st);
  vcsr_csr work = d;
  int *tot = nullptr;  // totals of the scans, read back together
  VCSR_TRY(sc.get(&tot, 8));

  // ---- dense 16x16 panels for the tensor cores; the rest is the residual
  if ((params.flags & VCSR_PLAN_TF32_PANELS) && M > 0) {
    if (params.panel_min_nnz < 0 || params.panel_min_nnz > 256)
      return fail(VCSR_ERR_INVALID, "panel_min_nnz must be in [0, 256]");
    const int min_nnz = params.panel_min_nnz > 0 ? params.panel_min_nnz : 128;
    const int nrb = (M + 15) / 16, nnz = d.nnz;
    int *ndense = nullptr, *first = nullptr, *row_of = nullptr, *resid = nullptr, *RF = nullptr;
    int *rbf = nullptr, *RBI = nullptr;
    VCSR_TRY(sc.get(&ndense, nrb));
    VCSR_TRY(sc.get(&first, nrb + 1));
    dense_blocks_kernel<<<grid_for((int64_t)nrb * 32), kThreads, 0, st>>>(
        d.row_ptr, d.col, M, min_nnz, 0, ndense, nullptr, nullptr);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(ndense, first, nrb, first + nrb, sc));
    int n_blk = 0;
    VCSR_TRY(read1(&n_blk, first + nrb, st));
    if (n_blk > 0) {
      VCSR_TRY(dmalloc(&p->d_blk_col, n_blk));
      VCSR_TRY(dmalloc(&p->d_blk_val, (int64_t)n_blk * 256));
      VCSR_CUDA(cudaMemsetAsync(p->d_blk_val, 0, sizeof(float) * 256 * (size_t)n_blk, st));
      dense_blocks_kernel<<<grid_for((int64_t)nrb * 32), kThreads, 0, st>>>(
          d.row_ptr, d.col, M, min_nnz, 1, ndense, first, p->d_blk_col);
      VCSR_CUDA(cudaGetLastError());
    }
    VCSR_TRY(sc.get(&row_of, nnz));
    VCSR_TRY(sc.get(&resid, nnz));
    VCSR_TRY(sc.get(&RF, (int64_t)nnz + 1));
    row_of_kernel<<<grid_for((int64_t)M * 32), kThreads, 0, st>>>(d.row_ptr, M, row_of);
    split_entries_kernel<<<grid_for(nnz), kThreads, 0, st>>>(
        d.row_ptr, d.col, d.val, row_of, nnz, ndense, first, p->d_blk_col, resid, p->d_blk_val);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(resid, RF, nnz, RF + nnz, sc));
    int n_res = 0;
    VCSR_TRY(read1(&n_res, RF + nnz, st));
    int *r_rp = nullptr, *r_col = nullptr;
    float *r_val = nullptr;
    VCSR_TRY(sc.get(&r_rp, (int64_t)M + 1));
    VCSR_TRY(sc.get(&r_col, n_res));
    VCSR_TRY(sc.get(&r_val, n_res));
    residual_kernel<<<grid_for(std::max<int64_t>(nnz, (int64_t)M + 1)), kThreads, 0, st>>>(
        d.row_ptr, d.col, d.val, resid, RF, M, nnz, r_rp, r_col, r_val);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(sc.get(&rbf, nrb));
    VCSR_TRY(sc.get(&RBI, nrb + 1));
    positive_flags_kernel<<<grid_for(nrb), kThreads, 0, st>>>(ndense, nrb, rbf);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(rbf, RBI, nrb, RBI + nrb, sc));
    int n_rb = 0;
    VCSR_TRY(read1(&n_rb, RBI + nrb, st));
    if (n_rb > 0) {
      VCSR_TRY(dmalloc(&p->d_rb_row, n_rb));
      VCSR_TRY(dmalloc(&p->d_rb_ptr, (int64_t)n_rb + 1));
      VCSR_TRY(dmalloc(&p->d_err, 1));
      VCSR_CUDA(cudaMemsetAsync(p->d_err, 0, sizeof(int), st));
      row_blocks_kernel<<<grid_for(nrb), kThreads, 0, st>>>(ndense, first, RBI, nrb, n_blk,
                                                             p->d_rb_row, p->d_rb_ptr);
      VCSR_CUDA(cudaGetLastError());
      acct(p, 4, n_rb);
      acct(p, 4, (int64_t)n_rb + 1);
      acct(p, 4, n_blk);
      acct(p, 4, (int64_t)n_blk * 256);
      acct(p, 4, 1);
    } else {
      cudaFree(p->d_blk_col);
      cudaFree(p->d_blk_val);
      p->d_blk_col = nullptr;
      p->d_blk_val = nullptr;
      n_blk = 0;
    }
    p->n_panel_rb = n_rb;
    p->n_panel_blocks = n_blk;
    p->panel_nnz = (int64_t)nnz - n_res;
    work.nnz = n_res;
    work.row_ptr = r_rp;
    work.col = r_col;
    work.val = r_val;
  }

  // ---- tensor-core segments: runs of consecutive columns of each 16-row
  // block (spmm_seg_tc.cu); entries of shorter runs form the residual
  if ((params.flags & VCSR_PLAN_TC_SEGMENTS) && M > 0) {
    if (params.flags & VCSR_PLAN_TF32_PANELS)
      return fail(VCSR_ERR_INVALID, "VCSR_PLAN_TC_SEGMENTS and VCSR_PLAN_TF32_PANELS exclude "
                                    "each other");
    if (params.seg_min_run < 0) return fail(VCSR_ERR_INVALID, "seg_min_run must be >= 0");
    const int nnz = d.nnz, V16 = (int)ceil_div(M, 16);
    int *row_of = nullptr, *flag = nullptr, *F = nullptr, *vp16 = nullptr, *uc16 = nullptr;
    float *uv16 = nullptr;
    unsigned *um16 = nullptr;
    int *st_tot = nullptr;
    VCSR_TRY(sc.get(&st_tot, 8));
    VCSR_CUDA(cudaMemsetAsync(st_tot, 0, 8 * sizeof(int), st));
    VCSR_TRY(sc.get(&row_of, nnz));
    VCSR_TRY(sc.get(&flag, nnz));
    VCSR_TRY(sc.get(&F, (int64_t)nnz + 1));
    VCSR_TRY(sc.get(&vp16, (int64_t)V16 + 1));
    row_of_kernel<<<grid_for((int64_t)M * 32), kThreads, 0, st>>>(d.row_ptr, M, row_of);
    first_flag_kernel<<<grid_for(nnz), kThreads, 0, st>>>(d.row_ptr, d.col, row_of, nnz, 16,
                                                           flag);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(flag, F, nnz, F + nnz, sc));
    int U16 = 0;
    VCSR_TRY(read1(&U16, F + nnz, st));
    VCSR_TRY(sc.get(&uc16, U16));
    VCSR_TRY(sc.get(&uv16, (int64_t)U16 * 16));
    VCSR_TRY(sc.get(&um16, U16));
    if (U16 > 0) {
      VCSR_CUDA(cudaMemsetAsync(uv16, 0, sizeof(float) * 16 * (size_t)U16, st));
      VCSR_CUDA(cudaMemsetAsync(um16, 0, sizeof(unsigned) * (size_t)U16, st));
    }
    vec_ptr_kernel<<<grid_for((int64_t)V16 + 1), kThreads, 0, st>>>(d.row_ptr, F, M, 16, V16,
                                                                     vp16);
    place_kernel<<<grid_for(nnz), kThreads, 0, st>>>(d.row_ptr, d.col, d.val, row_of, F, M, nnz,
                                                      16, uc16, uv16, um16);
    VCSR_CUDA(cudaGetLastError());
    // Runs shorter than 8 columns: padded to 8 rows on the tensor cores while
    // their padded rows stay below M (a residual pass costs C's write and a
    // read-modify-write of C), else left to the FP32 kernel.
    int min_run = params.seg_min_run;
    if (min_run == 0) {
      seg_runs_kernel<<<grid_for(V16), kThreads, 0, st>>>(
          vp16, uc16, uv16, um16, V16, 1, 0, st_tot, nullptr, nullptr, nullptr, nullptr, nullptr,
          nullptr, nullptr, nullptr, nullptr);
      VCSR_CUDA(cudaGetLastError());
      int short_runs = 0;
      VCSR_TRY(read1(&short_runs, st_tot, st));
      min_run = (int64_t)short_runs * 8 <= M ? 1 : 8;
    }
    int *nruns = nullptr, *npieces = nullptr, *nrows = nullptr, *run_off = nullptr,
        *piece_off = nullptr, *row_off = nullptr, *pflag = nullptr, *rbi = nullptr;
    VCSR_TRY(sc.get(&nruns, V16));
    VCSR_TRY(sc.get(&npieces, V16));
    VCSR_TRY(sc.get(&nrows, V16));
    VCSR_TRY(sc.get(&run_off, (int64_t)V16 + 1));
    VCSR_TRY(sc.get(&piece_off, (int64_t)V16 + 1));
    VCSR_TRY(sc.get(&row_off, (int64_t)V16 + 1));
    seg_runs_kernel<<<grid_for(V16), kThreads, 0, st>>>(
        vp16, uc16, uv16, um16, V16, min_run, 1, nullptr, nruns, npieces, nrows, nullptr,
        nullptr, nullptr, nullptr, nullptr, nullptr);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(nruns, run_off, V16, run_off + V16, sc));
    VCSR_TRY(scan_exclusive<int>(npieces, piece_off, V16, piece_off + V16, sc));
    VCSR_TRY(scan_exclusive<int>(nrows, row_off, V16, row_off + V16, sc));
    int h3[3];
    VCSR_TRY(read1(&h3[0], run_off + V16, st));
    VCSR_TRY(read1(&h3[1], piece_off + V16, st));
    VCSR_TRY(read1(&h3[2], row_off + V16, st));
    const int n_runs = h3[0], n_pieces = h3[1], seg_rows = h3[2];
    int2 *runs = nullptr;
    VCSR_TRY(sc.get(&runs, n_runs));
    VCSR_TRY(dmalloc(&p->d_seg_pieces, n_pieces));
    VCSR_TRY(dmalloc(&p->d_seg_a, (int64_t)seg_rows * 16));
    if (seg_rows > 0)
      VCSR_CUDA(cudaMemsetAsync(p->d_seg_a, 0, sizeof(float) * 16 * (size_t)seg_rows, st));
    seg_runs_kernel<<<grid_for(V16), kThreads, 0, st>>>(
        vp16, uc16, uv16, um16, V16, min_run, 2, nullptr, nullptr, nullptr, nullptr, run_off,
        piece_off, row_off, runs, p->d_seg_pieces, p->d_seg_a);
    VCSR_CUDA(cudaGetLastError());
    sc.release(uc16);
    sc.release(uv16);
    sc.release(um16);
    // row blocks with pieces
    VCSR_TRY(sc.get(&pflag, V16));
    VCSR_TRY(sc.get(&rbi, (int64_t)V16 + 1));
    positive_flags_kernel<<<grid_for(V16), kThreads, 0, st>>>(npieces, V16, pflag);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(pflag, rbi, V16, rbi + V16, sc));
    int n_seg_rb = 0;
    VCSR_TRY(read1(&n_seg_rb, rbi + V16, st));
    VCSR_TRY(dmalloc(&p->d_seg_rb_row, n_seg_rb));
    VCSR_TRY(dmalloc(&p->d_seg_pp, (int64_t)n_seg_rb + 1));
    seg_row_blocks_kernel<<<grid_for(V16), kThreads, 0, st>>>(npieces, piece_off, rbi, V16,
                                                               n_pieces, p->d_seg_rb_row,
                                                               p->d_seg_pp);
    VCSR_CUDA(cudaGetLastError());
    // the residual: entries outside every run of their row block
    int *resid = flag;  // reused
    seg_residual_flags_kernel<<<grid_for(nnz), kThreads, 0, st>>>(d.col, row_of, nnz, run_off,
                                                                   runs, resid);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(resid, F, nnz, F + nnz, sc));
    int n_res = 0;
    VCSR_TRY(read1(&n_res, F + nnz, st));
    int *r_rp = nullptr, *r_col = nullptr;
    float *r_val = nullptr;
    VCSR_TRY(sc.get(&r_rp, (int64_t)M + 1));
    VCSR_TRY(sc.get(&r_col, n_res));
    VCSR_TRY(sc.get(&r_val, n_res));
    residual_kernel<<<grid_for(std::max<int64_t>(nnz, (int64_t)M + 1)), kThreads, 0, st>>>(
        d.row_ptr, d.col, d.val, resid, F, M, nnz, r_rp, r_col, r_val);
    VCSR_CUDA(cudaGetLastError());
    // the whole CSR, for the exact recomputation of non-finite outputs
    VCSR_TRY(dmalloc(&p->d_seg_rp, (int64_t)M + 1));
    VCSR_TRY(dmalloc(&p->d_seg_col, nnz));
    VCSR_TRY(dmalloc(&p->d_seg_val, nnz));
    VCSR_CUDA(cudaMemcpyAsync(p->d_seg_rp, d.row_ptr, sizeof(int) * ((size_t)M + 1),
                              cudaMemcpyDeviceToDevice, st));
    if (nnz) {
      VCSR_CUDA(cudaMemcpyAsync(p->d_seg_col, d.col, sizeof(int) * (size_t)nnz,
                                cudaMemcpyDeviceToDevice, st));
      VCSR_CUDA(cudaMemcpyAsync(p->d_seg_val, d.val, sizeof(float) * (size_t)nnz,
                                cudaMemcpyDeviceToDevice, st));
    }
    if (!p->d_err && n_seg_rb > 0) {
      VCSR_TRY(dmalloc(&p->d_err, 1));
      VCSR_CUDA(cudaMemsetAsync(p->d_err, 0, sizeof(int), st));
    }
    p->n_seg_rb = n_seg_rb;
    p->n_seg_pieces = n_pieces;
    p->seg_rows = seg_rows;
    p->seg_min_run = min_run;
    p->seg_only = n_res == 0 && n_seg_rb == V16;
    acct(p, 4, n_seg_rb);
    acct(p, 4, (int64_t)n_seg_rb + 1);
    acct(p, 16, n_pieces);
    acct(p, 4, (int64_t)seg_rows * 16);
    acct(p, 4, (int64_t)M + 1);
    acct(p, 4, nnz);
    acct(p, 4, nnz);
    p->panel_nnz = (int64_t)nnz - n_res;
    work.nnz = n_res;
    work.row_ptr = r_rp;
    work.col = r_col;
    work.val = r_val;
  }

  // ---- vector height
  int R = params.vec_rows;
  if (R == 0) {
    VCSR_TRY(choose_vec_rows_device(work, sms, sc, &R));
    if (R == 8 && params.target_O > 128) R = 4;
  }
  if (R != 1 && R != 2 && R != 4 && R != 8 && R != 16)
    return fail(VCSR_ERR_INVALID, "vec_rows must be 1, 2, 4, 8 or 16 (got %d)", R);
  const int V = (int)ceil_div(M, R);
  const int nnz = work.nnz;

  // ---- vector panels: union columns, R values each, row masks
  int64_t U = nnz;
  VCSR_TRY(dmalloc(&p->d_vec_ptr, (int64_t)V + 1));
  if (R == 1) {
    VCSR_TRY(dmalloc(&p->d_ucol, U));
    VCSR_TRY(dmalloc(&p->d_uval, U));
    VCSR_CUDA(cudaMemcpyAsync(p->d_vec_ptr, work.row_ptr, sizeof(int) * ((size_t)M + 1),
                              cudaMemcpyDeviceToDevice, st));
    if (nnz) {
      VCSR_CUDA(cudaMemcpyAsync(p->d_ucol, work.col, sizeof(int) * (size_t)nnz,
                                cudaMemcpyDeviceToDevice, st));
      VCSR_CUDA(cudaMemcpyAsync(p->d_uval, work.val, sizeof(float) * (size_t)nnz,
                                cudaMemcpyDeviceToDevice, st));
    }
  } else {
    int *row_of = nullptr, *flag = nullptr, *F = nullptr;
    VCSR_TRY(sc.get(&row_of, nnz));
    VCSR_TRY(sc.get(&flag, nnz));
    VCSR_TRY(sc.get(&F, (int64_t)nnz + 1));
    row_of_kernel<<<grid_for((int64_t)M * 32), kThreads, 0, st>>>(work.row_ptr, M, row_of);
    first_flag_kernel<<<grid_for(nnz), kThreads, 0, st>>>(work.row_ptr, work.col, row_of, nnz,
                                                           R, flag);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(flag, F, nnz, F + nnz, sc));
    int u = 0;
    VCSR_TRY(read1(&u, F + nnz, st));
    U = u;
    if (U * R > ((int64_t)1 << 40))
      return fail(VCSR_ERR_UNSUPPORTED, "panel layout exceeds 32-bit indexing");
    VCSR_TRY(dmalloc(&p->d_ucol, U));
    VCSR_TRY(dmalloc(&p->d_uval, U * R));
    VCSR_TRY(dmalloc(&p->d_umask, U));
    VCSR_CUDA(cudaMemsetAsync(p->d_uval, 0, sizeof(float) * (size_t)(U * R), st));
    VCSR_CUDA(cudaMemsetAsync(p->d_umask, 0, sizeof(unsigned) * (size_t)U, st));
    vec_ptr_kernel<<<grid_for((int64_t)V + 1), kThreads, 0, st>>>(work.row_ptr, F, M, R, V,
                                                                    p->d_vec_ptr);
    place_kernel<<<grid_for(nnz), kThreads, 0, st>>>(work.row_ptr, work.col, work.val, row_of,
                                                      F, M, nnz, R, p->d_ucol, p->d_uval,
                                                      p->d_umask);
    VCSR_CUDA(cudaGetLastError());
    sc.release(row_of);
    sc.release(flag);
    sc.release(F);
  }
  p->R = R;
  p->num_vectors = V;
  p->num_union = U;
  acct(p, 4, (int64_t)V + 1);
  acct(p, 4, U);
  acct(p, 4, U * R);
  acct(p, 4, R > 1 ? U : 0);

  // ---- nnz-balanced units: chunk as the host builder picks it
  int chunk = params.chunk;
  if (chunk <= 0) {
    const int64_t per = U / ((int64_t)(sms > 0 ? sms : 148) * 32);
    const int64_t avg = V > 0 ? U / V : 0;
    const int64_t cap = std::max<int64_t>(512, 2 * avg);
    chunk = (int)std::max<int64_t>(256, std::min<int64_t>(std::min(per, cap), 2048));
  }
  p->chunk = chunk;
  int *nparts = nullptr, *split = nullptr, *sparts = nullptr, *uoff = nullptr, *svi = nullptr,
      *poff = nullptr;
  VCSR_TRY(sc.get(&nparts, V));
  VCSR_TRY(sc.get(&split, V));
  VCSR_TRY(sc.get(&sparts, V));
  VCSR_TRY(sc.get(&uoff, (int64_t)V + 1));
  VCSR_TRY(sc.get(&svi, (int64_t)V + 1));
  VCSR_TRY(sc.get(&poff, (int64_t)V + 1));
  vec_parts_kernel<<<grid_for(V), kThreads, 0, st>>>(p->d_vec_ptr, V, chunk, nparts, split,
                                                      sparts);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(scan_exclusive<int>(nparts, uoff, V, tot + 0, sc));
  VCSR_TRY(scan_exclusive<int>(split, svi, V, tot + 1, sc));
  VCSR_TRY(scan_exclusive<int>(sparts, poff, V, tot + 2, sc));
  int h3[3];
  VCSR_CUDA(cudaMemcpyAsync(h3, tot, sizeof h3, cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  const int n_units = V > 0 ? h3[0] : 0, n_sv = V > 0 ? h3[1] : 0, n_su = V > 0 ? h3[2] : 0;
  VCSR_TRY(dmalloc(&p->d_units, n_units));
  VCSR_TRY(dmalloc(&p->d_parts, n_su));
  VCSR_TRY(dmalloc(&p->d_svecs, n_sv));
  fill_units_kernel<<<grid_for(V), kThreads, 0, st>>>(p->d_vec_ptr, V, nparts, uoff, svi, poff,
                                                       p->d_units, p->d_parts, p->d_svecs);
  VCSR_CUDA(cudaGetLastError());
  p->n_units = n_units;
  p->n_split_units = n_su;
  p->n_split_vectors = n_sv;
  // split parts keep R x max_O partial sums and one ticket per O-tile
  p->pstride = std::max(params.max_O, 1);
  p->counter_stride = std::max(params.max_O, 1);

  // ---- long units and batches of short ones
  int *is_long = nullptr, *is_short = nullptr, *slen = nullptr, *lidx = nullptr, *kidx = nullptr,
      *Cs = nullptr, *bstart = nullptr, *bidx = nullptr;
  VCSR_TRY(sc.get(&is_long, n_units));
  VCSR_TRY(sc.get(&is_short, n_units));
  VCSR_TRY(sc.get(&slen, n_units));
  VCSR_TRY(sc.get(&lidx, (int64_t)n_units + 1));
  VCSR_TRY(sc.get(&kidx, (int64_t)n_units + 1));
  VCSR_TRY(sc.get(&Cs, (int64_t)n_units + 1));
  VCSR_TRY(sc.get(&bstart, n_units));
  VCSR_TRY(sc.get(&bidx, (int64_t)n_units + 1));
  classify_units_kernel<<<grid_for(n_units), kThreads, 0, st>>>(p->d_units, n_units, is_long,
                                                                 is_short, slen);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(scan_exclusive<int>(is_long, lidx, n_units, tot + 3, sc));
  VCSR_TRY(scan_exclusive<int>(is_short, kidx, n_units, tot + 4, sc));
  VCSR_TRY(scan_exclusive<int>(slen, Cs, n_units, tot + 5, sc));
  int h6[6];
  VCSR_CUDA(cudaMemcpyAsync(h6, tot, sizeof h6, cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  const int n_long = n_units > 0 ? h6[3] : 0;
  const int64_t short_cols = n_units > 0 ? h6[5] : 0;
  const int batch_cols =
      (int)std::max<int64_t>(16, std::min<int64_t>(256, short_cols / ((int64_t)sms * 64)));
  VCSR_TRY(dmalloc(&p->d_long, n_long));
  batch_start_kernel<<<grid_for(n_units), kThreads, 0, st>>>(n_units, R, batch_cols, is_long,
                                                              lidx, kidx, Cs, p->d_long, bstart);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(scan_exclusive<int>(bstart, bidx, n_units, tot + 6, sc));
  int n_batches = 0;
  if (n_units > 0) VCSR_TRY(read1(&n_batches, tot + 6, st));
  VCSR_TRY(dmalloc(&p->d_batches, n_batches));
  fill_batches_kernel<<<grid_for(n_units), kThreads, 0, st>>>(
      p->d_units, n_units, is_long, bstart, bidx, reinterpret_cast<int *>(p->d_batches));
  VCSR_CUDA(cudaGetLastError());
  p->n_batches = n_batches;
  p->n_long = n_long;
  acct(p, 16, n_units);
  acct(p, 8, n_su);
  acct(p, 8, n_sv);
  acct(p, 16, n_batches);
  acct(p, 4, n_long);

  // ---- row panels of the host entry point's row pipeline (plan.cu): cut at
  // vectors where a batch or a long unit starts, near 1/32, 1/6, ..., 5/6,
  // 31/32 of the entries
  if (p->n_panel_rb == 0 && p->n_seg_rb == 0 && M >= 8192 && nnz >= (1 << 20)) {
    constexpr int kRowPanels = 8;
    constexpr double kCut[kRowPanels - 1] = {1.0 / 32, 1.0 / 6, 2.0 / 6, 3.0 / 6,
                                             4.0 / 6,  5.0 / 6, 31.0 / 32};
    long long targets[kRowPanels - 1];
    for (int j = 0; j < kRowPanels - 1; ++j) targets[j] = (long long)(nnz * kCut[j]);
    long long *d_t = nullptr;
    int *d_rows = nullptr, *d_bv = nullptr, *d_lv = nullptr, *d_bounds = nullptr,
        *d_cm = nullptr;
    VCSR_TRY(sc.get(&d_t, kRowPanels - 1));
    VCSR_TRY(sc.get(&d_rows, kRowPanels - 1));
    VCSR_TRY(sc.get(&d_bv, n_batches));
    VCSR_TRY(sc.get(&d_lv, n_long));
    VCSR_CUDA(cudaMemcpyAsync(d_t, targets, sizeof targets, cudaMemcpyHostToDevice, st));
    row_cut_kernel<<<1, 32, 0, st>>>(work.row_ptr, M, d_t, kRowPanels - 1, d_rows);
    batch_v0_kernel<<<grid_for(n_batches), kThreads, 0, st>>>(
        reinterpret_cast<const int *>(p->d_batches), n_batches, d_bv);
    unit_vec_kernel<<<grid_for(n_long), kThreads, 0, st>>>(p->d_units, p->d_long, n_long, d_lv);
    VCSR_CUDA(cudaGetLastError());
    int rows[kRowPanels - 1];
    std::vector<int> bvec((size_t)n_batches), lvec((size_t)n_long);
    VCSR_CUDA(cudaMemcpyAsync(rows, d_rows, sizeof rows, cudaMemcpyDeviceToHost, st));
    if (n_batches)
      VCSR_CUDA(cudaMemcpyAsync(bvec.data(), d_bv, sizeof(int) * bvec.size(),
                                cudaMemcpyDeviceToHost, st));
    if (n_long)
      VCSR_CUDA(cudaMemcpyAsync(lvec.data(), d_lv, sizeof(int) * lvec.size(),
                                cudaMemcpyDeviceToHost, st));
    VCSR_CUDA(cudaStreamSynchronize(st));
    std::vector<int> cuts(bvec);
    cuts.insert(cuts.end(), lvec.begin(), lvec.end());
    std::sort(cuts.begin(), cuts.end());
    cuts.erase(std::unique(cuts.begin(), cuts.end()), cuts.end());
    std::vector<int> vb{0};
    for (int j = 0; j < kRowPanels - 1; ++j) {
      auto it = std::lower_bound(cuts.begin(), cuts.end(), rows[j] / R);
      if (it != cuts.end() && *it > vb.back()) vb.push_back(*it);
    }
    vb.push_back(V);
    const int np = (int)vb.size() - 1;
    std::vector<int> bounds(np), cm(np, -1);
    for (int j = 0; j < np; ++j) bounds[j] = vb[j] * R;
    VCSR_TRY(sc.get(&d_bounds, np));
    VCSR_TRY(sc.get(&d_cm, np));
    VCSR_CUDA(cudaMemcpyAsync(d_bounds, bounds.data(), sizeof(int) * np, cudaMemcpyHostToDevice,
                              st));
    VCSR_CUDA(cudaMemcpyAsync(d_cm, cm.data(), sizeof(int) * np, cudaMemcpyHostToDevice, st));
    panel_colmax_kernel<<<grid_for(M), kThreads, 0, st>>>(work.row_ptr, work.col, M, d_bounds,
                                                          np, d_cm);
    VCSR_CUDA(cudaGetLastError());
    VCSR_CUDA(cudaMemcpyAsync(cm.data(), d_cm, sizeof(int) * np, cudaMemcpyDeviceToHost, st));
    VCSR_CUDA(cudaStreamSynchronize(st));
    for (int j = 0; j < np; ++j) {
      vcsr_plan::RowPanel rp;
      rp.row0 = vb[j] * R;
      rp.row1 = std::min(M, vb[j + 1] * R);
      rp.b0 = (int)(std::lower_bound(bvec.begin(), bvec.end(), vb[j]) - bvec.begin());
      rp.b1 = (int)(std::lower_bound(bvec.begin(), bvec.end(), vb[j + 1]) - bvec.begin());
      rp.l0 = (int)(std::lower_bound(lvec.begin(), lvec.end(), vb[j]) - lvec.begin());
      rp.l1 = (int)(std::lower_bound(lvec.begin(), lvec.end(), vb[j + 1]) - lvec.begin());
      rp.col_max = cm[j];
      p->rpanels.push_back(rp);
    }
  }
  return VCSR_OK;
}

}  // namespace vcsr
