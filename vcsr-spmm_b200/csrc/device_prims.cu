// device_prims.cu — exclusive scan (reduce, scan the block sums, scan again
// with the block offsets) and stable LSD radix sort (per-tile digit
// histograms, one scan over [digit][tile], rank-preserving scatter).
#include "device_prims.cuh"

namespace vcsr {

namespace {

constexpr int kScanThreads = 512;
constexpr int kScanItems = 4;
constexpr int kScanTile = kScanThreads * kScanItems;

template <class T>
__device__ T block_exclusive_scan(T x, T *smem_warp, T *block_total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T incl = x;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) smem_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    T w = lane < nw ? smem_warp[lane] : T(0);
    T wi = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T y = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += y;
    }
    if (lane < nw) smem_warp[lane] = wi - w;
    if (lane == nw - 1) *block_total = wi;
  }
  __syncthreads();
  return incl - x + smem_warp[warp];
}

template <class T>
__global__ void scan_reduce_kernel(const T *in, int64_t n, T *sums) {
  __shared__ T warp_s[32];
  __shared__ T tot;
  const int64_t base = (int64_t)blockIdx.x * kScanTile + threadIdx.x * kScanItems;
  T s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i)
    if (base + i < n) s += in[base + i];
  block_exclusive_scan<T>(s, warp_s, &tot);
  if (threadIdx.x == 0) sums[blockIdx.x] = tot;
}

template <class T>
__global__ void scan_final_kernel(const T *in, T *out, int64_t n,
                                  const T *offsets, T *total) {
  __shared__ T warp_s[32];
  __shared__ T tot;
  const int64_t base = (int64_t)blockIdx.x * kScanTile + threadIdx.x * kScanItems;
  T v[kScanItems];
  T s = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    v[i] = (base + i < n) ? in[base + i] : T(0);
    s += v[i];
  }
  T ex = block_exclusive_scan<T>(s, warp_s, &tot);
  const T off = offsets ? offsets[blockIdx.x] : T(0);
  T run = ex + off;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    if (base + i < n) out[base + i] = run;
    run += v[i];
  }
  if (total && blockIdx.x == gridDim.x - 1 && threadIdx.x == 0) *total = off + tot;
}

template <class T>
__global__ void set_zero_kernel(T *p) { *p = 0; }

// ------------------------------------------------------------ radix sort
constexpr int kSortThreads = 256;
constexpr int kSortItems = 8;
constexpr int kSortTile = kSortThreads * kSortItems;
constexpr int kDigits = 256;

__global__ void radix_hist_kernel(const uint32_t *keys, int64_t n, int shift,
                                  int num_tiles, int *hist) {
  __shared__ int h[kDigits];
  h[threadIdx.x] = 0;
  __syncthreads();
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
#pragma unroll
  for (int i = 0; i < kSortItems; ++i) {
    const int64_t idx = base + (int64_t)i * kSortThreads + threadIdx.x;
    if (idx < n) atomicAdd(&h[(keys[idx] >> shift) & 0xFF], 1);
  }
  __syncthreads();
  hist[(int64_t)threadIdx.x * num_tiles + blockIdx.x] = h[threadIdx.x];
}

// Elements are visited round by round (round i covers tile positions
// i*256 .. i*256+255) and within a round in thread order, which is the input
// order, so equal digits keep their relative order.
__global__ void radix_scatter_kernel(const uint32_t *keys, const int *vals,
                                     int64_t n, int shift, int num_tiles,
                                     const int *offsets, uint32_t *keys_out,
                                     int *vals_out) {
  __shared__ int run[kDigits];        // elements of each digit placed so far
  __shared__ int wcount[8][kDigits];  // per-warp counts of this round
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  run[threadIdx.x] = 0;
  const int64_t base = (int64_t)blockIdx.x * kSortTile;
  const unsigned lt = (1u << lane) - 1u;
  for (int i = 0; i < kSortItems; ++i) {
    for (int w = 0; w < 8; ++w) wcount[w][threadIdx.x] = 0;
    __syncthreads();
    const int64_t idx = base + (int64_t)i * kSortThreads + threadIdx.x;
    const bool valid = idx < n;
    uint32_t key = valid ? keys[idx] : 0u;
    // invalid lanes use a digit slot of their own (never written)
    const int d = valid ? (int)((key >> shift) & 0xFF) : -1;
    const unsigned peers = __match_any_sync(0xffffffffu, d);
    const int within = __popc(peers & lt);
    if (valid && within == 0) wcount[warp][d] = __popc(peers);
    __syncthreads();
    if (valid) {
      int before = 0;
      for (int w = 0; w < warp; ++w) before += wcount[w][d];
      const int rank = run[d] + before + within;
      const int64_t pos = (int64_t)offsets[(int64_t)d * num_tiles + blockIdx.x] + rank;
      keys_out[pos] = key;
      vals_out[pos] = vals[idx];
    }
    __syncthreads();
    int add = 0;
    for (int w = 0; w < 8; ++w) add += wcount[w][threadIdx.x];
    run[threadIdx.x] += add;
    __syncthreads();
  }
}

}  // namespace

template <class T>
vcsr_status scan_exclusive(const T *in, T *out, int64_t n, T *total,
                           Scratch &sc) {
  if (n <= 0) {
    if (total) {
      set_zero_kernel<T><<<1, 1, 0, sc.st>>>(total);
      VCSR_CUDA(cudaGetLastError());
    }
    return VCSR_OK;
  }
  const int64_t blocks = ceil_div(n, kScanTile);
  if (blocks == 1) {
    scan_final_kernel<T><<<1, kScanThreads, 0, sc.st>>>(in, out, n, nullptr, total);
    VCSR_CUDA(cudaGetLastError());
    return VCSR_OK;
  }
  T *sums = nullptr, *offs = nullptr;
  VCSR_TRY(sc.get(&sums, blocks));
  VCSR_TRY(sc.get(&offs, blocks));
  scan_reduce_kernel<T><<<(unsigned)blocks, kScanThreads, 0, sc.st>>>(in, n, sums);
  VCSR_CUDA(cudaGetLastError());
  VCSR_TRY(scan_exclusive<T>(sums, offs, blocks, nullptr, sc));
  scan_final_kernel<T><<<(unsigned)blocks, kScanThreads, 0, sc.st>>>(in, out, n,
                                                                     offs, total);
  VCSR_CUDA(cudaGetLastError());
  return VCSR_OK;
}

template vcsr_status scan_exclusive<int>(const int *, int *, int64_t, int *,
                                         Scratch &);
template vcsr_status scan_exclusive<long long>(const long long *, long long *,
                                               int64_t, long long *, Scratch &);

vcsr_status radix_sort_pairs(const uint32_t *keys_in, const int *vals_in,
                             uint32_t *keys_out, int *vals_out, int64_t n,
                             int bits, Scratch &sc) {
  if (n <= 0) return VCSR_OK;
  if (n > INT32_MAX) return fail(VCSR_ERR_UNSUPPORTED, "sort of > 2^31 items");
  const int passes = bits <= 0 ? 1 : (int)ceil_div(bits, 8);
  const int64_t tiles = ceil_div(n, kSortTile);
  int *hist = nullptr, *offs = nullptr;
  uint32_t *kb = nullptr;
  int *vb = nullptr;
  VCSR_TRY(sc.get(&hist, tiles * kDigits));
  VCSR_TRY(sc.get(&offs, tiles * kDigits));
  VCSR_TRY(sc.get(&kb, n));
  VCSR_TRY(sc.get(&vb, n));
  // ping-pong so that the last pass writes keys_out / vals_out
  const uint32_t *src_k = keys_in;
  const int *src_v = vals_in;
  for (int p = 0; p < passes; ++p) {
    const bool to_out = ((passes - 1 - p) % 2) == 0;
    uint32_t *dk = to_out ? keys_out : kb;
    int *dv = to_out ? vals_out : vb;
    radix_hist_kernel<<<(unsigned)tiles, kSortThreads, 0, sc.st>>>(src_k, n, 8 * p,
                                                                  (int)tiles, hist);
    VCSR_CUDA(cudaGetLastError());
    VCSR_TRY(scan_exclusive<int>(hist, offs, tiles * kDigits, nullptr, sc));
    radix_scatter_kernel<<<(unsigned)tiles, kSortThreads, 0, sc.st>>>(
        src_k, src_v, n, 8 * p, (int)tiles, offs, dk, dv);
    VCSR_CUDA(cudaGetLastError());
    src_k = dk;
    src_v = dv;
  }
  return VCSR_OK;
}

}  // namespace vcsr
