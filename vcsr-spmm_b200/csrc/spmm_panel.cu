// spmm_panel.cu — the row-stationary VCSR SpMM kernel for sm_100a.
//
// C[M x O] = A * B with A in vector panels (panel.h).  One sub-warp of L lanes
// owns one work item = (unit, O-tile).  Lanes lie across O: lane l holds
// columns k = tile*W + v*L*VW + l*VW (VW = 4 floats per 128-bit access, NV
// such vectors per lane), so a B row segment is one coalesced 128-bit load per
// lane.  The R rows of the vector accumulate in registers (C stationary) while
// the sub-warp walks the unit's union columns in order: per column one load
// of the column index, one 16..64-byte load of the R values (the same address
// for the whole sub-warp) and NV B loads feed R*NV*VW FMAs per lane.  Each
// row's FMA chain follows its CSR order, so an unsplit vector's row equals the
// CSR reference bit for bit.  Unsplit units store C once with streaming
// stores (beta = 0, no zero-fill pass); parts of a split vector store partial
// sums and the last part to arrive (atomic ticket, no waiting) adds the parts
// in part order and writes C.
//
// The long-row scheme of src/aspt.cu:38-142 (a warp shares one row's entries
// and broadcasts them) appears here as the sub-warp walking one vector, with
// the entries read by address-uniform loads instead of __shfl_sync.
#include <cuda_runtime.h>

#include <mutex>

#include "common.h"
#include "spmm_kernels.h"

namespace vcsr {

namespace {

template <int VW>
struct VecT;
template <>
struct VecT<4> {
  using T = float4;
  static __device__ __forceinline__ T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
  static __device__ __forceinline__ T ld(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
  }
  static __device__ __forceinline__ T ldcg(const float *p) {
    return __ldcg(reinterpret_cast<const float4 *>(p));
  }
  static __device__ __forceinline__ void st(float *p, T v) {
    *reinterpret_cast<float4 *>(p) = v;
  }
  static __device__ __forceinline__ void stcs(float *p, T v) {
    __stcs(reinterpret_cast<float4 *>(p), v);
  }
  static __device__ __forceinline__ T fma(float a, T b, T c) {
    return make_float4(fmaf(a, b.x, c.x), fmaf(a, b.y, c.y), fmaf(a, b.z, c.z),
                       fmaf(a, b.w, c.w));
  }
  static __device__ __forceinline__ T add(T a, T b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  }
};
template <>
struct VecT<1> {
  using T = float;
  static __device__ __forceinline__ T zero() { return 0.f; }
  static __device__ __forceinline__ T ld(const float *p) { return __ldg(p); }
  static __device__ __forceinline__ T ldcg(const float *p) { return __ldcg(p); }
  static __device__ __forceinline__ void st(float *p, T v) { *p = v; }
  static __device__ __forceinline__ void stcs(float *p, T v) { __stcs(p, v); }
  static __device__ __forceinline__ T fma(float a, T b, T c) { return fmaf(a, b, c); }
  static __device__ __forceinline__ T add(T a, T b) { return a + b; }
};

template <int R>
__device__ __forceinline__ void load_vals(const float *__restrict__ uval, int j,
                                          float (&a)[R]) {
  if constexpr (R == 1) {
    a[0] = __ldg(uval + j);
  } else if constexpr (R == 2) {
    const float2 t = __ldg(reinterpret_cast<const float2 *>(uval) + j);
    a[0] = t.x;
    a[1] = t.y;
  } else {
    const float4 *p = reinterpret_cast<const float4 *>(uval + (size_t)j * R);
#pragma unroll
    for (int q = 0; q < R / 4; ++q) {
      const float4 t = __ldg(p + q);
      a[4 * q + 0] = t.x;
      a[4 * q + 1] = t.y;
      a[4 * q + 2] = t.z;
      a[4 * q + 3] = t.w;
    }
  }
}

template <int R, int NV, int VW, int UNROLL, bool ROWPTR>
__global__ void __launch_bounds__(256)
    panel_spmm_kernel(const PanelDevView P, const float *__restrict__ B, int ldb,
                      float *__restrict__ C, int ldc, int O, int lshift,
                      int n_otiles, int W) {
  using V = VecT<VW>;
  using T = typename V::T;
  const int L = 1 << lshift;
  const int lane = threadIdx.x & 31;
  const int sub = lane >> lshift;
  const int sl = lane & (L - 1);
  const unsigned submask =
      (L == 32) ? 0xffffffffu : (((1u << L) - 1u) << (sub * L));
  const int subs = 32 >> lshift;
  const long long gsw =
      ((long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * subs + sub;
  const long long nsw = (long long)gridDim.x * (blockDim.x >> 5) * subs;
  const long long n_items = (long long)P.n_units * n_otiles;

  for (long long item = gsw; item < n_items; item += nsw) {
    const int u = (int)(item / n_otiles);
    const int ot = (int)(item - (long long)u * n_otiles);
    int4 U;
    if constexpr (ROWPTR) {
      U = make_int4(u, __ldg(P.row_ptr + u), __ldg(P.row_ptr + u + 1), -1);
    } else {
      U = __ldg(P.units + u);
    }
    int kk[NV];
    bool ok[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      kk[v] = ot * W + v * (L * VW) + sl * VW;
      ok[v] = kk[v] < O;
    }
    T acc[R][NV];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v) acc[r][v] = V::zero();

    int j = U.y;
    const int end = U.z;
    for (; j + UNROLL <= end; j += UNROLL) {
      int c[UNROLL];
      float a[UNROLL][R];
      T b[UNROLL][NV];
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) c[q] = __ldg(P.ucol + j + q);
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) load_vals<R>(P.uval, j + q, a[q]);
#pragma unroll
      for (int q = 0; q < UNROLL; ++q) {
        const float *bp = B + (size_t)c[q] * ldb;
#pragma unroll
        for (int v = 0; v < NV; ++v) b[q][v] = ok[v] ? V::ld(bp + kk[v]) : V::zero();
      }
#pragma unroll
      for (int q = 0; q < UNROLL; ++q)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int v = 0; v < NV; ++v) acc[r][v] = V::fma(a[q][r], b[q][v], acc[r][v]);
    }
    for (; j < end; ++j) {
      const int c = __ldg(P.ucol + j);
      float a[R];
      load_vals<R>(P.uval, j, a);
      const float *bp = B + (size_t)c * ldb;
      T b[NV];
#pragma unroll
      for (int v = 0; v < NV; ++v) b[v] = ok[v] ? V::ld(bp + kk[v]) : V::zero();
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = V::fma(a[r], b[v], acc[r][v]);
    }

    const int row0 = U.x * R;
    if (U.w < 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (row < P.M) {
#pragma unroll
          for (int v = 0; v < NV; ++v)
            if (ok[v]) V::stcs(C + (size_t)row * ldc + kk[v], acc[r][v]);
        }
      }
    } else {
      // split vector: publish this part, last part to arrive reduces
      const int slot = U.w;
      float *part = P.partials + (size_t)slot * R * P.pstride;
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v)
          if (ok[v]) V::st(part + (size_t)r * P.pstride + kk[v], acc[r][v]);
      __threadfence();
      __syncwarp(submask);
      const int2 sp = __ldg(P.parts + slot);       // {split vector, part}
      const int2 svi = __ldg(P.svecs + sp.x);      // {first slot, nparts}
      int ticket = 0;
      int *ctr = P.counters + (size_t)sp.x * P.counter_stride + ot;
      if (sl == 0) ticket = atomicAdd(ctr, 1);
      ticket = __shfl_sync(submask, ticket, 0, L);
      if (ticket == svi.y - 1) {
        __threadfence();
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int row = row0 + r;
          if (row >= P.M) continue;
#pragma unroll
          for (int v = 0; v < NV; ++v) {
            if (!ok[v]) continue;
            T s = V::zero();
            for (int p = 0; p < svi.y; ++p)
              s = V::add(s, V::ldcg(P.partials +
                                    ((size_t)(svi.x + p) * R + r) * P.pstride + kk[v]));
            V::stcs(C + (size_t)row * ldc + kk[v], s);
          }
        }
        if (sl == 0) *ctr = 0;  // ready for the next launch
      }
    }
  }
}

using KernelFn = void (*)(const PanelDevView, const float *, int, float *, int,
                          int, int, int, int);

template <int R, int NV, int VW, bool ROWPTR>
constexpr KernelFn kfn() {
  return panel_spmm_kernel<R, NV, VW, (R <= 4 ? 4 : (R == 8 ? 2 : 1)), ROWPTR>;
}

KernelFn select_kernel(int R, int NV, int VW, bool rowptr) {
  if (rowptr) {
    if (NV == 1) return VW == 4 ? kfn<1, 1, 4, true>() : kfn<1, 1, 1, true>();
    return VW == 4 ? kfn<1, 2, 4, true>() : kfn<1, 2, 1, true>();
  }
#define VCSR_SEL(RR)                                                         \
  case RR:                                                                   \
    if (NV == 1) return VW == 4 ? kfn<RR, 1, 4, false>() : kfn<RR, 1, 1, false>(); \
    return VW == 4 ? kfn<RR, 2, 4, false>() : kfn<RR, 2, 1, false>();
  switch (R) {
    VCSR_SEL(1)
    VCSR_SEL(2)
    VCSR_SEL(4)
    VCSR_SEL(8)
    case 16:
      return VW == 4 ? kfn<16, 1, 4, false>() : kfn<16, 1, 1, false>();
  }
#undef VCSR_SEL
  return nullptr;
}

int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

int sm_count() {
  static int cached = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (!cached) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&cached, cudaDevAttrMultiProcessorCount, dev);
    if (cached <= 0) cached = 148;
  }
  return cached;
}

}  // namespace

LaunchShape pick_shape(int O, int R, bool vec4) {
  LaunchShape s;
  s.VW = vec4 ? 4 : 1;
  const int per = (int)ceil_div(O, s.VW);
  const int L = next_pow2(per < 32 ? (per > 0 ? per : 1) : 32);
  s.NV = (per > 32 && R <= 8) ? 2 : 1;
  s.lshift = 0;
  while ((1 << s.lshift) < L) ++s.lshift;
  s.W = L * s.VW * s.NV;
  s.n_otiles = (int)ceil_div(O, s.W);
  return s;
}

vcsr_status launch_panel_spmm(const PanelDevView &P, bool rowptr,
                              const float *B, int ldb, float *C, int ldc, int O,
                              cudaStream_t st, int *launches) {
  if (launches) *launches = 0;
  if (O <= 0 || P.n_units <= 0) return VCSR_OK;
  const bool vec4 = (O % 4 == 0) && (ldb % 4 == 0) && (ldc % 4 == 0) &&
                    ((uintptr_t)B % 16 == 0) && ((uintptr_t)C % 16 == 0);
  const LaunchShape s = pick_shape(O, P.R, vec4);
  KernelFn fn = select_kernel(P.R, s.NV, s.VW, rowptr);
  if (!fn) return fail(VCSR_ERR_UNSUPPORTED, "no kernel for R=%d", P.R);
  if (!rowptr && P.n_split_units > 0 && (O > P.pstride || s.n_otiles > P.counter_stride))
    return fail(VCSR_ERR_INVALID, "O=%d exceeds the plan's max_O=%d", O, P.pstride);
  const int threads = 256;
  int per_sm = 0;
  VCSR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0));
  if (per_sm <= 0) per_sm = 1;
  const int subs_per_block = (threads / 32) * (32 >> s.lshift);
  const long long items = (long long)P.n_units * s.n_otiles;
  long long blocks = (items + subs_per_block - 1) / subs_per_block;
  const long long cap = (long long)sm_count() * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  fn<<<(int)blocks, threads, 0, st>>>(P, B, ldb, C, ldc, O, s.lshift, s.n_otiles, s.W);
  VCSR_CUDA(cudaGetLastError());
  if (launches) *launches = 1;
  return VCSR_OK;
}

}  // namespace vcsr

extern "C" vcsr_status vcsr_csr_spmm(int M, const int *d_row_ptr, const int *d_col,
                                     const float *d_val, const float *dB, int O,
                                     float *dC, vcsr_stream_t stream) {
  vcsr::clear_error();
  if (M < 0 || O < 0) return vcsr::fail(VCSR_ERR_INVALID, "negative size");
  if (M == 0 || O == 0) return VCSR_OK;
  if (!d_row_ptr || !dB || !dC)
    return vcsr::fail(VCSR_ERR_INVALID, "null device pointer");
  vcsr::PanelDevView P{};
  P.row_ptr = d_row_ptr;
  P.ucol = d_col;
  P.uval = d_val;
  P.n_units = M;
  P.M = M;
  P.R = 1;
  return vcsr::launch_panel_spmm(P, true, dB, O, dC, O, O, (cudaStream_t)stream,
                                 nullptr);
}
