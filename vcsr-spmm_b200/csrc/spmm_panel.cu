// spmm_panel.cu — the row-stationary VCSR SpMM kernel for sm_100a.
//
// C[M x O] = A * B with A in vector panels (panel.h).  Lanes lie across O: a
// sub-warp of L lanes covers an O-tile of W = L*VW*NV columns (VW = 4 floats
// per 128-bit access, NV accesses per lane), so one B row segment is one
// coalesced 128-bit load per lane.  The R rows of a vector accumulate in
// registers (C stationary) while the team walks the unit's union columns.
//
// Per team and per chunk of union columns, the column indices and R-value
// vectors are copied global -> shared with cp.async into one of two buffers
// (the next chunk is in flight while the current one is consumed), so B row
// addresses never wait on a global load; B rows are then loaded U at a time
// per lane before the FMAs that use them.
//
// Two team shapes share one launch (a warp takes one work item):
//  * a group of 32/L short units, one per sub-warp; each row's FMA chain
//    follows its CSR order, so such rows equal the CSR reference bit for bit;
//  * one long unit, all 32/L sub-warps of the warp ("column groups") taking
//    every (32/L)-th union column; the column groups are then summed with a
//    fixed xor-shuffle tree (the long-row scheme of src/aspt.cu:38-142 --
//    a warp shares one row -- with the warp split over columns instead of
//    the row's entries being broadcast).
// A vector longer than the plan's chunk is split over several units; each
// part stores its R x O partial sums and the last part to finish (atomic
// ticket, no waiting) adds the parts in fixed order and writes C.  Results
// are therefore deterministic run to run.  C is written, never read
// (beta = 0), with streaming stores.
#include <cuda_runtime.h>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

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
  static __device__ __forceinline__ T shfl_xor(unsigned m, T v, int o) {
    return make_float4(__shfl_xor_sync(m, v.x, o), __shfl_xor_sync(m, v.y, o),
                       __shfl_xor_sync(m, v.z, o), __shfl_xor_sync(m, v.w, o));
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
  static __device__ __forceinline__ T shfl_xor(unsigned m, T v, int o) {
    return __shfl_xor_sync(m, v, o);
  }
};

// B values widened to FP32 as they are loaded: FP32 as stored; BF16 by
// placing its 16 bits in the high half of a float, FP16 by the half-to-float
// conversion (both exact), four values per 8-byte load with 128-bit lanes.
template <int VW>
struct LdB;
template <>
struct LdB<4> {
  static __device__ __forceinline__ float4 ld(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
  }
  static __device__ __forceinline__ float4 ld(const __nv_bfloat16 *p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p));
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                       __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
  }
  static __device__ __forceinline__ float4 ld(const __half *p) {
    const uint2 u = __ldg(reinterpret_cast<const uint2 *>(p));
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&u.y));
    return make_float4(a.x, a.y, b.x, b.y);
  }
};
template <>
struct LdB<1> {
  static __device__ __forceinline__ float ld(const float *p) { return __ldg(p); }
  static __device__ __forceinline__ float ld(const __nv_bfloat16 *p) {
    return __uint_as_float((unsigned)__ldg(reinterpret_cast<const unsigned short *>(p)) << 16);
  }
  static __device__ __forceinline__ float ld(const __half *p) {
    return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short *>(p))));
  }
};

// ---------------------------------------------------------------- cp.async
__device__ __forceinline__ void cp_async4(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async8(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::);
}
__device__ __forceinline__ void cp_async_wait_1() {
  asm volatile("cp.async.wait_group 1;\n" ::);
}

// Copy union columns [c0, c0+n) of a unit into a team buffer:
// scol[0..n) and sval[0..n*R).  Lanes t = 0..T-1 of the team share the work.
template <int R>
__device__ __forceinline__ void stage_chunk(const int *__restrict__ ucol,
                                            const float *__restrict__ uval, int c0,
                                            int n, int *scol, float *sval, int t,
                                            int T) {
  for (int i = t; i < n; i += T) cp_async4(scol + i, ucol + c0 + i);
  if constexpr (R >= 4) {
    const int nv = n * (R / 4);
    const float *src = uval + (size_t)c0 * R;
    for (int i = t; i < nv; i += T) cp_async16(sval + 4 * i, src + 4 * i);
  } else if constexpr (R == 2) {
    const float *src = uval + (size_t)c0 * 2;
    for (int i = t; i < n; i += T) cp_async8(sval + 2 * i, src + 2 * i);
  } else {
    for (int i = t; i < n; i += T) cp_async4(sval + i, uval + c0 + i);
  }
}

template <int R>
__device__ __forceinline__ void load_vals_smem(const float *sval, int j, float (&a)[R]) {
  if constexpr (R == 1) {
    a[0] = sval[j];
  } else if constexpr (R == 2) {
    const float2 t = reinterpret_cast<const float2 *>(sval)[j];
    a[0] = t.x;
    a[1] = t.y;
  } else {
    const float4 *p = reinterpret_cast<const float4 *>(sval + j * R);
#pragma unroll
    for (int q = 0; q < R / 4; ++q) {
      const float4 t = p[q];
      a[4 * q + 0] = t.x;
      a[4 * q + 1] = t.y;
      a[4 * q + 2] = t.z;
      a[4 * q + 3] = t.w;
    }
  }
}

// Columns per prefetch group: B loads of group g+1 are in flight while
// group g is consumed, so a lane holds 2 * UN * NV 128-bit B values.
// Per-instantiation tuning, measured on B200 (tests of unroll depth and
// register caps over the five workloads): UN = columns per prefetch group
// (two groups in flight), MINB = blocks of 256 threads that must fit on an
// SM (caps registers at 65536 / (256 * MINB)).  VCSR_TUNE_UN / _MINB override
// both for experiments.
template <int R, int NV, int VW>
constexpr int unroll_for() {
#ifdef VCSR_TUNE_UN
  return VCSR_TUNE_UN;
#else
  if (VW == 1) return R <= 4 ? (NV == 1 ? 8 : 4) : (R == 8 ? (NV == 1 ? 4 : 2) : 2);
  if (R <= 4) return NV == 1 ? 4 : (R == 4 ? 2 : (R == 2 ? 4 : 2));
  return 2 + (R == 8 && NV == 1 ? 2 : 0);
#endif
}
template <int R, int NV, int VW>
constexpr int min_blocks_for() {
#ifdef VCSR_TUNE_MINB
  return VCSR_TUNE_MINB;
#else
  if (VW == 1) return 1;
  if (NV == 4) return 2;
  if (R <= 4) return NV == 1 ? 3 : (R == 1 ? 4 : 2);
  if (R == 8) return NV == 1 ? 2 : 1;
  return 2;
#endif
}

// The long-unit kernel also runs the split fixup, so it keeps at most 2
// blocks per SM, except R = 1 with two column vectors per lane (power-law
// rows at O >= 256), measured faster at 3 (80 registers, no real spill:
// R-MAT 2^22 at O = 256, 7.3 -> 6.5 ms).
template <int R, int NV, int VW>
constexpr int long_min_blocks_for() {
  if (VW == 4 && R == 1 && NV == 2) return 3;
  return min_blocks_for<R, NV, VW>() < 2 ? min_blocks_for<R, NV, VW>() : 2;
}

// Accumulators.  With 128-bit lanes the sums are kept as float2 pairs so that
// one packed FFMA2 (__ffma2_rn: two round-to-nearest fused multiply-adds,
// bit-identical to two fmaf) does two updates: pairs of rows (r, r+1) at one
// column when R >= 2, pairs of columns of one row when R = 1.  The scalar
// path (VW = 1) keeps one float per row.
template <int R, int NV, int VW>
struct Acc;

template <int R, int NV>
struct Acc<R, NV, 4> {
  static constexpr bool kRowPairs = R >= 2;
  static constexpr int kP = kRowPairs ? R / 2 : 1;
  static constexpr int kC = kRowPairs ? 4 : 2;
  float2 p[kP][NV][kC];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < kP; ++i)
#pragma unroll
      for (int v = 0; v < NV; ++v)
#pragma unroll
        for (int c = 0; c < kC; ++c) p[i][v][c] = make_float2(0.f, 0.f);
  }
  // one union column: values a[R] of the R rows, B values b[NV]
  __device__ __forceinline__ void fma(const float (&a)[R], const float4 (&b)[NV]) {
    if constexpr (kRowPairs) {
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const float2 bx = make_float2(b[v].x, b[v].x), by = make_float2(b[v].y, b[v].y);
        const float2 bz = make_float2(b[v].z, b[v].z), bw = make_float2(b[v].w, b[v].w);
#pragma unroll
        for (int i = 0; i < kP; ++i) {
          const float2 ar = make_float2(a[2 * i], a[2 * i + 1]);
          p[i][v][0] = __ffma2_rn(ar, bx, p[i][v][0]);
          p[i][v][1] = __ffma2_rn(ar, by, p[i][v][1]);
          p[i][v][2] = __ffma2_rn(ar, bz, p[i][v][2]);
          p[i][v][3] = __ffma2_rn(ar, bw, p[i][v][3]);
        }
      }
    } else {
      const float2 aa = make_float2(a[0], a[0]);
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        p[0][v][0] = __ffma2_rn(aa, make_float2(b[v].x, b[v].y), p[0][v][0]);
        p[0][v][1] = __ffma2_rn(aa, make_float2(b[v].z, b[v].w), p[0][v][1]);
      }
    }
  }
  __device__ __forceinline__ void store(float4 (&out)[R][NV]) const {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if constexpr (kRowPairs) {
#pragma unroll
        for (int i = 0; i < kP; ++i) {
          out[2 * i][v] = make_float4(p[i][v][0].x, p[i][v][1].x, p[i][v][2].x, p[i][v][3].x);
          out[2 * i + 1][v] = make_float4(p[i][v][0].y, p[i][v][1].y, p[i][v][2].y, p[i][v][3].y);
        }
      } else {
        out[0][v] = make_float4(p[0][v][0].x, p[0][v][0].y, p[0][v][1].x, p[0][v][1].y);
      }
    }
  }
};

template <int R, int NV>
struct Acc<R, NV, 1> {
  float s[R][NV];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v) s[r][v] = 0.f;
  }
  __device__ __forceinline__ void fma(const float (&a)[R], const float (&b)[NV]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v) s[r][v] = fmaf(a[r], b[v], s[r][v]);
  }
  __device__ __forceinline__ void store(float (&out)[R][NV]) const {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v) out[r][v] = s[r][v];
  }
};

// B row `c` at this lane's offset: one wide multiply-add of the column
// index by the row pitch in bytes (a 32 x 32 -> 64-bit product; the host
// refuses pitches of 2^31 bytes or more).  Measured on B200 against a 64-bit
// index product: FEM O=128 57.3 -> 53.4 us, block-dense O=512 1.86 -> 1.68 ms.
template <class TB>
__device__ __forceinline__ const TB *b_row(const TB *Bk, int c, int ldb) {
  return reinterpret_cast<const TB *>(reinterpret_cast<const char *>(Bk) +
                                      (long long)c * (int)(ldb * (int)sizeof(TB)));
}

// B values of UN columns j0, j0+step, ...; FULL = all UN exist.
template <int NV, int VW, int UN, bool FULL, class TB = float>
__device__ __forceinline__ void load_group(const TB *__restrict__ Bk, int ldb,
                                           const int *scol, int j0, int step, int n,
                                           const bool (&ok)[NV], int vstride,
                                           typename VecT<VW>::T (&b)[UN][NV]) {
  using V = VecT<VW>;
  if constexpr (FULL && UN % 4 == 0) {
    // consecutive columns from a 16-byte aligned start: one shared-memory
    // load of four column indices (staging buffers hold multiples of four)
    if (step == 1 && (j0 & 3) == 0) {
#pragma unroll
      for (int q4 = 0; q4 < UN / 4; ++q4) {
        const int4 c4 = *reinterpret_cast<const int4 *>(scol + j0 + 4 * q4);
        const int cs[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const TB *bp = b_row(Bk, cs[e], ldb);
#pragma unroll
          for (int v = 0; v < NV; ++v)
            b[4 * q4 + e][v] = ok[v] ? LdB<VW>::ld(bp + v * vstride) : V::zero();
        }
      }
      return;
    }
  }
#pragma unroll
  for (int q = 0; q < UN; ++q) {
    const int j = j0 + q * step;
    if (FULL || j < n) {
      const TB *bp = b_row(Bk, scol[j], ldb);
#pragma unroll
      for (int v = 0; v < NV; ++v) b[q][v] = ok[v] ? LdB<VW>::ld(bp + v * vstride) : V::zero();
    }
  }
}

// Vector boundaries inside a batch of consecutive vectors: `v` is the vector
// being summed, [vb, ve) its union range (svp holds vec_ptr[v0..v1]).
struct BatchCursor {
  int v, ve, v0;
  const int *svp;
  int vb;
};

// Non-finite padding.  A vector of R > 1 rows multiplies, for each union
// column, all R rows' values by the B row, zeros included where a row lacks
// the column.  For finite B that adds exact zeros, but a padding zero times an
// Inf or NaN of B is NaN, in a row whose CSR sum (src/kernels.cu:27-31) never
// reads that B row.  Such a wrong value is always NaN, so a lane whose sums
// hold a NaN (or an Inf - Inf: the check is one sum) recomputes its columns of
// the vector's rows over the rows' own entries (umask), in union order, which
// is each row's CSR order.  The common, finite case costs one sum per store.
template <int R, int NV, int VW>
__device__ __forceinline__ bool sums_have_nan(const typename VecT<VW>::T (&o)[R][NV]) {
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if constexpr (VW == 4) {
        s += (o[r][v].x + o[r][v].y) + (o[r][v].z + o[r][v].w);
      } else {
        s += o[r][v];
      }
    }
  return s != s;
}

// This lane's columns kk[] of the vector's R rows over union columns
// [begin, end), multiplying only the entries each row holds: the CSR sum.
template <int R, int NV, int VW, class TB>
__device__ __forceinline__ void exact_rows(const PanelDevView &P, const TB *__restrict__ B,
                                           int ldb, int begin, int end, const int (&kk)[NV],
                                           const bool (&ok)[NV],
                                           typename VecT<VW>::T (&out)[R][NV]) {
  using V = VecT<VW>;
  typename V::T s[R][NV];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int v = 0; v < NV; ++v) s[r][v] = V::zero();
  for (int j = begin; j < end; ++j) {
    const int c = __ldg(P.ucol + j);
    const unsigned m = __ldg(P.umask + j);
    typename V::T b[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v)
      b[v] = ok[v] ? LdB<VW>::ld(B + (size_t)c * ldb + kk[v]) : V::zero();
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if ((m >> r) & 1u) {
        const float a = __ldg(P.uval + (size_t)j * R + r);
#pragma unroll
        for (int v = 0; v < NV; ++v) s[r][v] = V::fma(a, b[v], s[r][v]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int v = 0; v < NV; ++v) out[r][v] = s[r][v];
}

// Replace a lane's padded sums by the exact ones when they hold a NaN.
template <int R, int NV, int VW, class TB>
__device__ __forceinline__ void settle_rows(const PanelDevView &P, const TB *__restrict__ B,
                                            int ldb, int begin, int end, const int (&kk)[NV],
                                            const bool (&ok)[NV],
                                            typename VecT<VW>::T (&o)[R][NV]) {
  if constexpr (R > 1) {
    if (sums_have_nan<R, NV, VW>(o)) exact_rows<R, NV, VW, TB>(P, B, ldb, begin, end, kk, ok, o);
  }
}

// One finished value of C: written (C = A * B), or with `accumulate` added
// to what C holds (C += A * B, the contract of the reference's launcher,
// src/kernels.cu:120-167, whose caller zeroes C).
template <int VW>
__device__ __forceinline__ void put_c(bool accumulate, float *p, typename VecT<VW>::T v) {
  if (accumulate) v = VecT<VW>::add(VecT<VW>::ldcg(p), v);
  VecT<VW>::stcs(p, v);
}

template <int R, int NV, int VW>
__device__ __forceinline__ void store_rows(const PanelDevView &P, float *__restrict__ C,
                                           int ldc, int row0, const int (&kk)[NV],
                                           const bool (&ok)[NV],
                                           const typename VecT<VW>::T (&out)[R][NV]) {
  const bool accumulate = P.accumulate != 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int row = row0 + r;
    if (row < P.M) {
#pragma unroll
      for (int v = 0; v < NV; ++v)
        if (ok[v]) put_c<VW>(accumulate, C + (size_t)row * ldc + kk[v], out[r][v]);
    }
  }
}

// Write the finished vector(s) before union index `a` and start the next.
template <int R, int NV, int VW, class TB>
__device__ __forceinline__ void cross_boundaries(int a, BatchCursor &bc, Acc<R, NV, VW> &acc,
                                                 const PanelDevView &P, const TB *__restrict__ B,
                                                 int ldb, float *__restrict__ C, int ldc,
                                                 const int (&kk)[NV], const bool (&ok)[NV]) {
  while (a >= bc.ve) {
    typename VecT<VW>::T o[R][NV];
    acc.store(o);
    settle_rows<R, NV, VW, TB>(P, B, ldb, bc.vb, bc.ve, kk, ok, o);
    store_rows<R, NV, VW>(P, C, ldc, bc.v * R, kk, ok, o);
    acc.zero();
    ++bc.v;
    bc.vb = bc.ve;
    bc.ve = bc.svp[bc.v - bc.v0 + 1];
  }
}

template <int R, int NV, int VW, int UN, bool FULL, bool BATCH, class TB>
__device__ __forceinline__ void fma_group(const float *sval, int j0, int step, int n,
                                          const typename VecT<VW>::T (&b)[UN][NV],
                                          Acc<R, NV, VW> &acc, int cbase, BatchCursor &bc,
                                          const PanelDevView &P, const TB *__restrict__ B,
                                          int ldb, float *__restrict__ C, int ldc,
                                          const int (&kk)[NV], const bool (&ok)[NV]) {
#pragma unroll
  for (int q = 0; q < UN; ++q) {
    const int j = j0 + q * step;
    if (FULL || j < n) {
      if constexpr (BATCH)
        cross_boundaries<R, NV, VW, TB>(cbase + j, bc, acc, P, B, ldb, C, ldc, kk, ok);
      float a[R];
      load_vals_smem<R>(sval, j, a);
      acc.fma(a, b[q]);
    }
  }
}

// One team walks union columns [begin, end).  cg / ncg: this lane's column
// group and the number of column groups (1 for a sub-warp team); t / T: lane
// index and size of the team for staging; tmask: the team's lanes.
// Without BATCH the columns belong to one vector and its column-group sums
// are left reduced in `out`.  With BATCH (ncg = 1) they span vectors
// [bc.v0, v1): each vector's rows are written to C when its last column has
// been added, the last ones (and trailing empty vectors) at the end.
template <int R, int NV, int VW, bool BATCH, class TB = float>
__device__ __forceinline__ void walk_unit(
    const PanelDevView &P, const TB *__restrict__ B, int ldb, int begin, int end,
    const int (&kk)[NV], const bool (&ok)[NV], int cg, int ncg, int t, int T,
    unsigned tmask, int L, int chunk, int *buf_col, float *buf_val,
    typename VecT<VW>::T (&out)[R][NV], BatchCursor &bc, int v1,
    float *__restrict__ C, int ldc) {
  using V = VecT<VW>;
  using Tv = typename V::T;
  constexpr int UN = unroll_for<R, NV, VW>();
  Acc<R, NV, VW> acc;
  acc.zero();
  const TB *Bk = B + kk[0];
  const int vstride = L * VW;
  if (begin < end) {
    // prologue: stage chunk 0 into buffer 0
    int n0 = min(chunk, end - begin);
    stage_chunk<R>(P.ucol, P.uval, begin, n0, buf_col, buf_val, t, T);
    cp_async_commit();
    int cur = 0;
    for (int c0 = begin; c0 < end; c0 += chunk) {
      const int n = min(chunk, end - c0);
      const int nx = c0 + chunk < end ? min(chunk, end - c0 - chunk) : 0;
      int *ncol = buf_col + (cur ^ 1) * chunk;
      float *nval = buf_val + (size_t)(cur ^ 1) * chunk * R;
      if (nx > 0) stage_chunk<R>(P.ucol, P.uval, c0 + chunk, nx, ncol, nval, t, T);
      cp_async_commit();
      cp_async_wait_1();
      __syncwarp(tmask);
      const int *scol = buf_col + cur * chunk;
      const float *sval = buf_val + (size_t)cur * chunk * R;
      // this column group's columns: cg, cg+ncg, ...; full groups of UN of
      // them are pipelined two deep, the remainder is one guarded group
      const int mine = cg < n ? (n - cg + ncg - 1) / ncg : 0;
      const int nfull = mine / UN;
      const int gstep = UN * ncg;
      Tv b0[UN][NV], b1[UN][NV];
      int j = cg;
      if (nfull > 0)
        load_group<NV, VW, UN, true, TB>(Bk, ldb, scol, j, ncg, n, ok, vstride, b0);
      for (int g = 0; g < nfull; g += 2) {
        if (g + 1 < nfull)
          load_group<NV, VW, UN, true, TB>(Bk, ldb, scol, j + gstep, ncg, n, ok, vstride, b1);
        fma_group<R, NV, VW, UN, true, BATCH, TB>(sval, j, ncg, n, b0, acc, c0, bc, P, B, ldb,
                                                  C, ldc, kk, ok);
        if (g + 1 >= nfull) {
          j += gstep;
          break;
        }
        if (g + 2 < nfull)
          load_group<NV, VW, UN, true, TB>(Bk, ldb, scol, j + 2 * gstep, ncg, n, ok, vstride,
                                       b0);
        fma_group<R, NV, VW, UN, true, BATCH, TB>(sval, j + gstep, ncg, n, b1, acc, c0, bc, P,
                                                  B, ldb, C, ldc, kk, ok);
        j += 2 * gstep;
      }
      if (j < n) {
        load_group<NV, VW, UN, false, TB>(Bk, ldb, scol, j, ncg, n, ok, vstride, b0);
        fma_group<R, NV, VW, UN, false, BATCH, TB>(sval, j, ncg, n, b0, acc, c0, bc, P, B, ldb,
                                                   C, ldc, kk, ok);
      }
      __syncwarp(tmask);  // everyone is done with `cur` before it is refilled
      cur ^= 1;
    }
  }
  if constexpr (BATCH) {
    // the last vector (union columns [bc.vb, end)) and any empty vectors
    // after it
    while (bc.v < v1) {
      acc.store(out);
      settle_rows<R, NV, VW, TB>(P, B, ldb, bc.vb, end, kk, ok, out);
      bc.vb = end;
      store_rows<R, NV, VW>(P, C, ldc, bc.v * R, kk, ok, out);
      acc.zero();
      ++bc.v;
    }
    return;
  }
  acc.store(out);
  // sum the column groups: fixed xor tree over the lane bits above L
  for (int off = L; off < L * ncg; off <<= 1) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v) out[r][v] = V::add(out[r][v], V::shfl_xor(tmask, out[r][v], off));
  }
}

// Store a finished unit: straight to C, or (split vector) publish the part
// and let the last part reduce all parts into C.
template <int R, int NV, int VW>
__device__ __forceinline__ void finish_unit(
    const PanelDevView &P, float *__restrict__ C, int ldc, const int4 &U, int ot,
    const int (&kk)[NV], const bool (&ok)[NV], int cg, int ncg, int lead_lane,
    unsigned tmask, typename VecT<VW>::T (&acc)[R][NV]) {
  using V = VecT<VW>;
  using Tv = typename V::T;
  const int row0 = U.x * R;
  if (U.w < 0) {
    if (cg == 0) {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (row < P.M) {
#pragma unroll
          for (int v = 0; v < NV; ++v)
            if (ok[v]) put_c<VW>(P.accumulate != 0, C + (size_t)row * ldc + kk[v], acc[r][v]);
        }
      }
    }
    return;
  }
  const int slot = U.w;
  if (cg == 0) {
    float *part = P.partials + (size_t)slot * R * P.pstride;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int v = 0; v < NV; ++v)
        if (ok[v]) V::st(part + (size_t)r * P.pstride + kk[v], acc[r][v]);
  }
  __threadfence();
  __syncwarp(tmask);
  const int2 sp = __ldg(P.parts + slot);   // {split vector, part}
  const int2 svi = __ldg(P.svecs + sp.x);  // {first slot, nparts}
  int *ctr = P.counters + (size_t)sp.x * P.counter_stride + ot;
  int ticket = 0;
  if ((threadIdx.x & 31) == lead_lane) ticket = atomicAdd(ctr, 1);
  ticket = __shfl_sync(tmask, ticket, lead_lane);
  if (ticket != svi.y - 1) return;
  __threadfence();
  // last part: column group g sums parts g, g+ncg, ... with four independent
  // chains, then the groups are summed by the fixed xor tree
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      Tv s0 = V::zero(), s1 = V::zero(), s2 = V::zero(), s3 = V::zero();
      if (ok[v]) {
        const float *base = P.partials + (size_t)svi.x * R * P.pstride +
                            (size_t)r * P.pstride + kk[v];
        const size_t step = (size_t)R * P.pstride;
        int p = cg;
        for (; p + 3 * ncg < svi.y; p += 4 * ncg) {
          s0 = V::add(s0, V::ldcg(base + (size_t)p * step));
          s1 = V::add(s1, V::ldcg(base + (size_t)(p + ncg) * step));
          s2 = V::add(s2, V::ldcg(base + (size_t)(p + 2 * ncg) * step));
          s3 = V::add(s3, V::ldcg(base + (size_t)(p + 3 * ncg) * step));
        }
        for (; p < svi.y; p += ncg) s0 = V::add(s0, V::ldcg(base + (size_t)p * step));
      }
      acc[r][v] = V::add(V::add(s0, s1), V::add(s2, s3));
    }
  }
  const int L32 = 32 / ncg;  // lanes per column group
  if (ncg > 1) {
    for (int off = L32; off < 32; off <<= 1) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int v = 0; v < NV; ++v) acc[r][v] = V::add(acc[r][v], V::shfl_xor(tmask, acc[r][v], off));
    }
  }
  if (cg == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = row0 + r;
      if (row < P.M) {
#pragma unroll
        for (int v = 0; v < NV; ++v)
          if (ok[v]) put_c<VW>(P.accumulate != 0, C + (size_t)row * ldc + kk[v], acc[r][v]);
      }
    }
  }
  if ((threadIdx.x & 31) == lead_lane) *ctr = 0;  // ready for the next launch
}

constexpr int kBatchVecs = 64;  // vectors per batch at most
constexpr int kBatchVP = 68;    // staged vec_ptr entries per team (>= kBatchVecs + 1)

// Short work: one sub-warp per item.  Plans: a batch of consecutive short
// vectors (for R <= 2 the sub-warp streams through all of them and writes
// each vector's rows at its boundary; for R >= 4 a batch is one vector).
// ROWPTR (plain CSR): one row.
template <int R, int NV, int VW, bool ROWPTR, class TB>
__global__ void __launch_bounds__(256, (min_blocks_for<R, NV, VW>()))
    panel_short_kernel(const PanelDevView P, const void *__restrict__ Bv, int ldb,
                       float *__restrict__ C, int ldc, int O, int lshift, int n_otiles,
                       int W, int chunk) {
  const TB *B = static_cast<const TB *>(Bv);
  using Tv = typename VecT<VW>::T;
  constexpr bool kBatch = !ROWPTR && R <= 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int L = 1 << lshift;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = 32 >> lshift, sub = lane >> lshift, sl = lane & (L - 1);
  const unsigned submask = (L == 32) ? 0xffffffffu : (((1u << L) - 1u) << (sub * L));
  // per warp: G teams x 2 buffers x chunk columns x (1 int + R floats), then
  // G staged vec_ptr windows
  int *wcol = reinterpret_cast<int *>(smem_raw) +
              (size_t)warp * (2 * G * chunk * (R + 1) + G * kBatchVP);
  float *wval = reinterpret_cast<float *>(wcol + 2 * G * chunk);
  int *svp = reinterpret_cast<int *>(wval + (size_t)2 * G * chunk * R) + sub * kBatchVP;
  int *bcol = wcol + sub * chunk * 2;
  float *bval = wval + (size_t)sub * chunk * 2 * R;
  const int n_sub = ROWPTR ? P.n_units : P.n_batches;
  const long long per_tile = (n_sub + G - 1) / G;
  const long long n_items = per_tile * n_otiles;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp; item < n_items;
       item += nwarps) {
    const int ot = (int)(item / per_tile);
    const long long s = (item - (long long)ot * per_tile) * G + sub;
    if (s >= n_sub) continue;  // idle sub-warp
    int kk[NV];
    bool ok[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      kk[v] = ot * W + v * (L * VW) + sl * VW;
      ok[v] = kk[v] < O;
    }
    Tv acc[R][NV];
    BatchCursor bc{0, 0, 0, nullptr, 0};
    if constexpr (kBatch) {
      const int4 bt = __ldg(P.batches + s);  // {v0, v1, first column, end column}
      if (bt.y - bt.x == 1) {
        // one vector: it ends where the batch ends, no boundaries to stage
        bc = BatchCursor{bt.x, bt.w, bt.x, svp, bt.z};
      } else {
        for (int i = sl; i <= bt.y - bt.x; i += L) svp[i] = __ldg(P.vec_ptr + bt.x + i);
        __syncwarp(submask);
        bc = BatchCursor{bt.x, svp[1], bt.x, svp, bt.z};
      }
      walk_unit<R, NV, VW, true>(P, B, ldb, bt.z, bt.w, kk, ok, 0, 1, sl, L, submask, L,
                                 chunk, bcol, bval, acc, bc, bt.y, C, ldc);
      __syncwarp(submask);  // svp is rewritten by the next batch
    } else {
      int4 U;
      if constexpr (ROWPTR) {
        U = make_int4((int)s, __ldg(P.row_ptr + s), __ldg(P.row_ptr + s + 1), -1);
      } else {
        const int4 bt = __ldg(P.batches + s);  // one vector
        U = make_int4(bt.x, bt.z, bt.w, -1);
      }
      walk_unit<R, NV, VW, false>(P, B, ldb, U.y, U.z, kk, ok, 0, 1, sl, L, submask, L,
                                  chunk, bcol, bval, acc, bc, 0, C, ldc);
      settle_rows<R, NV, VW, TB>(P, B, ldb, U.y, U.z, kk, ok, acc);
      store_rows<R, NV, VW>(P, C, ldc, U.x * R, kk, ok, acc);
    }
  }
}

// Long work: a whole warp per long unit or split part, its sub-warps taking
// every G-th union column; split parts finish through the part tickets.
template <int R, int NV, int VW, class TB>
__global__ void __launch_bounds__(256, (long_min_blocks_for<R, NV, VW>()))
    panel_long_kernel(const PanelDevView P, const void *__restrict__ Bv, int ldb,
                      float *__restrict__ C, int ldc, int O, int lshift, int n_otiles,
                      int W, int chunk) {
  const TB *B = static_cast<const TB *>(Bv);
  using Tv = typename VecT<VW>::T;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int L = 1 << lshift;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = 32 >> lshift, sub = lane >> lshift, sl = lane & (L - 1);
  const int wcols = G * chunk;
  int *wcol = reinterpret_cast<int *>(smem_raw) +
              (size_t)warp * (2 * wcols * (R + 1) + G * kBatchVP);
  float *wval = reinterpret_cast<float *>(wcol + 2 * wcols);
  const long long per_tile = P.n_long;
  const long long n_items = per_tile * n_otiles;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp; item < n_items;
       item += nwarps) {
    const int ot = (int)(item / per_tile);
    const long long w = item - (long long)ot * per_tile;
    int kk[NV];
    bool ok[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      kk[v] = ot * W + v * (L * VW) + sl * VW;
      ok[v] = kk[v] < O;
    }
    Tv acc[R][NV];
    BatchCursor bc{0, 0, 0, nullptr, 0};
    const int4 U = __ldg(P.units + __ldg(P.long_idx + w));
    walk_unit<R, NV, VW, false>(P, B, ldb, U.y, U.z, kk, ok, sub, G, lane, 32, 0xffffffffu,
                                L, wcols, wcol, wval, acc, bc, 0, C, ldc);
    // every column group holds the unit's sums; group 0 stores them
    if (sub == 0) settle_rows<R, NV, VW, TB>(P, B, ldb, U.y, U.z, kk, ok, acc);
    finish_unit<R, NV, VW>(P, C, ldc, U, ot, kk, ok, sub, G, 0, 0xffffffffu, acc);
  }
}

using KernelFn = void (*)(const PanelDevView, const void *, int, float *, int, int,
                          int, int, int, int);

template <int R, int NV, int VW, class TB>
KernelFn pick_rv(bool is_long, bool rowptr) {
  if (is_long) return panel_long_kernel<R, NV, VW, TB>;
  if constexpr (R == 1) {
    if (rowptr) {
      if constexpr (std::is_same<TB, float>::value) return panel_short_kernel<1, NV, VW, true, TB>;
      return nullptr;  // the plain-CSR entry points take FP32 B only
    }
  }
  return panel_short_kernel<R, NV, VW, false, TB>;
}

template <int R, class TB>
KernelFn pick_r(int NV, int VW, bool is_long, bool rowptr) {
  if constexpr (R == 16) {
    return VW == 4 ? pick_rv<16, 1, 4, TB>(is_long, rowptr) : pick_rv<16, 1, 1, TB>(is_long, rowptr);
  } else {
    if constexpr (R == 1) {
      if (NV == 4 && VW == 4) return pick_rv<1, 4, 4, TB>(is_long, rowptr);
    }
    if (NV == 1)
      return VW == 4 ? pick_rv<R, 1, 4, TB>(is_long, rowptr) : pick_rv<R, 1, 1, TB>(is_long, rowptr);
    return VW == 4 ? pick_rv<R, 2, 4, TB>(is_long, rowptr) : pick_rv<R, 2, 1, TB>(is_long, rowptr);
  }
}

template <class TB>
KernelFn select_kernel_t(int R, int NV, int VW, bool is_long, bool rowptr) {
  switch (R) {
    case 1: return pick_r<1, TB>(NV, VW, is_long, rowptr);
    case 2: return pick_r<2, TB>(NV, VW, is_long, rowptr);
    case 4: return pick_r<4, TB>(NV, VW, is_long, rowptr);
    case 8: return pick_r<8, TB>(NV, VW, is_long, rowptr);
    case 16: return pick_r<16, TB>(NV, VW, is_long, rowptr);
  }
  return nullptr;
}

KernelFn select_kernel(int R, int NV, int VW, bool is_long, bool rowptr, BType bt) {
  switch (bt) {
    case BType::kBF16: return select_kernel_t<__nv_bfloat16>(R, NV, VW, is_long, rowptr);
    case BType::kF16: return select_kernel_t<__half>(R, NV, VW, is_long, rowptr);
    default: return select_kernel_t<float>(R, NV, VW, is_long, rowptr);
  }
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

// The vector-panel kernels' shape: pick_shape's, except that single-row
// vectors at O >= 256 take sub-warps of 16 lanes with four 128-bit columns
// per lane (twice the B loads in flight per lane; same 256-column tiles).
// Measured on B200 against 32 lanes x two columns: power-law O=256 403 ->
// 350 us, uniform O=256 14.5 -> 12.5 us, R-MAT 2^22 O=256 within the run to
// run spread (6.4-6.7 ms either way).
static LaunchShape panel_shape(int O, int R, bool vec4) {
  LaunchShape s = pick_shape(O, R, vec4);
  if (R == 1 && s.VW == 4 && (int)ceil_div(O, 4) >= 64) {
    s.lshift = 4;
    s.NV = 4;
    s.W = 16 * 4 * 4;
    s.n_otiles = (int)ceil_div(O, s.W);
  }
  return s;
}

// Columns staged per sub-warp per buffer: about 10 KB of shared memory per
// warp for both buffers, between 4 and 128 columns (a multiple of 4).
int stage_chunk_cols(int R, int G) {
  int c = 10240 / (2 * G * (R + 1) * 4);
  c = c < 4 ? 4 : (c > 128 ? 128 : c);
  return c & ~3;
}

namespace {

// Resident CTAs per SM of (kernel, dynamic shared memory, device), asked of
// the runtime once: the query (and the shared-memory attribute) cost host time
// that a small launch would otherwise wait for on the GPU.
vcsr_status resident_per_sm(const void *fn, int threads, size_t smem, int *per_sm) {
  struct Key {
    const void *fn;
    size_t smem;
    int dev;
  };
  static std::vector<std::pair<Key, int>> cache;
  static std::mutex mu;
  int dev = 0;
  VCSR_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  for (const auto &e : cache)
    if (e.first.fn == fn && e.first.smem == smem && e.first.dev == dev) {
      *per_sm = e.second;
      return VCSR_OK;
    }
  // the kernel's dynamic shared-memory limit is raised once, to the device's
  // opt-in maximum (it only bounds what a launch may ask for), so that no
  // launch ever lowers it under the size of another
  bool raised = false;
  for (const auto &e : cache) raised = raised || (e.first.fn == fn && e.first.dev == dev);
  if (!raised) {
    int optin = 0;
    VCSR_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    VCSR_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, optin));
  }
  int n = 0;
  VCSR_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, threads, smem));
  if (n <= 0) n = 1;
  cache.push_back({Key{fn, smem, dev}, n});
  *per_sm = n;
  return VCSR_OK;
}

vcsr_status launch_one(KernelFn fn, const PanelDevView &P, long long team_items, int G,
                       const LaunchShape &s, int chunk, size_t smem, const void *B, int ldb,
                       float *C, int ldc, int O, cudaStream_t st, int reserve_sms) {
  const int threads = 256;
  int per_sm = 0;
  VCSR_TRY(resident_per_sm(reinterpret_cast<const void *>(fn), threads, smem, &per_sm));
  const long long items = team_items * s.n_otiles;
  long long blocks = (items + (threads / 32) - 1) / (threads / 32);
  const long long cap = (long long)std::max(1, sm_count() - reserve_sms) * per_sm;
  blocks = blocks > cap ? cap : (blocks < 1 ? 1 : blocks);
  fn<<<(int)blocks, threads, smem, st>>>(P, B, ldb, C, ldc, O, s.lshift, s.n_otiles, s.W,
                                         chunk);
  VCSR_CUDA(cudaGetLastError());
  return VCSR_OK;
}

}  // namespace

vcsr_status launch_panel_spmm(const PanelDevView &P, bool rowptr, const void *B, int ldb,
                              float *C, int ldc, int O, cudaStream_t st, int *launches,
                              cudaStream_t side, cudaEvent_t fork, cudaEvent_t join,
                              BType bt, int reserve_sms) {
  if (launches) *launches = 0;
  const int n_short = rowptr ? P.n_units : P.n_batches;
  const int n_long = rowptr ? 0 : P.n_long;
  if (O <= 0 || n_short + n_long <= 0) return VCSR_OK;
  // 128-bit lanes: four B values per load (16 bytes FP32, 8 bytes BF16 / FP16)
  const bool vec4 = (O % 4 == 0) && (ldb % 4 == 0) && (ldc % 4 == 0) &&
                    ((uintptr_t)B % (bt == BType::kF32 ? 16 : 8) == 0) && ((uintptr_t)C % 16 == 0);
  if ((long long)ldb * (bt == BType::kF32 ? 4 : 2) > 0x7fffffffLL)
    return fail(VCSR_ERR_INVALID, "ldb=%d: B rows of 2^31 bytes or more are not supported", ldb);
  const LaunchShape s = panel_shape(O, P.R, vec4);
  if (!rowptr && P.n_split_units > 0 && (O > P.pstride || s.n_otiles > P.counter_stride))
    return fail(VCSR_ERR_INVALID, "O=%d exceeds the plan's max_O=%d", O, P.pstride);
  const int G = 32 >> s.lshift;
  const int chunk = stage_chunk_cols(P.R, G);
  const size_t smem = (size_t)8 * (2 * G * chunk * (P.R + 1) + G * kBatchVP) * 4;
  const bool both = n_short > 0 && n_long > 0 && side != nullptr;
  if (both) {  // the long units run beside the short ones on the plan's side stream
    VCSR_CUDA(cudaEventRecord(fork, st));
    VCSR_CUDA(cudaStreamWaitEvent(side, fork, 0));
  }
  int n = 0;
  if (n_long > 0) {
    KernelFn fl = select_kernel(P.R, s.NV, s.VW, true, false, bt);
    if (!fl) return fail(VCSR_ERR_UNSUPPORTED, "no kernel for R=%d", P.R);
    VCSR_TRY(launch_one(fl, P, n_long, G, s, chunk, smem, B, ldb, C, ldc, O,
                        both ? side : st, reserve_sms));
    ++n;
  }
  if (n_short > 0) {
    KernelFn fs = select_kernel(P.R, s.NV, s.VW, false, rowptr, bt);
    if (!fs) return fail(VCSR_ERR_UNSUPPORTED, "no kernel for R=%d", P.R);
    VCSR_TRY(launch_one(fs, P, (n_short + G - 1) / G, G, s, chunk, smem, B, ldb, C, ldc, O,
                        st, reserve_sms));
    ++n;
  }
  if (both) {
    VCSR_CUDA(cudaEventRecord(join, side));
    VCSR_CUDA(cudaStreamWaitEvent(st, join, 0));
  }
  if (launches) *launches = n;
  return VCSR_OK;
}

}  // namespace vcsr

extern "C" vcsr_status vcsr_csr_spmm(int M, const int *d_row_ptr, const int *d_col,
                                     const float *d_val, const float *dB, int O,
                                     float *dC, vcsr_stream_t stream) {
  vcsr::clear_error();
  if (M < 0 || O < 0) return vcsr::fail(VCSR_ERR_INVALID, "negative size");
  if (M == 0 || O == 0) return VCSR_OK;
  if (!d_row_ptr || !dB || !dC) return vcsr::fail(VCSR_ERR_INVALID, "null device pointer");
  vcsr::PanelDevView P{};
  P.row_ptr = d_row_ptr;
  P.ucol = d_col;
  P.uval = d_val;
  P.n_units = M;
  P.M = M;
  P.R = 1;
  return vcsr::launch_panel_spmm(P, true, dB, O, dC, O, O, (cudaStream_t)stream, nullptr,
                                 nullptr, nullptr, nullptr);
}

// ------------------------------------------------- allocation-free CSR SpMM
//
// vcsr_csr_spmm_noalloc is the CSR row-wise SpMM above with long rows split
// over several warps, for callers that may not allocate device memory.  The
// split needs scratch (which rows are long, their part bookkeeping, the
// partial sums and the last-part tickets); here it lives in one file-scope
// __device__ array instead of memory the library would allocate.  Nothing in
// the reference corresponds to it.
namespace vcsr {
namespace noalloc {

constexpr int kMaxO = VCSR_NOALLOC_MAX_O;
constexpr int kMaxLong = VCSR_NOALLOC_MAX_LONG_ROWS;
constexpr int kMaxParts = VCSR_NOALLOC_MAX_PARTS;
constexpr int kSplit = VCSR_NOALLOC_SPLIT;
constexpr size_t round256(size_t x) { return (x + 255) & ~(size_t)255; }
// ctrl[0] long rows found, ctrl[1] error bits, ctrl[2] parts reserved
constexpr size_t kCtrl = 0;
constexpr size_t kLong = 256;                                    // int[kMaxLong]
constexpr size_t kSvec = round256(kLong + 4 * (size_t)kMaxLong);   // int2[kMaxLong]
constexpr size_t kParts = round256(kSvec + 8 * (size_t)kMaxLong);  // int2[kMaxParts]
constexpr size_t kTickets = round256(kParts + 8 * (size_t)kMaxParts);  // int[kMaxLong*kMaxO]
constexpr size_t kPartials =
    round256(kTickets + 4 * (size_t)kMaxLong * kMaxO);           // float[kMaxParts*kMaxO]
constexpr size_t kBytes = kPartials + 4 * (size_t)kMaxParts * kMaxO;
static_assert(kBytes == VCSR_NOALLOC_SCRATCH_BYTES, "header and layout disagree");

}  // namespace noalloc
}  // namespace vcsr

// The scratch.  In host code this name is only a handle for the runtime;
// kernels get its device address from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[vcsr::noalloc::kBytes];

namespace vcsr {
namespace {

// Rows longer than kSplit entries get a slot, a range of part slots and
// their {slot, part} records, and the slot's n_otiles tickets are zeroed;
// overflow sets an error bit and skips the row.  Every part record below
// min(parts reserved, kMaxParts) is written by this pass (-1 where a row did
// not fit), so nothing of an earlier call is read.
__global__ void noalloc_classify_kernel(const int *__restrict__ rp, int M, int n_otiles,
                                        unsigned char *S) {
  using namespace noalloc;
  int *ctrl = reinterpret_cast<int *>(S + kCtrl);
  int *lr = reinterpret_cast<int *>(S + kLong);
  int2 *sv = reinterpret_cast<int2 *>(S + kSvec);
  int2 *parts = reinterpret_cast<int2 *>(S + kParts);
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < M; r += gridDim.x * blockDim.x) {
    const int len = rp[r + 1] - rp[r];
    if (len <= kSplit) continue;
    const int np = (len + kSplit - 1) / kSplit;
    const int s = atomicAdd(&ctrl[0], 1);
    if (s >= kMaxLong) {
      atomicOr(&ctrl[1], 1);
      continue;
    }
    const int base = atomicAdd(&ctrl[2], np);
    if (base + np > kMaxParts) {
      atomicOr(&ctrl[1], 2);
      lr[s] = -1;
      for (int p = base; p < kMaxParts; ++p) parts[p] = make_int2(-1, -1);
      continue;
    }
    lr[s] = r;
    sv[s] = make_int2(base, np);
    for (int p = 0; p < np; ++p) parts[base + p] = make_int2(s, p);
    int *tk = reinterpret_cast<int *>(S + kTickets) + (size_t)s * n_otiles;
    for (int t = 0; t < n_otiles; ++t) tk[t] = 0;
  }
}

// Short rows: one sub-warp per row, exactly as vcsr_csr_spmm.  Long rows:
// one warp per (part, O-tile); the parts are added by the last one to finish.
template <int NV, int VW>
__global__ void __launch_bounds__(256, (min_blocks_for<1, NV, VW>()))
    noalloc_spmm_kernel(const int *__restrict__ rp, const int *__restrict__ col,
                        const float *__restrict__ val, int M,
                        const float *__restrict__ B, int ldb, float *__restrict__ C,
                        int ldc, int O, int lshift, int n_otiles, int W, int chunk,
                        unsigned char *S) {
  using namespace noalloc;
  using Tv = typename VecT<VW>::T;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int *ctrl = reinterpret_cast<const int *>(S + kCtrl);
  const int *lr = reinterpret_cast<const int *>(S + kLong);
  PanelDevView P{};
  P.ucol = col;
  P.uval = val;
  P.M = M;
  P.R = 1;
  P.parts = reinterpret_cast<const int2 *>(S + kParts);
  P.svecs = reinterpret_cast<const int2 *>(S + kSvec);
  P.partials = reinterpret_cast<float *>(S + kPartials);
  P.counters = reinterpret_cast<int *>(S + kTickets);
  P.pstride = O;
  P.counter_stride = n_otiles;
  const int L = 1 << lshift;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = 32 >> lshift, sub = lane >> lshift, sl = lane & (L - 1);
  const unsigned submask = (L == 32) ? 0xffffffffu : (((1u << L) - 1u) << (sub * L));
  const int wcols = G * chunk;
  int *wcol = reinterpret_cast<int *>(smem_raw) + (size_t)warp * 2 * wcols * 2;
  float *wval = reinterpret_cast<float *>(wcol + 2 * wcols);
  const int n_parts = min(ctrl[2], kMaxParts);
  const long long n_sg = (M + G - 1) / G;
  const long long per_tile = n_parts + n_sg;
  const long long n_items = per_tile * n_otiles;
  const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long item = (long long)blockIdx.x * (blockDim.x >> 5) + warp; item < n_items;
       item += nwarps) {
    const int ot = (int)(item / per_tile);
    const long long w = item - (long long)ot * per_tile;
    int4 U;
    int cg, ncg, t, T, lead, chk;
    unsigned tmask;
    int *bcol;
    float *bval;
    if (w < n_parts) {  // one part of a long row, whole warp
      const int2 sp = P.parts[w];
      const int r = sp.x >= 0 ? lr[sp.x] : -1;
      if (r < 0) continue;
      const int b = rp[r] + sp.y * kSplit;
      U = make_int4(r, b, min(b + kSplit, rp[r + 1]), (int)w);
      cg = sub; ncg = G; t = lane; T = 32; tmask = 0xffffffffu; lead = 0;
      bcol = wcol; bval = wval; chk = wcols;
    } else {
      const long long r = (w - n_parts) * G + sub;
      if (r >= M) {
        U = make_int4(0, 0, 0, -2);
      } else {
        const int b = rp[r], e = rp[r + 1];
        U = (e - b > kSplit) ? make_int4(0, 0, 0, -2) : make_int4((int)r, b, e, -1);
      }
      cg = 0; ncg = 1; t = sl; T = L; tmask = submask; lead = sub * L;
      bcol = wcol + sub * chunk * 2;
      bval = wval + (size_t)sub * chunk * 2;
      chk = chunk;
    }
    if (U.w == -2) continue;
    int kk[NV];
    bool ok[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      kk[v] = ot * W + v * (L * VW) + sl * VW;
      ok[v] = kk[v] < O;
    }
    Tv acc[1][NV];
    BatchCursor bc{0, 0, 0, nullptr, 0};
    walk_unit<1, NV, VW, false>(P, B, ldb, U.y, U.z, kk, ok, cg, ncg, t, T, tmask, L, chk,
                                bcol, bval, acc, bc, 0, C, ldc);
    finish_unit<1, NV, VW>(P, C, ldc, U, ot, kk, ok, cg, ncg, lead, tmask, acc);
  }
}

std::mutex g_noalloc_mu;
unsigned char *g_noalloc_ptr[64] = {};

// Device address of the scratch on the current device (set up once per
// device, with that device current).
vcsr_status noalloc_scratch(unsigned char **out) {
  int dev = 0;
  VCSR_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(VCSR_ERR_UNSUPPORTED, "device ordinal %d >= 64", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void *p = nullptr;
    VCSR_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = static_cast<unsigned char *>(p);
  }
  *out = g_noalloc_ptr[dev];
  return VCSR_OK;
}

}  // namespace
}  // namespace vcsr

extern "C" vcsr_status vcsr_csr_spmm_noalloc(int M, const int *d_row_ptr,
                                             const int *d_col, const float *d_val,
                                             const float *dB, int O, float *dC,
                                             vcsr_stream_t stream) {
  using namespace vcsr;
  using namespace vcsr::noalloc;
  clear_error();
  if (M < 0 || O < 0) return fail(VCSR_ERR_INVALID, "negative size");
  if (O > kMaxO)
    return fail(VCSR_ERR_RANGE, "O = %d exceeds the allocation-free limit of %d columns",
                O, kMaxO);
  if (M == 0 || O == 0) return VCSR_OK;
  if (!d_row_ptr || !dB || !dC) return fail(VCSR_ERR_INVALID, "null device pointer");
  unsigned char *S = nullptr;
  VCSR_TRY(noalloc_scratch(&S));
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec4 = (O % 4 == 0) && ((uintptr_t)dB % 16 == 0) && ((uintptr_t)dC % 16 == 0);
  const LaunchShape s = pick_shape(O, 1, vec4);
  // the three counters start at zero; the classify pass writes every part
  // record and zeroes every ticket the product will use
  VCSR_CUDA(cudaMemsetAsync(S + kCtrl, 0, 256, st));
  const int sms = sm_count();
  noalloc_classify_kernel<<<sms * 4, 256, 0, st>>>(d_row_ptr, M, s.n_otiles, S);
  VCSR_CUDA(cudaGetLastError());
  using Fn = void (*)(const int *, const int *, const float *, int, const float *, int,
                      float *, int, int, int, int, int, int, unsigned char *);
  Fn fn = s.VW == 4 ? (s.NV == 1 ? (Fn)noalloc_spmm_kernel<1, 4> : (Fn)noalloc_spmm_kernel<2, 4>)
                    : (s.NV == 1 ? (Fn)noalloc_spmm_kernel<1, 1> : (Fn)noalloc_spmm_kernel<2, 1>);
  const int threads = 256, G = 32 >> s.lshift;
  const int chunk = stage_chunk_cols(1, G);
  const size_t smem = (size_t)(threads / 32) * 2 * G * chunk * 2 * 4;
  int per_sm = 0;  // asked of the runtime once per (kernel, shared memory, device)
  VCSR_TRY(resident_per_sm(reinterpret_cast<const void *>(fn), threads, smem, &per_sm));
  const long long items = ((long long)kMaxParts + (M + G - 1) / G) * s.n_otiles;
  long long blocks = (items + (threads / 32) - 1) / (threads / 32);
  const long long cap = (long long)sms * (per_sm > 0 ? per_sm : 1);
  blocks = blocks > cap ? cap : (blocks < 1 ? 1 : blocks);
  fn<<<(int)blocks, threads, smem, st>>>(d_row_ptr, d_col, d_val, M, dB, O, dC, O, O,
                                         s.lshift, s.n_otiles, s.W, chunk, S);
  VCSR_CUDA(cudaGetLastError());
  int err = 0;
  VCSR_CUDA(cudaMemcpyAsync(&err, S + kCtrl + 4, sizeof(int), cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  if (err & 1)
    return fail(VCSR_ERR_RANGE,
                "more than %d rows longer than %d entries: exceeds the allocation-free "
                "scratch (C is incomplete)", kMaxLong, kSplit);
  if (err & 2)
    return fail(VCSR_ERR_RANGE,
                "long rows need more than %d parts of %d entries: exceeds the "
                "allocation-free scratch (C is incomplete)", kMaxParts, kSplit);
  return VCSR_OK;
}
