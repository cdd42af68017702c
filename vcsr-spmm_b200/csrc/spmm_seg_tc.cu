// spmm_seg_tc.cu — the tensor-core segment kernel: FP32-accurate SpMM on
// tcgen05 for matrices whose rows come in column runs (sm_100a).
//
// The reference's VCSR cuts A into column segments and stages each
// segment's B rows as a tile in shared memory (src/kernels.cu:37-103,
// segw x tileK).  Here a plan built with VCSR_PLAN_TC_SEGMENTS takes 16 rows
// at a time (a row block) and cuts the union of their columns into runs of
// consecutive columns ("segments"); each run becomes pieces of at most 32
// B rows (a multiple of 8), and the row block's values in a piece's columns
// are a dense 16 x L tile (zeros where a row has no entry).  Per row block and
// 128-column slice of O the kernel computes, in tensor memory,
//     D[128 x 16] = sum over pieces  B[c0 .. c0+L, slice]^T  x  A_piece^T
// with tcgen05.mma kind::tf32 (M = 128 = the O slice, N = 16 = the rows,
// K = 8 per instruction), and writes D to C (or adds it, when short runs
// left a residual that the FP32 kernel wrote first).
//
// FP32 accuracy from TF32 products: every value x (of B and of A) is split
// into hi = x with its 13 low mantissa bits cleared (exactly a TF32 value)
// and lo = x - hi (exact), and each K step issues three MMAs,
// hi_B*hi_A + lo_B*hi_A + hi_B*lo_A, accumulated in FP32; the dropped lo*lo
// term is below 2^-22 of the product.  The split runs in shared memory
// between the copy and the MMAs (converter warps), so B and A are read from
// memory once, as stored.
//
// B tiles come by TMA: per piece one box of L rows x 32 floats x 4 chunks
// (a 3-D view of B when O is a multiple of 32, else four 2-D boxes) in the
// 128-byte swizzle with 32-byte atoms that the MN-major TF32 operand needs;
// rows past N read as zeros.  The A tile is one bulk copy.  Roles (320
// threads): warps 0-3 read the accumulator (warp w owns TMEM lanes 32w..) and
// write C; warp 4 allocates TMEM and its lane 0 issues the copies into a
// ring of stages; lane 0 of warp 5 issues the MMAs; warps 6-9 split the
// values.  Barriers per stage: full (copies landed), conv (split done), empty
// (MMAs done); two accumulators alternate between items.  Every wait is
// bounded: after ~2^22 polls the kernel records where it gave up and stops,
// waiting (bounded) for the copies and MMAs it issued before it frees TMEM.
//
// Outputs the split product leaves non-finite (a padding zero or the lo part
// of an Inf or NaN of B) are recomputed by the epilogue thread over the
// row's CSR entries in CSR order, so C equals the CSR sum's value there
// (src/kernels.cu:27-31), Inf and NaN included.
#include <cuda.h>
#include <cuda_runtime.h>

#include "common.h"
#include "seg_tc.h"
#include "spmm_tc.h"
#include "tcgen05.cuh"

namespace vcsr {
namespace {

using namespace tc;

#ifndef VCSR_SEG_STAGES
#define VCSR_SEG_STAGES 3
#endif
#ifndef VCSR_SEG_CTAS
#define VCSR_SEG_CTAS 2
#endif
constexpr int kSegStages = VCSR_SEG_STAGES;
constexpr int kSegCtas = VCSR_SEG_CTAS;  // resident CTAs per SM (shared memory)
constexpr int kGroupBytes = 8 * 128 * 4;                 // 8 rows x 128 floats: one K step of B
constexpr int kPieceB = kSegPieceRows / 8 * kGroupBytes;  // 16 KB
constexpr int kPieceA = kSegPieceRows * 16 * 4;           // 2 KB
constexpr int kSegStageBytes = 2 * kPieceB + 2 * kPieceA;  // hi and lo of both
constexpr int kSegThreads = 320;
constexpr int kSegProducer = 4, kSegMma = 5, kSegConv0 = 6;
constexpr int kSegConvThreads = 128;
constexpr uint32_t kSegTmemCols = 32;  // two 16-column accumulators
constexpr int kWaitConv = 6;
constexpr uint32_t kHiMask = 0xFFFFE000u;  // sign, exponent and 10 mantissa bits

__device__ __forceinline__ void split4(float4 &x, float4 &lo) {
  const float hx = __uint_as_float(__float_as_uint(x.x) & kHiMask);
  const float hy = __uint_as_float(__float_as_uint(x.y) & kHiMask);
  const float hz = __uint_as_float(__float_as_uint(x.z) & kHiMask);
  const float hw = __uint_as_float(__float_as_uint(x.w) & kHiMask);
  lo = make_float4(x.x - hx, x.y - hy, x.z - hz, x.w - hw);
  x = make_float4(hx, hy, hz, hw);
}

// B's tensor maps, one per piece height L = 8, 16, 24, 32: a piece's B rows
// come in with one copy (3-D view: box {32, L, 4}; 2-D view: four boxes
// {32, L}), chunk-major, chunk c at c * L * 128 bytes.
struct SegMaps {
  CUtensorMap m[kSegPieceRows / 8];
};

__global__ void __launch_bounds__(kSegThreads, kSegCtas)
    seg_tc_kernel(const SegView V, const __grid_constant__ SegMaps maps) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char *base = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  unsigned char *stage = base;
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + kSegStages * kSegStageBytes);
  uint64_t *full = bars, *conv = bars + kSegStages, *empty = bars + 2 * kSegStages;
  uint64_t *dfull = bars + 3 * kSegStages;      // accumulator b ready (count 1)
  uint64_t *dfree = bars + 3 * kSegStages + 2;  // accumulator b read (count 128)
  uint64_t *drain = bars + 3 * kSegStages + 4;  // all MMAs of this CTA done
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 3 * kSegStages + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  // pieces whose copies the converters waited for (the rest are drained)
  volatile long long *seen = reinterpret_cast<volatile long long *>(bars + 3 * kSegStages + 6);
  // per stage, written by the producer before the stage's copies: the
  // piece's rows L | 256 (first piece of an item) | 512 (last piece of an
  // item), or -1 when the CTA has no more pieces.  Converters and the MMA
  // thread read it from here instead of loading piece records themselves.
  volatile int *meta = reinterpret_cast<volatile int *>(bars + 3 * kSegStages + 7);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSegStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(conv + s, kSegConvThreads);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(dfull + b, 1);
      mbar_init(dfree + b, 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *seen = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kSegProducer) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kSegTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const int n_items = V.n_rb * V.n_ochunks;
  long long g_load = 0;  // producer: pieces issued

  if (warp == kSegProducer) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      // piece records and item bounds are loaded one step ahead of use
      bool ok = true;
      int t = blockIdx.x;
      int q0 = 0, q1 = 0;
      if (t < n_items) {
        const int rbi = t % V.n_rb;
        q0 = V.pp[rbi];
        q1 = V.pp[rbi + 1];
      }
      while (t < n_items && ok && !*abort_flag) {
        const int oc = t / V.n_rb;
        const int tn = t + gridDim.x;
        int nq0 = 0, nq1 = 0;
        if (tn < n_items) {
          const int rbn = tn % V.n_rb;
          nq0 = V.pp[rbn];
          nq1 = V.pp[rbn + 1];
        }
        int4 pc = V.pieces[q0];  // {c0, L, koff}
        for (int q = q0; q < q1; ++q) {
          const int4 pn = q + 1 < q1 ? V.pieces[q + 1] : make_int4(0, 0, 0, 0);
          const int s = (int)(g_load % kSegStages);
          const long long ph = g_load / kSegStages;
          if (ph > 0 && !mbar_wait(empty + s, (uint32_t)((ph - 1) & 1), abort_flag, kWaitEmpty)) {
            ok = false;
            break;
          }
          meta[s] = pc.y | (q == q0 ? 256 : 0) | (q == q1 - 1 ? 512 : 0);
          unsigned char *st = stage + (size_t)s * kSegStageBytes;
          const CUtensorMap *tm = &maps.m[(pc.y >> 3) - 1];
          mbar_add_tx(full + s, (uint32_t)(pc.y * 512 + pc.y * 64));
          if (V.slab3d) {
            tma_load_3d(st, tm, 0, pc.x, oc * 4, full + s);
          } else {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_2d(st + c * pc.y * 128, tm, oc * 128 + 32 * c, pc.x, full + s);
          }
          bulk_load(st + 2 * kPieceB, V.a + (size_t)pc.z * 16, (uint32_t)(pc.y * 64), full + s);
          mbar_arrive(full + s);
          ++g_load;
          pc = pn;
        }
        t = tn;
        q0 = nq0;
        q1 = nq1;
      }
      if (ok && !*abort_flag) {  // the end mark, through a stage of its own
        const int s = (int)(g_load % kSegStages);
        const long long ph = g_load / kSegStages;
        if (ph == 0 || mbar_wait(empty + s, (uint32_t)((ph - 1) & 1), abort_flag, kWaitEmpty)) {
          meta[s] = -1;
          mbar_arrive(full + s);
          ++g_load;
        }
      }
    }
  } else if (warp >= kSegConv0) {
    // ------------------------------------------------ hi / lo split
    const int ct = threadIdx.x - kSegConv0 * 32;
    for (long long g = 0;; ++g) {
      const int s = (int)(g % kSegStages);
      if (!mbar_wait(full + s, (uint32_t)((g / kSegStages) & 1), abort_flag, kWaitFull)) break;
      if (ct == 0) *seen = g + 1;
      const int mt = meta[s];
      if (mt >= 0) {
        const int L = mt & 255;
        unsigned char *st = stage + (size_t)s * kSegStageBytes;
        float4 *bh = reinterpret_cast<float4 *>(st);
        float4 *bl = reinterpret_cast<float4 *>(st + kPieceB);
        float4 *ah = reinterpret_cast<float4 *>(st + 2 * kPieceB);
        float4 *al = reinterpret_cast<float4 *>(st + 2 * kPieceB + kPieceA);
        for (int i = ct; i < L * 32; i += kSegConvThreads) {  // L x 128 floats of B
          float4 x = bh[i], lo;
          split4(x, lo);
          bh[i] = x;
          bl[i] = lo;
        }
        for (int i = ct; i < L * 4; i += kSegConvThreads) {  // L x 16 values of A
          float4 x = ah[i], lo;
          split4(x, lo);
          ah[i] = x;
          al[i] = lo;
        }
        // the tensor core reads through the async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      }
      mbar_arrive(conv + s);  // the end mark is passed on too
      if (mt < 0) break;
    }
  } else if (warp == kSegMma) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issue
      int lt = -1, buf = 0;
      uint32_t dt = tmem;
      bool first = true;
      for (long long g = 0;; ++g) {
        const int s = (int)(g % kSegStages);
        if (!mbar_wait(conv + s, (uint32_t)((g / kSegStages) & 1), abort_flag, kWaitConv)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const int mt = meta[s];
        if (mt < 0) break;
        if (mt & 256) {  // first piece of an item: the next accumulator
          ++lt;
          buf = lt & 1;
          if (lt >= 2 && !mbar_wait(dfree + buf, (uint32_t)(((lt - 2) >> 1) & 1), abort_flag,
                                    kWaitAccFree))
            break;
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          dt = tmem + (uint32_t)(buf * 16);
          first = true;
        }
        const int L = mt & 255;
        const uint32_t bh = smem_u32(stage + (size_t)s * kSegStageBytes);
        const uint32_t bl = bh + kPieceB, ah = bh + 2 * kPieceB, al = ah + kPieceA;
        for (int h = 0; h < (L >> 3); ++h) {
          // B: 32-float chunks L * 128 bytes apart, this K step's rows at
          // h * 1024, 4-row swizzle atoms 512 apart; A: core matrices 128
          // bytes apart along N, 256 along K
          const uint64_t bdh = smem_desc(bh + h * 1024, L * 128, 512, 1);
          const uint64_t bdl = smem_desc(bl + h * 1024, L * 128, 512, 1);
          const uint64_t adh = smem_desc(ah + h * 512, 256, 128, 0);
          const uint64_t adl = smem_desc(al + h * 512, 256, 128, 0);
          mma_tf32(dt, bdh, adh, first ? 0u : 1u);
          first = false;
          mma_tf32(dt, bdl, adh, 1u);
          mma_tf32(dt, bdh, adl, 1u);
        }
        mma_commit(empty + s);
        if (mt & 512) mma_commit(dfull + buf);  // the item's accumulator is complete
      }
      // every MMA issued by this thread has finished before TMEM is freed
      mma_commit(drain);
      volatile int no_abort = 0;
      if (!mbar_wait(drain, 0, &no_abort, kWaitDrain)) *abort_flag = kWaitDrain;
    }
  } else {
    // -------------------------------------------------------- epilogue
    int lt = 0;
    for (int t = blockIdx.x; t < n_items; t += gridDim.x, ++lt) {
      const int oc = t / V.n_rb, rbi = t - oc * V.n_rb;
      const int buf = lt & 1;
      const int row0 = V.rb_row[rbi];  // loaded while the MMAs run
      if (!mbar_wait(dfull + buf, (uint32_t)((lt >> 1) & 1), abort_flag, kWaitAccFull)) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t r[16];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * 16);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
          "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
          : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
            "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
            "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
          : "r"(taddr));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(dfree + buf);
      const int m = oc * 128 + warp * 32 + lane;  // column of C
      if (m < V.O) {
        const int nrow = min(16, V.M - row0);
        float *c = V.C + (size_t)row0 * V.ldc + m;
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          if (n >= nrow) break;
          const float v = __uint_as_float(r[n]);
          float *cp = c + (size_t)n * V.ldc;
          if (!isfinite(v)) {  // the CSR sum, in CSR order
            const int row = row0 + n;
            float s = 0.f;
            for (int p = V.rp[row]; p < V.rp[row + 1]; ++p)
              s = fmaf(V.val[p], V.B[(size_t)V.col[p] * V.ldb + m], s);
            *cp = s;
          } else {
            *cp = V.accumulate ? *cp + v : v;
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kSegProducer && lane == 0 && *abort_flag) {
    // copies issued but never waited for must land before the CTA exits
    for (long long g = *seen; g < g_load; ++g) {
      volatile int no_abort = 0;
      if (!mbar_wait(full + (int)(g % kSegStages), (uint32_t)((g / kSegStages) & 1), &no_abort,
                     kWaitFull))
        break;
    }
  }
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(V.err, 0, *abort_flag | (int)(blockIdx.x << 4));
  __syncwarp();
  if (warp == kSegProducer) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kSegTmemCols));
  }
}

}  // namespace

size_t seg_smem_bytes() { return (size_t)kSegStages * kSegStageBytes + 1024 + 256; }
static_assert(8 * (3 * kSegStages + 7) + 4 * kSegStages <= 256, "barrier area");

vcsr_status launch_seg_tc(const SegView &V0, const float *B, int N, int ldb, float *C, int ldc,
                          int O, cudaStream_t st, int *launches) {
  if (launches) *launches = 0;
  if (V0.n_rb == 0 || O == 0) return VCSR_OK;
  if (O % 4 || ldb % 4 || ((uintptr_t)B % 16) || ((uintptr_t)C % 4))
    return fail(VCSR_ERR_UNSUPPORTED,
                "tensor-core segments need O and ldb multiples of 4 and a 16-byte aligned B");
  EncodeTiledFn enc;
  VCSR_TRY(tensor_map_encoder(&enc));
  SegMaps maps;
  // O a multiple of 32: the 3-D view {32 floats, N rows, O/32 chunks} (strides
  // ldb*4 and 128 bytes) with {32, L, 4} boxes lands a piece's four chunks
  // with one copy; chunks past O/32 read as zeros.  Otherwise the 2-D view
  // {O, N} with 32 x L boxes zero-fills past O.
  const bool slab3d = (O % 32) == 0;
  const cuuint32_t estr[3] = {1, 1, 1};
  for (int k = 0; k < kSegPieceRows / 8; ++k) {
    const cuuint32_t L = (cuuint32_t)(8 * (k + 1));
    CUresult r;
    if (slab3d) {
      const cuuint64_t dims[3] = {32, (cuuint64_t)N, (cuuint64_t)(O / 32)};
      const cuuint64_t strides[2] = {(cuuint64_t)ldb * 4, 128};
      const cuuint32_t box[3] = {32, L, 4};
      r = enc(&maps.m[k], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)B, dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
      const cuuint64_t dims[2] = {(cuuint64_t)O, (cuuint64_t)N};
      const cuuint64_t strides[1] = {(cuuint64_t)ldb * 4};
      const cuuint32_t box[2] = {32, L};
      r = enc(&maps.m[k], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)B, dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS)
      return fail(VCSR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  }
  SegView V = V0;
  V.slab3d = slab3d ? 1 : 0;
  V.O = O;
  V.N = N;
  V.ldb = ldb;
  V.ldc = ldc;
  V.B = B;
  V.C = C;
  V.n_ochunks = (int)ceil_div(O, 128);
  const size_t smem = seg_smem_bytes();
  VCSR_CUDA(cudaFuncSetAttribute(seg_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
  int dev = 0, sms = 148;
  VCSR_CUDA(cudaGetDevice(&dev));
  VCSR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const long long items = (long long)V.n_rb * V.n_ochunks;
  long long grid = (long long)sms * kSegCtas;  // resident CTAs (shared memory)
  if (grid > items) grid = items;
  seg_tc_kernel<<<(int)grid, kSegThreads, smem, st>>>(V, maps);
  VCSR_CUDA(cudaGetLastError());
  if (launches) *launches = 1;
  return VCSR_OK;
}

}  // namespace vcsr
