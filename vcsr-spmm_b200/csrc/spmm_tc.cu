// spmm_tc.cu — tcgen05 TF32 SpMM on dense 16x16 panels of A (sm_100a).
//
// A plan built with VCSR_PLAN_TF32_PANELS keeps every 16x16 block of A (rows
// 16i.., columns 16j..) holding at least `panel_min_nnz` entries as a dense
// TF32 tile; the other entries stay in the FP32 row-stationary layout and
// are computed first (C written).  This kernel then adds the panels' product:
// for one row block i and one 128-column slice of O,
//     D[128 x 16] = sum over the row block's dense blocks j of
//                   B[16j .. 16j+15, slice]^T (128 x 16)  x  A_ij^T (16 x 16)
// in tensor memory, i.e. tcgen05.mma kind::tf32 with M = 128 (the O slice),
// N = 16 (the block's rows), K = 16 (two K = 8 instructions).  Operand A is B
// as stored (row-major, O contiguous): MN-major, loaded by 2-D TMA boxes of
// 16 rows x 32 floats.  An MN-major TF32 operand has one shared-memory
// layout, the 128-byte swizzle with 32-byte atoms (descriptor layout 1, TMA
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B): the four 32-byte chunks of each
// 128-byte row are exchanged by row % 4, so a swizzle atom is 4 rows (512
// bytes) of K; with the plain 128-byte swizzle the MMA reads TF32 operands as
// zeros.  Operand B is the dense block, pre-packed by the plan in the K-major
// core-matrix order (8 rows x 16 bytes per core matrix, no swizzle) and
// fetched with one 1-KB bulk copy.  This is the reference's tensor-core idea
// (src/vcsr_tc.cu:122-195: one FP16 WMMA per depth step, 16x16 groups,
// atomics into C) rebuilt with TF32 inputs, FP32 accumulation in TMEM, no
// atomics, and the O dimension on the tensor core's M side.
//
// Roles (192 threads): warps 0-3 read the accumulator (warp w owns TMEM lanes
// 32w..32w+31) and add it into C; warp 4 allocates TMEM and its lane 0 issues
// the copies into a ring of stages of kG blocks each (`full`/`empty`
// mbarriers); lane 0 of warp 5 issues the MMAs.  The producer runs up to
// kStages * kG blocks ahead of the MMAs.  Measured on B200 the copy issue
// rate of the SM's TMA unit (about 46 cycles per 2-KB box) bounds this
// kernel; grouping blocks per stage saves barrier round trips, and when O is
// a multiple of 32 a 3-D view of B (32 floats, rows, 32-float chunks) brings
// a slab's four boxes in with one copy that lands them at the same swizzled
// addresses.  Two
// accumulators alternate between items so the epilogue of item t runs while
// the MMAs of item t+1 are issued.  Every mbarrier wait is bounded: after
// ~2^22 polls the kernel records which wait gave up and stops; before it
// frees its TMEM and exits it still waits (bounded) for its issued MMAs and
// for the copies it issued but did not consume.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "common.h"
#include "spmm_tc.h"
#include "tcgen05.cuh"

namespace vcsr {
namespace {

using namespace tc;

#ifndef VCSR_TC_BLOCKS_PER_STAGE
#define VCSR_TC_BLOCKS_PER_STAGE 4
#endif
#ifndef VCSR_TC_STAGES
#define VCSR_TC_STAGES 2
#endif
// A stage holds kG dense blocks with their B slabs: one full/empty round
// trip (copies landing, MMA issue, MMA completion) per kG blocks.
constexpr int kG = VCSR_TC_BLOCKS_PER_STAGE;
constexpr int kStages = VCSR_TC_STAGES;
constexpr int kBTileBytes = 16 * 128 * 4;  // 16 rows x 128 floats, 4 swizzled boxes
constexpr int kABlockBytes = 16 * 16 * 4;  // one dense block
constexpr int kBlockBytes = kBTileBytes + kABlockBytes;
constexpr int kStageBytes = kG * kBlockBytes;  // slabs first, then the blocks
constexpr int kThreads = 192;
constexpr int kProducerWarp = 4, kMmaWarp = 5;
constexpr uint32_t kTmemCols = 32;  // two 16-column accumulators
__global__ void __launch_bounds__(kThreads, 1)
    tc_panel_kernel(const TcView V, const __grid_constant__ CUtensorMap tmB) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 1024-byte aligned stage ring (each K = 8 step starts on a 1-KB boundary)
  unsigned char *base = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  unsigned char *stage = base;
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + kStages * kStageBytes);
  uint64_t *full = bars, *empty = bars + kStages;
  uint64_t *dfull = bars + 2 * kStages;      // accumulator b ready (count 1)
  uint64_t *dfree = bars + 2 * kStages + 2;  // accumulator b read (count 128)
  uint64_t *drain = bars + 2 * kStages + 4;  // all MMAs of this CTA done
  uint32_t *tmem_holder = reinterpret_cast<uint32_t *>(bars + 2 * kStages + 5);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_holder + 1);
  long long *consumed = reinterpret_cast<long long *>(bars + 2 * kStages + 6);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(dfull + b, 1);
      mbar_init(dfree + b, 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kProducerWarp) {  // one warp allocates the accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_holder;
  const int n_items = V.n_rb * V.n_ochunks;
  long long g_load = 0;  // producer: blocks issued

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      // block g goes to slot g % kG of stage (g / kG) % kStages; each block
      // adds its bytes to the stage's transaction count and the last block
      // of a stage (or of this CTA's work) arrives on it
      for (int t = blockIdx.x; t < n_items && !*abort_flag; t += gridDim.x) {
        const int oc = t / V.n_rb, rbi = t - oc * V.n_rb;
        const int b0 = V.rb_ptr[rbi], b1 = V.rb_ptr[rbi + 1];
        bool ok = true;
        for (int bi = b0; bi < b1; ++bi) {
          const int u = (int)(g_load % kG);
          const long long sidx = g_load / kG;
          const int s = (int)(sidx % kStages);
          if (u == 0 && sidx >= kStages &&
              !mbar_wait(empty + s, (uint32_t)(((sidx / kStages) - 1) & 1), abort_flag,
                         kWaitEmpty)) {
            ok = false;
            break;
          }
          unsigned char *st = stage + s * kStageBytes;
          const int j = V.blk_col[bi];
          // the values of a run of blocks that stays in this item and this
          // stage are contiguous on both sides: one bulk copy at its start,
          // its bytes expected before it is issued
          const int run = (u == 0 || bi == b0) ? min(kG - u, b1 - bi) : 0;
          mbar_add_tx(full + s, (uint32_t)(kBTileBytes + run * kABlockBytes));
          if (run > 0)
            bulk_load(st + kG * kBTileBytes + u * kABlockBytes, V.blk_val + (size_t)bi * 256,
                      (uint32_t)(run * kABlockBytes), full + s);
          if (V.slab3d) {
            tma_load_3d(st + u * kBTileBytes, &tmB, 0, 16 * j, oc * 4, full + s);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              tma_load_2d(st + u * kBTileBytes + q * 2048, &tmB, oc * 128 + 32 * q, 16 * j,
                          full + s);
          }
          ++g_load;
          if (u == kG - 1) mbar_arrive(full + s);
        }
        if (!ok) break;
      }
      if (g_load % kG) mbar_arrive(full + (int)((g_load / kG) % kStages));  // partial stage
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issue
      long long g = 0;
      int lt = 0;  // local item count
      for (int t = blockIdx.x; t < n_items && !*abort_flag; t += gridDim.x, ++lt) {
        const int rbi = t % V.n_rb;  // items run over row blocks within each slice
        const int nblk = V.rb_ptr[rbi + 1] - V.rb_ptr[rbi];
        const int buf = lt & 1;
        if (lt >= 2 && !mbar_wait(dfree + buf, (uint32_t)(((lt - 2) >> 1) & 1), abort_flag,
                                  kWaitAccFree))
          break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t dt = tmem + (uint32_t)(buf * 16);
        bool ok = true;
        for (int b = 0; b < nblk; ++b) {
          const int u = (int)(g % kG);
          const long long sidx = g / kG;
          const int s = (int)(sidx % kStages);
          if (u == 0) {
            if (!mbar_wait(full + s, (uint32_t)((sidx / kStages) & 1), abort_flag, kWaitFull)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          }
          const uint32_t a_addr = smem_u32(stage + s * kStageBytes + u * kBTileBytes);
          const uint32_t b_addr =
              smem_u32(stage + s * kStageBytes + kG * kBTileBytes + u * kABlockBytes);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // A: MN atoms (32 floats) 2048 bytes apart (one TMA box each),
            // K atoms (4 rows) 512 bytes apart; this K = 8 step starts at row 8h
            const uint64_t ad = smem_desc(a_addr + h * 1024, 2048, 512, 1);
            // B: core matrices 128 bytes apart along N, 256 along K
            const uint64_t bd = smem_desc(b_addr + h * 512, 256, 128, 0);
            mma_tf32(dt, ad, bd, (b > 0 || h > 0) ? 1u : 0u);
          }
          ++g;
          if (u == kG - 1) mma_commit(empty + s);
        }
        if (!ok) break;
        // the plan lists only row blocks with dense blocks; a test may
        // withhold block 0's first accumulator-ready signal (TcView::inject)
        if (!(V.inject && blockIdx.x == 0 && lt == 0)) mma_commit(dfull + buf);
      }
      *consumed = (g + kG - 1) / kG;  // stages whose copies were waited for
      // every MMA issued by this thread has finished before TMEM is freed
      mma_commit(drain);
      volatile int no_abort = 0;  // wait even when another role gave up
      if (!mbar_wait(drain, 0, &no_abort, kWaitDrain)) *abort_flag = kWaitDrain;
    }
  } else {
    // -------------------------------------------------------- epilogue
    int lt = 0;
    for (int t = blockIdx.x; t < n_items; t += gridDim.x, ++lt) {
      const int oc = t / V.n_rb, rbi = t - oc * V.n_rb;
      const int buf = lt & 1;
      const long long lim = (V.inject && blockIdx.x == 0 && lt == 0) ? kTestPollLimit : kPollLimit;
      if (!mbar_wait(dfull + buf, (uint32_t)((lt >> 1) & 1), abort_flag, kWaitAccFull, lim))
        break;
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
      const int row0 = V.rb_row[rbi];
      if (m < V.O) {
        float *c = V.C + (size_t)row0 * V.ldc + m;
        const int nrow = min(16, V.M - row0);
        float cv[16];
#pragma unroll
        for (int n = 0; n < 16; ++n)
          if (n < nrow) cv[n] = c[(size_t)n * V.ldc];
#pragma unroll
        for (int n = 0; n < 16; ++n)
          if (n < nrow) c[(size_t)n * V.ldc] = cv[n] + __uint_as_float(r[n]);
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == kProducerWarp && lane == 0 && *abort_flag) {
    // copies issued but never consumed must land before the CTA exits
    for (long long g = *consumed; g < (g_load + kG - 1) / kG; ++g) {
      volatile int no_abort = 0;
      if (!mbar_wait(full + (int)(g % kStages), (uint32_t)((g / kStages) & 1), &no_abort,
                     kWaitFull))
        break;
    }
  }
  if (threadIdx.x == 0 && *abort_flag) atomicCAS(V.err, 0, *abort_flag | (int)(blockIdx.x << 4));
  __syncwarp();
  if (warp == kProducerWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

}  // namespace

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
vcsr_status tensor_map_encoder(EncodeTiledFn *out) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    VCSR_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p)
      return fail(VCSR_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return VCSR_OK;
}

size_t tc_smem_bytes() { return (size_t)kStages * kStageBytes + 1024 + 256; }

void describe_tc_error(int word, char *buf, size_t n) {
  static const char *const site[] = {"?",          "stage-full",       "stage-empty",
                                     "accumulator-full", "accumulator-free", "MMA-drain",
                                     "stage-converted"};
  const int w = word & 15;
  snprintf(buf, n, "tensor-core kernel: bounded wait on the %s barrier ran out (block %d)",
           site[(w >= 1 && w <= 6) ? w : 0], word >> 4);
}

vcsr_status launch_tc_panels(const TcView &V0, const float *B, int N, int ldb, float *C,
                             int ldc, int O, cudaStream_t st, int *launches) {
  if (launches) *launches = 0;
  if (V0.n_rb == 0 || O == 0) return VCSR_OK;
  if (O % 4 || ldb % 4 || ((uintptr_t)B % 16) || ((uintptr_t)C % 4))
    return fail(VCSR_ERR_UNSUPPORTED,
                "TF32 panels need O and ldb multiples of 4 and a 16-byte aligned B");
  EncodeTiledFn enc;
  VCSR_TRY(tensor_map_encoder(&enc));
  CUtensorMap tm;
  // With O a multiple of 32 the 3-D view {32 floats, N rows, O/32 chunks}
  // (strides ldb*4 and 128 bytes) covers exactly B's N x O values: every
  // in-range coordinate addresses inside B, and chunks past O/32 (a partial
  // last 128-column slice) read as zeros.  Otherwise the 2-D view {O, N}
  // with boxes of 32 x 16 zero-fills past O.
  const bool slab3d = (O % 32) == 0;
  CUresult r;
  const cuuint32_t estr[3] = {1, 1, 1};
  if (slab3d) {
    const cuuint64_t dims[3] = {32, (cuuint64_t)N, (cuuint64_t)(O / 32)};
    const cuuint64_t strides[2] = {(cuuint64_t)ldb * 4, 128};
    const cuuint32_t box[3] = {32, 16, 4};
    r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, (void *)B, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t dims[2] = {(cuuint64_t)O, (cuuint64_t)N};
    const cuuint64_t strides[1] = {(cuuint64_t)ldb * 4};
    const cuuint32_t box[2] = {32, 16};
    r = enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)B, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return fail(VCSR_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  TcView V = V0;
  V.slab3d = slab3d ? 1 : 0;
  V.O = O;
  V.ldc = ldc;
  V.C = C;
  V.n_ochunks = (int)ceil_div(O, 128);
  const size_t smem = tc_smem_bytes();
  VCSR_CUDA(cudaFuncSetAttribute(tc_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
  int dev = 0, sms = 148, per_sm = 1;
  VCSR_CUDA(cudaGetDevice(&dev));
  VCSR_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  // resident CTAs per SM from shared memory (each also holds kTmemCols of
  // the SM's 512 TMEM columns)
  int smem_sm = 0, smem_reserved = 0;
  VCSR_CUDA(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
  VCSR_CUDA(cudaDeviceGetAttribute(&smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev));
  per_sm = (int)(smem_sm / (smem + (size_t)smem_reserved));
  if (per_sm < 1) per_sm = 1;
  if (per_sm > (int)(512 / kTmemCols)) per_sm = (int)(512 / kTmemCols);
  const long long items = (long long)V.n_rb * V.n_ochunks;
  long long grid = (long long)sms * per_sm;
  if (grid > items) grid = items;
  tc_panel_kernel<<<(int)grid, kThreads, smem, st>>>(V, tm);
  VCSR_CUDA(cudaGetLastError());
  if (launches) *launches = 1;
  return VCSR_OK;
}

}  // namespace vcsr
