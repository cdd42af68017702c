// spmm_segmented.cu — SpMM straight on the segment-major VCSR, race-free.
//
// Same contract as run_vcsr_spmm_gpu (src/kernels.cu:120): C += A*B with
// ld = O.  The reference kernel (src/kernels.cu:37-103) adds every product
// into global C without atomics, so groups of different segments that share
// a row race; it also reads B rows past N-1 when N % segw != 0.  Here a warp
// takes one (group, 32-column slice): the lanes stage the segment's B rows
// (rows >= N read as zero) in shared memory, each lane keeps one group row's
// 32 sums in registers over the group's depth, and the sums are transposed
// through shared memory so that each atomic add instruction covers 32
// consecutive columns of one C row.  The result is exact up to the order of
// the floating-point additions across groups.
#include <cuda_runtime.h>

#include "common.h"

using vcsr::fail;

namespace {

constexpr int kWarps = 4;

__global__ void __launch_bounds__(kWarps * 32)
    segmented_kernel(int G, const int *__restrict__ group_ptr,
                     const int *__restrict__ group_depth,
                     const int *__restrict__ group_seg_base,
                     const int *__restrict__ group_rows,
                     const int *__restrict__ lcol, const float *__restrict__ aval,
                     int bundle, int segw, int N, const float *__restrict__ B,
                     int O, float *__restrict__ C) {
  extern __shared__ float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float *SB = smem + warp * (segw + 32) * 33;  // segw x 33 B tile
  float *T = SB + segw * 33;                   // 32 x 33 transpose tile
  const int chunks = (O + 31) / 32;
  const long long pairs = (long long)G * chunks;
  for (long long it = (long long)blockIdx.x * kWarps + warp; it < pairs;
       it += (long long)gridDim.x * kWarps) {
    const int g = (int)(it / chunks);
    const int k0 = (int)(it - (long long)g * chunks) * 32;
    const int base = group_ptr[g], depth = group_depth[g];
    const int sb = group_seg_base[g];
    __syncwarp();
    for (int r = 0; r < segw; ++r) {
      const int brow = sb + r, k = k0 + lane;
      SB[r * 33 + lane] = (brow < N && k < O) ? B[(size_t)brow * O + k] : 0.f;
    }
    __syncwarp();
    for (int l0 = 0; l0 < bundle; l0 += 32) {
      const int l = l0 + lane;
      float acc[32];
#pragma unroll
      for (int kk = 0; kk < 32; ++kk) acc[kk] = 0.f;
      int row = -1;
      if (l < bundle) {
        row = group_rows[(size_t)g * bundle + l];
        for (int d = 0; d < depth; ++d) {
          const size_t slot = (size_t)base + (size_t)d * bundle + l;
          const int lc = lcol[slot];
          if (lc >= 0 && lc < segw) {
            const float a = aval[slot];
#pragma unroll
            for (int kk = 0; kk < 32; ++kk) acc[kk] = fmaf(a, SB[lc * 33 + kk], acc[kk]);
          }
        }
      }
#pragma unroll
      for (int kk = 0; kk < 32; ++kk) T[lane * 33 + kk] = acc[kk];
      __syncwarp();
      const int nl = min(32, bundle - l0);
      for (int q = 0; q < nl; ++q) {
        const int rq = __shfl_sync(0xffffffffu, row, q);
        const int k = k0 + lane;
        if (rq >= 0 && k < O) atomicAdd(C + (size_t)rq * O + k, T[q * 33 + lane]);
      }
      __syncwarp();
    }
  }
}

}  // namespace

extern "C" vcsr_status vcsr_spmm_segmented(const vcsr_vcsr *v, const float *dB,
                                           int O, int tileK, float *dC,
                                           vcsr_stream_t stream) {
  vcsr::clear_error();
  if (!v) return fail(VCSR_ERR_INVALID, "null VCSR");
  if (O < 0 || tileK <= 0) return fail(VCSR_ERR_INVALID, "need O >= 0, tileK > 0");
  if (v->num_groups == 0 || O == 0) return VCSR_OK;
  if (!dB || !dC) return fail(VCSR_ERR_INVALID, "null B or C");
  const size_t smem = sizeof(float) * kWarps * (size_t)(v->segw + 32) * 33;
  int dev = 0, optin = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if ((int64_t)smem > optin)
    return fail(VCSR_ERR_UNSUPPORTED, "segw=%d needs %zu B of shared memory", v->segw,
                smem);
  VCSR_CUDA(cudaFuncSetAttribute(segmented_kernel,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem));
  const long long pairs = (long long)v->num_groups * ((O + 31) / 32);
  long long blocks = (pairs + kWarps - 1) / kWarps;
  if (blocks > (long long)sms * 16) blocks = (long long)sms * 16;
  segmented_kernel<<<(int)blocks, kWarps * 32, smem, (cudaStream_t)stream>>>(
      v->num_groups, v->group_ptr, v->group_depth, v->group_seg_base, v->group_rows,
      v->lcol, v->val, v->bundle, v->segw, v->N, dB, O, dC);
  VCSR_CUDA(cudaGetLastError());
  return VCSR_OK;
}
