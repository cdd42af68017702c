// ref_gpu_shim.cu — C entry points over the reference's own GPU launchers,
// compiled for sm_100a from the reference tree, where its sources lie, by
// baseline/Makefile into baseline/_ref/libref_gpu.so.  Nothing is copied.
//
// BENCHMARK PEERS ONLY: bench.py times these kernels beside the engine on the
// same B200 ("the reference rebuilt for sm_100a").  They are never the
// product path and never an oracle (the VCSR kernels race on C or use
// atomics).  Each launcher times its own kernel with CUDA events, as the
// reference's harness does (src/main.cpp:119-163).
//   run_csr_spmm_gpu       src/kernels.cu:107   (csr_spmm_kernel)
//   run_vcsr_spmm_gpu      src/kernels.cu:120   (vcsr_spmm_kernel; uploads the
//                                               format on every call, untimed)
//   run_vcsr_opt_spmm_gpu  src/vcsr_opt.cu:243  (vcsr_opt_kernel)
//   run_vcsr_seg_spmm_gpu  src/vcsr_seg.cu:191  (vcsr_seg_prefetch_kernel)
//   run_aspt_spmm_gpu      src/aspt.cu:153      (aspt_spmm_kernel)
// Inputs the kernels need to stay in bounds, which the caller provides (read
// from the kernels' sources): B with at least ceil(N/segw)*segw rows (the
// segment kernels read whole segments), tileK <= 64 (vcsr_seg keeps 64
// accumulators per thread), O a multiple of 64 and col/val arrays holding 32
// entries past nnz for ASpT (its long-row loop loads 32 entries at a time).
#include "kernels.cu"
#include "vcsr_opt.cu"
#include "vcsr_seg.cu"
#include "aspt.cu"

namespace {

// One VCSR format (the reference's packing, include/vcsr.hpp:12-23) held in
// the three structs the launchers take.
struct Variants {
  VCSRSpMM base;
  VCSROpt opt;
  VCSRSeg seg;
};

template <class T>
void fill(T &v, int M, int N, int segw, int bundle, int G, const int *gp, const int *gd,
          const int *gs, const int *gr, long long P, const int *lc, const float *val) {
  v.M = M;
  v.N = N;
  v.segw = segw;
  v.bundle = bundle;
  v.group_ptr.assign(gp, gp + G + 1);
  v.group_depth.assign(gd, gd + G);
  v.group_seg_base.assign(gs, gs + G);
  v.group_rows.assign(gr, gr + (size_t)G * bundle);
  v.lcol.assign(lc, lc + P);
  v.val.assign(val, val + P);
}

}  // namespace

extern "C" {

int ref_gpu_csr(int M, const int *rp, const int *col, const float *val, const float *dB, int O,
                float *dC, void *stream, float *ms) {
  float t = 0.f;
  run_csr_spmm_gpu(M, rp, col, val, dB, O, dC, (cudaStream_t)stream, t);
  *ms = t;
  return (int)cudaGetLastError();
}

int ref_gpu_aspt(int M, const int *rp, const int *col, const float *val, const float *dB, int O,
                 float *dC, void *stream, float *ms) {
  if (O % 64) return -1;  // the launcher would exit(1)
  float t = 0.f;
  run_aspt_spmm_gpu(M, rp, col, val, dB, O, dC, (CUstream)stream, t);
  *ms = t;
  return (int)cudaGetLastError();
}

void *ref_vcsr_create(int M, int N, int segw, int bundle, int G, const int *gp, const int *gd,
                      const int *gs, const int *gr, long long P, const int *lc,
                      const float *val) {
  Variants *v = new Variants();
  fill(v->base, M, N, segw, bundle, G, gp, gd, gs, gr, P, lc, val);
  fill(v->opt, M, N, segw, bundle, G, gp, gd, gs, gr, P, lc, val);
  fill(v->seg, M, N, segw, bundle, G, gp, gd, gs, gr, P, lc, val);
  v->opt.num_segments = v->seg.num_segments = (N + segw - 1) / segw;
  return v;
}

// which: 0 vcsr_spmm_kernel, 1 vcsr_opt_kernel, 2 vcsr_seg_prefetch_kernel
int ref_vcsr_run(void *h, int which, const float *dB, int O, int tileK, float *dC,
                 void *stream, float *ms) {
  Variants *v = static_cast<Variants *>(h);
  if (tileK < 1 || tileK > 64) return -1;
  float t = 0.f;
  cudaStream_t st = (cudaStream_t)stream;
  if (which == 0) run_vcsr_spmm_gpu(v->base, dB, O, tileK, dC, st, t);
  else if (which == 1) run_vcsr_opt_spmm_gpu(v->opt, dB, O, tileK, dC, st, t);
  else if (which == 2) run_vcsr_seg_spmm_gpu(v->seg, dB, O, tileK, dC, st, t, true);
  else return -1;
  *ms = t;
  return (int)cudaGetLastError();
}

// Frees the launchers' file-static device copies (vcsr_opt, vcsr_seg) and the
// host structs.
void ref_vcsr_destroy(void *h, void *stream) {
  destroy_vcsr_opt_device((cudaStream_t)stream);
  destroy_vcsr_seg_device((cudaStream_t)stream);
  delete static_cast<Variants *>(h);
}

}  // extern "C"
