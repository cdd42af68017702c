// A caller written against the reference's host interface (include/mmio.hpp,
// include/csr.hpp, include/vcsr.hpp and the launchers of src/kernels.cu),
// built against include/vcsr_spmm.hpp and the engine library.  Fills B as
// src/main.cpp:108 does, runs run_csr_spmm_gpu (the ground truth),
// run_vcsr_spmm_gpu twice (C += A*B: the second call doubles C) and
// run_vcsr_spmm_segmented_gpu, and prints one line of relative L2 errors and
// the timed milliseconds.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "vcsr_spmm.hpp"

static double rel_l2(const std::vector<float> &a, const std::vector<float> &b, double scale) {
  double num = 0, den = 0;
  for (size_t i = 0; i < a.size(); ++i) {
    const double d = a[i] - scale * b[i];
    num += d * d;
    den += scale * scale * (double)b[i] * b[i];
  }
  return den > 0 ? std::sqrt(num / den) : std::sqrt(num);
}

int main(int argc, char **argv) {
  if (argc < 3) {
    std::fprintf(stderr, "usage: drop_in file.mtx O\n");
    return 2;
  }
  const int O = std::atoi(argv[2]);
  COO coo = read_matrix_market_coo(argv[1]);
  CSR csr = coo_to_csr(coo);
  VCSRSpMM V = csr_to_vcsr_spmm(csr, 4, 32);
  std::vector<float> B((size_t)csr.N * O);
  for (size_t i = 0; i < B.size(); ++i) B[i] = (float)((int)(i % 13) - 6) / 7.0f;
  int *d_rp, *d_col;
  float *d_val, *dB, *dC;
  cudaMalloc(&d_rp, sizeof(int) * (csr.M + 1));
  cudaMalloc(&d_col, sizeof(int) * (csr.nnz > 0 ? csr.nnz : 1));
  cudaMalloc(&d_val, sizeof(float) * (csr.nnz > 0 ? csr.nnz : 1));
  cudaMalloc(&dB, sizeof(float) * (B.size() > 0 ? B.size() : 1));
  cudaMalloc(&dC, sizeof(float) * (size_t)csr.M * O);
  cudaMemcpy(d_rp, csr.row_ptr.data(), sizeof(int) * (csr.M + 1), cudaMemcpyHostToDevice);
  cudaMemcpy(d_col, csr.col.data(), sizeof(int) * csr.nnz, cudaMemcpyHostToDevice);
  cudaMemcpy(d_val, csr.val.data(), sizeof(float) * csr.nnz, cudaMemcpyHostToDevice);
  cudaMemcpy(dB, B.data(), sizeof(float) * B.size(), cudaMemcpyHostToDevice);
  cudaStream_t st;
  cudaStreamCreate(&st);
  const size_t bytesC = sizeof(float) * (size_t)csr.M * O;
  std::vector<float> ref((size_t)csr.M * O), c1(ref.size()), c2(ref.size()), c3(ref.size());
  float ms_csr = 0, ms_engine = 0, ms_seg = 0;
  cudaMemset(dC, 0, bytesC);
  run_csr_spmm_gpu(csr.M, d_rp, d_col, d_val, dB, O, dC, st, ms_csr);
  cudaMemcpy(ref.data(), dC, bytesC, cudaMemcpyDeviceToHost);
  cudaMemset(dC, 0, bytesC);
  run_vcsr_spmm_gpu(V, dB, O, 64, dC, st, ms_engine);
  cudaMemcpy(c1.data(), dC, bytesC, cudaMemcpyDeviceToHost);
  run_vcsr_spmm_gpu(V, dB, O, 64, dC, st, ms_engine);
  cudaMemcpy(c2.data(), dC, bytesC, cudaMemcpyDeviceToHost);
  cudaMemset(dC, 0, bytesC);
  run_vcsr_spmm_segmented_gpu(V, dB, O, 64, dC, st, ms_seg);
  cudaMemcpy(c3.data(), dC, bytesC, cudaMemcpyDeviceToHost);
  std::printf("engine %.3e twice %.3e segmented %.3e ms %.4f %.4f %.4f\n",
              rel_l2(c1, ref, 1.0), rel_l2(c2, ref, 2.0), rel_l2(c3, ref, 1.0), ms_csr,
              ms_engine, ms_seg);
  cudaStreamDestroy(st);
  cudaFree(d_rp); cudaFree(d_col); cudaFree(d_val); cudaFree(dB); cudaFree(dC);
  return 0;
}
