// cli.cpp — spmm_vcsr, the command-line driver with the reference's flags
// (src/main.cpp:73-168): --mtx --O --segw --bundle --tileK --repeat --algo,
// the same table and GFLOP/s = 2*nnz*O/t (src/main.cpp:111), and one
// "Name: <ms> ms <gflops> GFLOP/s [params]" line per kernel in the format the
// reference's bench scripts parse (reports/h100/*_vcsr_*.txt,
// run_h100_bench.slurm:60-61).  Extra flags: --gen <config> [--size S]
// [--seed s] for synthetic matrices, --gpus N for row panels on N GPUs,
// --check for a relative-L2 comparison against cuSPARSE.
//
// Algorithms: cusparse (vendor), csr (row-wise CSR kernel), aspt (the
// engine at one row per vector: a sub-warp per short row, a whole warp with
// xor-shuffle sums per long row and long rows split over several warps --
// the warp-per-row scheme of src/aspt.cu:38-142 without its O % 64 limit),
// vcsr (the row-stationary engine), vcsr_seg / vcsr_baseline (race-free
// kernel on the segment-major VCSRSpMM built on the GPU), vcsr_tc (dense
// 16x16 blocks in TF32), vcsr_tcseg (column runs on the tensor cores at FP32
// accuracy), fast / fastspmm (the row-window condensation of
// src/fastspmm.cu:129-253 -- 16-row windows, the window's distinct columns
// condensed, a dense 16-value tile per condensed column -- which is the
// engine's vector panel at 16 rows per vector, computed in FP32), all.
// vcsr_naive is reported as not provided.
#include <cuda_runtime.h>
#include <getopt.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "vcsr_spmm.h"
#include "vcsr_spmm.hpp"

namespace {

void usage() {
  printf("Usage: spmm_vcsr (--mtx file.mtx | --gen uniform|fem|powerlaw|rmat|blockdense)"
         " --O 128 [options]\n");
  printf("Options: --segw w --bundle b --tileK t --repeat r --algo a --size s --seed s"
         " --gpus n --check --mtx-banner\n");
  printf("Algorithms: cusparse, csr, aspt, vcsr, vcsr_seg, vcsr_baseline, vcsr_tc, vcsr_tcseg,"
         " fast, all\n");
}

#define CK(x)                                                              \
  do {                                                                     \
    cudaError_t e_ = (x);                                                  \
    if (e_ != cudaSuccess) {                                               \
      fprintf(stderr, "CUDA error %s:%d: %s\n", __FILE__, __LINE__,        \
              cudaGetErrorString(e_));                                     \
      std::exit(1);                                                        \
    }                                                                      \
  } while (0)

#define VK(x)                                                              \
  do {                                                                     \
    vcsr_status s_ = (x);                                                  \
    if (s_ != VCSR_OK) {                                                   \
      fprintf(stderr, "error: %s (%s)\n", vcsr_last_error(),               \
              vcsr_status_string(s_));                                     \
      std::exit(2);                                                        \
    }                                                                      \
  } while (0)

struct Timer {
  cudaEvent_t a, b;
  Timer() { cudaEventCreate(&a); cudaEventCreate(&b); }
  ~Timer() { cudaEventDestroy(a); cudaEventDestroy(b); }
};

double rel_l2(const std::vector<float> &x, const std::vector<float> &r) {
  double num = 0, den = 0;
  for (size_t i = 0; i < x.size(); ++i) {
    double d = (double)x[i] - r[i];
    num += d * d;
    den += (double)r[i] * r[i];
  }
  return den > 0 ? std::sqrt(num / den) : std::sqrt(num);
}

}  // namespace

int main(int argc, char **argv) {
  std::string mtx, gen, algo = "all";
  bool mtx_banner = false;  // follow the %%MatrixMarket banner (symmetric expansion)
  int O = 128, segw = 16, bundle = 32, tileK = 64, repeat = 10, size = 0, gpus = 1;
  unsigned long long seed = 0;
  bool check = false;
  static struct option opts[] = {
      {"mtx", required_argument, 0, 'm'},   {"O", required_argument, 0, 'o'},
      {"segw", required_argument, 0, 's'},  {"bundle", required_argument, 0, 'b'},
      {"tileK", required_argument, 0, 't'}, {"repeat", required_argument, 0, 'r'},
      {"algo", required_argument, 0, 'a'},  {"gen", required_argument, 0, 'g'},
      {"size", required_argument, 0, 'z'},  {"seed", required_argument, 0, 'e'},
      {"gpus", required_argument, 0, 'n'},  {"check", no_argument, 0, 'c'},
      {"help", no_argument, 0, 'h'},        {"mtx-banner", no_argument, 0, 'x'},
      {0, 0, 0, 0}};
  int c, idx;
  while ((c = getopt_long(argc, argv, "", opts, &idx)) != -1) {
    switch (c) {
      case 'm': mtx = optarg; break;
      case 'x': mtx_banner = true; break;
      case 'o': O = atoi(optarg); break;
      case 's': segw = atoi(optarg); break;
      case 'b': bundle = atoi(optarg); break;
      case 't': tileK = atoi(optarg); break;
      case 'r': repeat = atoi(optarg); break;
      case 'a': algo = optarg; break;
      case 'g': gen = optarg; break;
      case 'z': size = atoi(optarg); break;
      case 'e': seed = strtoull(optarg, nullptr, 10); break;
      case 'n': gpus = atoi(optarg); break;
      case 'c': check = true; break;
      default: usage(); return 1;
    }
  }
  if (mtx.empty() == gen.empty() || O <= 0 || repeat <= 0 || segw <= 0 ||
      bundle <= 0 || tileK <= 0 || gpus <= 0) {
    usage();
    return 1;
  }
  printf("=== VCSR-SpMM Benchmark (B200, sm_100a) ===\n");
  CSR csr;
  try {
    if (!mtx.empty()) {
      printf("Loading: %s\n", mtx.c_str());
      COO coo = read_matrix_market_coo(mtx, mtx_banner);
      csr = coo_to_csr(coo);
    } else {
      printf("Generating: %s (size %d, seed %llu)\n", gen.c_str(), size, seed);
      vcsr_csr g{};
      VK(vcsr_gen_csr(gen.c_str(), seed, size, &g));
      csr.M = g.M; csr.N = g.N; csr.nnz = g.nnz;
      csr.row_ptr.assign(g.row_ptr, g.row_ptr + g.M + 1);
      csr.col.assign(g.col, g.col + g.nnz);
      csr.val.assign(g.val, g.val + g.nnz);
      vcsr_csr_free(&g, VCSR_HOST);
    }
  } catch (const std::exception &e) {
    fprintf(stderr, "error: %s\n", e.what());
    return 2;
  }
  printf("Matrix: %d x %d, nnz=%d\n", csr.M, csr.N, csr.nnz);
  printf("Params: O=%d, segw=%d, bundle=%d, tileK=%d, gpus=%d\n\n", O, segw, bundle,
         tileK, gpus);
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (gpus > ndev) {
    fprintf(stderr, "error: --gpus %d but %d devices visible\n", gpus, ndev);
    return 2;
  }

  const size_t nB = (size_t)csr.N * O, nC = (size_t)csr.M * O;
  std::vector<float> hB(nB);
  for (size_t i = 0; i < nB; ++i) hB[i] = (float)((int)(i % 13) - 6) / 7.f;  // main.cpp:108
  auto gflops = [&](double ms) { return 2.0 * csr.nnz * O / (ms * 1e6); };
  std::vector<std::string> summary;
  std::vector<float> ref_c;
  auto report = [&](const char *name, const char *tag, double ms, const std::string &note,
                    const std::vector<float> *hc) {
    printf("%-16s %10.3f %12.2f %s\n", name, ms, gflops(ms), note.c_str());
    char line[512];
    snprintf(line, sizeof line, "%s: %.3f ms %.2f GFLOP/s [%s]", tag, ms, gflops(ms),
             note.c_str());
    summary.push_back(line);
    if (check && hc) {
      if (ref_c.empty()) ref_c = *hc;
      else printf("%-16s rel_l2 vs first kernel = %.3e\n", "", rel_l2(*hc, ref_c));
    }
  };
  const bool all = algo == "all";

  if (gpus > 1) {
    if (!(all || algo == "vcsr")) {
      fprintf(stderr, "error: --gpus > 1 runs --algo vcsr only\n");
      return 2;
    }
    vcsr_plan_params p;
    vcsr_plan_params_default(&p);
    p.segw = segw; p.bundle = bundle; p.max_O = std::max(O, 512);
    vcsr_mgpu *mg = nullptr;
    vcsr_csr view = as_view(csr);
    VK(vcsr_mgpu_create(&view, gpus, nullptr, &p, &mg));
    float bcast_ms = 0.f;
    VK(vcsr_mgpu_set_b(mg, hB.data(), O, &bcast_ms));
    float ms = 0.f;
    for (int i = 0; i < 3; ++i) VK(vcsr_mgpu_spmm(mg, O, &ms));
    double sum = 0;
    for (int i = 0; i < repeat; ++i) {
      VK(vcsr_mgpu_spmm(mg, O, &ms));
      sum += ms;
    }
    std::vector<float> hc(check ? nC : 0);
    if (check) VK(vcsr_mgpu_gather_c(mg, hc.data()));
    char note[256];
    snprintf(note, sizeof note, "gpus=%d,row panels,bcast_B=%.3f ms", gpus, bcast_ms);
    printf("%-16s %10s %12s %s\n", "Kernel", "Time (ms)", "GFLOP/s", "Notes");
    report("VCSR (x-GPU)", "VCSR (mgpu)", sum / repeat, note, check ? &hc : nullptr);
    vcsr_mgpu_destroy(mg);
    printf("\n");
    for (auto &s : summary) printf("%s\n", s.c_str());
    return 0;
  }

  float *dB = nullptr, *dC = nullptr;
  int *d_rp = nullptr, *d_col = nullptr;
  float *d_val = nullptr;
  CK(cudaMalloc(&dB, sizeof(float) * (nB ? nB : 1)));
  CK(cudaMalloc(&dC, sizeof(float) * (nC ? nC : 1)));
  CK(cudaMalloc(&d_rp, sizeof(int) * ((size_t)csr.M + 1)));
  CK(cudaMalloc(&d_col, sizeof(int) * (csr.nnz ? csr.nnz : 1)));
  CK(cudaMalloc(&d_val, sizeof(float) * (csr.nnz ? csr.nnz : 1)));
  CK(cudaMemcpy(dB, hB.data(), sizeof(float) * nB, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(d_rp, csr.row_ptr.data(), sizeof(int) * ((size_t)csr.M + 1),
                cudaMemcpyHostToDevice));
  if (csr.nnz) {
    CK(cudaMemcpy(d_col, csr.col.data(), sizeof(int) * csr.nnz, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(d_val, csr.val.data(), sizeof(float) * csr.nnz, cudaMemcpyHostToDevice));
  }
  cudaStream_t st;
  CK(cudaStreamCreate(&st));
  std::vector<float> hc(check ? nC : 0);
  auto fetch = [&]() -> const std::vector<float> * {
    if (!check) return nullptr;
    CK(cudaMemcpy(hc.data(), dC, sizeof(float) * nC, cudaMemcpyDeviceToHost));
    return &hc;
  };
  // times `repeat` launches after 3 warm-ups; zero_first for C += A*B kernels
  auto timed = [&](auto &&launch, bool zero_first) {
    Timer t;
    double sum = 0;
    for (int i = 0; i < 3 + repeat; ++i) {
      if (zero_first) CK(cudaMemsetAsync(dC, 0, sizeof(float) * nC, st));
      CK(cudaEventRecord(t.a, st));
      launch();
      CK(cudaEventRecord(t.b, st));
      CK(cudaEventSynchronize(t.b));
      float ms = 0;
      CK(cudaEventElapsedTime(&ms, t.a, t.b));
      if (i >= 3) sum += ms;
    }
    return sum / repeat;
  };

  printf("%-16s %10s %12s %s\n", "Kernel", "Time (ms)", "GFLOP/s", "Notes");
  printf("%-16s %10s %12s %s\n", "----------------", "----------", "------------", "-----");
  if (all || algo == "cusparse") {
    const char *names[] = {"ALG_DEFAULT", "CSR_ALG1", "CSR_ALG2", "CSR_ALG3"};
    double best = 1e30;
    int best_alg = -1;
    for (int a = 0; a < 4; ++a) {
      vcsr_cusparse *h = nullptr;
      if (vcsr_cusparse_create(csr.M, csr.N, csr.nnz, d_rp, d_col, d_val, dB, O, dC, a,
                               st, &h) != VCSR_OK)
        continue;
      double ms = timed([&] { VK(vcsr_cusparse_run(h, st)); }, false);
      vcsr_cusparse_destroy(h);
      if (ms < best) { best = ms; best_alg = a; }
    }
    if (best_alg >= 0) {
      vcsr_cusparse *h = nullptr;
      VK(vcsr_cusparse_create(csr.M, csr.N, csr.nnz, d_rp, d_col, d_val, dB, O, dC,
                              best_alg, st, &h));
      VK(vcsr_cusparse_run(h, st));
      CK(cudaStreamSynchronize(st));
      vcsr_cusparse_destroy(h);
      report("cuSPARSE", "cuSPARSE", best, std::string("vendor, best ") + names[best_alg],
             fetch());
    }
  }
  if (all || algo == "csr") {
    double ms = timed([&] {
      VK(vcsr_csr_spmm(csr.M, d_rp, d_col, d_val, dB, O, dC, st));
    }, false);
    report("CSR (row-wise)", "CSR", ms, "warp-per-row CSR", fetch());
  }
  // a plan of the engine with the given flags and vector height; its note
  // names the kernels that ran
  auto run_plan = [&](const char *name, const char *tag, int flags, int vec_rows,
                      const char *what) {
    vcsr_plan_params p;
    vcsr_plan_params_default(&p);
    p.segw = segw; p.bundle = bundle; p.tileK = tileK; p.max_O = std::max(O, 512);
    p.flags = flags;
    p.vec_rows = vec_rows;
    vcsr_plan *plan = nullptr;
    vcsr_csr view = as_view(csr);
    VK(vcsr_plan_create(&view, VCSR_HOST, &p, &plan, st));
    vcsr_plan_info info{};
    VK(vcsr_plan_get_info(plan, &info));
    int launches = 0;
    double ms = timed([&] { VK(vcsr_spmm(plan, dB, O, dC, O, O, st, &launches)); }, false);
    VK(vcsr_plan_check(plan, st));
    char note[320];
    snprintf(note, sizeof note,
             "%s,vec_rows=%d,units=%d,split=%d,long=%d,tc_nnz=%lld,launches=%d,build=%.1f ms",
             what, info.vec_rows, info.num_units, info.num_split_units, info.num_long_units,
             (long long)info.panel_nnz, launches, info.build_ms);
    report(name, tag, ms, note, fetch());
    vcsr_plan_destroy(plan);
  };
  if (all || algo == "aspt")
    run_plan("ASPT (engine)", "ASPT", 0, 1,
             "engine panels at 1 row/vector: sub-warp per short row, warp per long row");
  if (all || algo == "vcsr") {
    vcsr_plan_params p;
    vcsr_plan_params_default(&p);
    p.segw = segw; p.bundle = bundle; p.tileK = tileK; p.max_O = std::max(O, 512);
    vcsr_plan *plan = nullptr;
    vcsr_csr view = as_view(csr);
    VK(vcsr_plan_create(&view, VCSR_HOST, &p, &plan, st));
    vcsr_plan_info info{};
    VK(vcsr_plan_get_info(plan, &info));
    double ms = timed([&] { VK(vcsr_spmm(plan, dB, O, dC, O, O, st, nullptr)); }, false);
    char note[256];
    snprintf(note, sizeof note, "row-stationary,vec_rows=%d,units=%d,split=%d,build=%.1f ms",
             info.vec_rows, info.num_units, info.num_split_units, info.build_ms);
    report("VCSR (engine)", "VCSR", ms, note, fetch());
    vcsr_plan_destroy(plan);
  }
  if (all || algo == "vcsr_seg" || algo == "vcsr_baseline") {
    vcsr_csr dv{csr.M, csr.N, csr.nnz, d_rp, d_col, d_val};
    vcsr_vcsr v{};
    VK(vcsr_build_vcsr(&dv, segw, bundle, &v, st));
    double ms = timed([&] { VK(vcsr_spmm_segmented(&v, dB, O, tileK, dC, st)); }, true);
    char note[256];
    snprintf(note, sizeof note, "segw=%d,bundle=%d,tileK=%d,groups=%d", segw, bundle,
             tileK, v.num_groups);
    report("VCSR (seg)", "VCSR (seg)", ms, note, fetch());
    vcsr_vcsr_free(&v, VCSR_DEVICE);
  }
  if (all || algo == "vcsr_tc") {  // dense 16x16 blocks on the tensor cores (TF32)
    if (O % 4) {
      printf("%-16s %10s %12s (TF32 panels need O %% 4 == 0)\n", "VCSR_TC", "N/A", "N/A");
    } else {
      vcsr_plan_params p;
      vcsr_plan_params_default(&p);
      p.segw = segw; p.bundle = bundle; p.tileK = tileK; p.max_O = std::max(O, 512);
      p.flags = VCSR_PLAN_TF32_PANELS;
      vcsr_plan *plan = nullptr;
      vcsr_csr view = as_view(csr);
      VK(vcsr_plan_create(&view, VCSR_HOST, &p, &plan, st));
      vcsr_plan_info info{};
      VK(vcsr_plan_get_info(plan, &info));
      double ms = timed([&] { VK(vcsr_spmm(plan, dB, O, dC, O, O, st, nullptr)); }, false);
      VK(vcsr_plan_check(plan, st));
      char note[256];
      snprintf(note, sizeof note, "tcgen05 TF32 panels=%d (%lld nnz),residual vec_rows=%d",
               info.num_panel_blocks, (long long)info.panel_nnz, info.vec_rows);
      report("VCSR_TC (TF32)", "VCSR_TC", ms, note, fetch());
      vcsr_plan_destroy(plan);
    }
  }
  if (all || algo == "vcsr_tcseg") {  // column runs on the tensor cores, FP32 accuracy
    if (O % 4) {
      printf("%-16s %10s %12s (tensor-core segments need O %% 4 == 0)\n", "VCSR_TCSEG", "N/A",
             "N/A");
    } else {
      run_plan("VCSR_TCSEG", "VCSR_TCSEG", VCSR_PLAN_TC_SEGMENTS, 0,
               "tcgen05 split-TF32 column runs + FP32 residual");
    }
  }
  if (all || algo == "fast" || algo == "fastspmm")
    run_plan("FastSpMM (engine)", "FAST", 0, 16,
             "16-row windows with condensed columns: engine panels at 16 rows/vector, FP32");
  if (algo == "vcsr_naive")
    printf("%-16s %10s %12s (not provided by this engine)\n", "vcsr_naive", "N/A", "N/A");
  printf("\n");
  for (auto &s : summary) printf("%s\n", s.c_str());
  cudaStreamDestroy(st);
  cudaFree(dB); cudaFree(dC); cudaFree(d_rp); cudaFree(d_col); cudaFree(d_val);
  return 0;
}
