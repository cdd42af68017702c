// gen.cpp — deterministic synthetic matrices for the five workloads.
//
// Every random draw is rnd(stream_key(seed, stream), index) (rng.h), so the
// output depends only on (config, seed, size_param), not on thread count or
// scheduling.  The configurations are synthetic stand-ins with the shapes,
// sizes and value distributions the benchmark configurations name:
//   uniform    4096 x 4096, exactly 16 distinct uniform columns per row,
//              values U[-1,1)
//   fem        62,451 x 62,451 structural-mechanics-like banded pattern: 3
//              degrees of freedom per mesh node (rows 3n..3n+2 share a
//              pattern), node n linked to node m (m > n) with probability 0.78
//              when m-n <= 4 or |m-n-150| <= 4, pattern symmetric; three bands
//              (the diagonal band and +-450 rows, all within +-500); ~64 nnz
//              per row; values U[-1,1) symmetric, diagonal |row sum| + 1
//   powerlaw   321,821 x 321,821 circuit-like: row lengths Zipf(2.1) on
//              1..330, columns 70% within +-50 of the row and 30% uniform,
//              plus 3 dense rows and 3 dense columns (~150k entries each);
//              values lognormal(0,1) with a random sign
//   rmat       2^scale square R-MAT (a,b,c,d) = (.57,.19,.19,.05) with
//              16 * 2^scale edges, duplicates merged, values U[0,1)
//   blockdense 65,536 x 65,536: dense 16x16 blocks on 1% of the block grid
//              plus 8 uniform residual entries per row (merged), U[-1,1)
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <omp.h>

#include "common.h"
#include "rng.h"

using vcsr::fail;
using vcsr::rnd;
using vcsr::stream_key;

namespace {

enum Stream : uint64_t {
  S_COLS = 1, S_VALS = 2, S_EDGE = 3, S_LEN = 4, S_DENSE = 5, S_SIGN = 6,
  S_BLOCK = 7, S_PICK = 8
};

struct RowLists {
  std::vector<std::vector<int>> cols;
  std::vector<std::vector<float>> vals;
};

vcsr_status pack_rows(int M, int N, RowLists &rl, vcsr_csr *out) {
  std::vector<int64_t> rp(M + 1, 0);
  for (int r = 0; r < M; ++r) rp[r + 1] = rp[r] + (int64_t)rl.cols[r].size();
  if (rp[M] > INT32_MAX)
    return fail(VCSR_ERR_UNSUPPORTED, "generated nnz %lld exceeds int32",
                (long long)rp[M]);
  const int nnz = (int)rp[M];
  out->row_ptr = (int *)malloc(sizeof(int) * ((size_t)M + 1));
  out->col = (int *)malloc(sizeof(int) * (size_t)(nnz ? nnz : 1));
  out->val = (float *)malloc(sizeof(float) * (size_t)(nnz ? nnz : 1));
  if (!out->row_ptr || !out->col || !out->val) {
    free(out->row_ptr); free(out->col); free(out->val);
    std::memset(out, 0, sizeof *out);
    return fail(VCSR_ERR_ALLOC, "out of host memory");
  }
  for (int r = 0; r <= M; ++r) out->row_ptr[r] = (int)rp[r];
#pragma omp parallel for schedule(dynamic, 1024)
  for (int r = 0; r < M; ++r) {
    std::copy(rl.cols[r].begin(), rl.cols[r].end(), out->col + rp[r]);
    std::copy(rl.vals[r].begin(), rl.vals[r].end(), out->val + rp[r]);
  }
  out->M = M; out->N = N; out->nnz = nnz;
  return VCSR_OK;
}

// -------------------------------------------------------------- uniform
vcsr_status gen_uniform(uint64_t seed, int M, vcsr_csr *out) {
  const int N = M, per = std::min(16, N);
  RowLists rl;
  rl.cols.resize(M);
  rl.vals.resize(M);
  const uint64_t kc = stream_key(seed, S_COLS), kv = stream_key(seed, S_VALS);
#pragma omp parallel for schedule(static)
  for (int r = 0; r < M; ++r) {
    auto &c = rl.cols[r];
    uint64_t t = 0;
    while ((int)c.size() < per) {
      int x = (int)vcsr::below(rnd(kc, (uint64_t)r * 1024 + t++), (uint32_t)N);
      if (std::find(c.begin(), c.end(), x) == c.end()) c.push_back(x);
    }
    std::sort(c.begin(), c.end());
    rl.vals[r].resize(per);
    for (int j = 0; j < per; ++j)
      rl.vals[r][j] = vcsr::uniform_f(rnd(kv, (uint64_t)r * per + j), -1.f, 1.f);
  }
  return pack_rows(M, N, rl, out);
}

// ------------------------------------------------------------------ fem
vcsr_status gen_fem(uint64_t seed, int M, vcsr_csr *out) {
  const int N = M;
  const int dof = 3, H0 = 4, D = 150, H1 = 4;
  const double p_link = 0.78;
  const int64_t nodes = (M + dof - 1) / dof;
  const uint64_t ke = stream_key(seed, S_EDGE), kv = stream_key(seed, S_VALS);
  auto linked = [&](int64_t a, int64_t b) -> bool {  // a < b
    int64_t d = b - a;
    if (!((d >= 1 && d <= H0) || (d >= D - H1 && d <= D + H1))) return false;
    return vcsr::u01d(rnd(ke, (uint64_t)a * (uint64_t)nodes + (uint64_t)b)) <
           p_link;
  };
  auto offval = [&](int64_t i, int64_t j) -> float {  // symmetric in (i, j)
    int64_t a = std::min(i, j), b = std::max(i, j);
    return vcsr::uniform_f(rnd(kv, (uint64_t)a * (uint64_t)N + (uint64_t)b),
                           -1.f, 1.f);
  };
  RowLists rl;
  rl.cols.resize(M);
  rl.vals.resize(M);
#pragma omp parallel for schedule(dynamic, 64)
  for (int64_t n = 0; n < nodes; ++n) {
    std::vector<int64_t> adj;
    for (int64_t d = -(D + H1); d <= D + H1; ++d) {
      int64_t m = n + d;
      if (m < 0 || m >= nodes) continue;
      if (d == 0) { adj.push_back(m); continue; }
      if (d > 0 ? linked(n, m) : linked(m, n)) adj.push_back(m);
    }
    for (int k = 0; k < dof; ++k) {
      const int64_t i = n * dof + k;
      if (i >= M) break;
      auto &c = rl.cols[i];
      auto &v = rl.vals[i];
      for (int64_t m : adj)
        for (int q = 0; q < dof; ++q) {
          int64_t j = m * dof + q;
          if (j < N) c.push_back((int)j);
        }
      v.resize(c.size());
      double rowsum = 0.0;
      size_t diag = 0;
      for (size_t t = 0; t < c.size(); ++t) {
        if (c[t] == i) { diag = t; continue; }
        v[t] = offval(i, c[t]);
        rowsum += v[t];
      }
      v[diag] = (float)(std::fabs(rowsum) + 1.0);
    }
  }
  return pack_rows(M, N, rl, out);
}

// ------------------------------------------------------------- powerlaw
vcsr_status gen_powerlaw(uint64_t seed, int M, vcsr_csr *out) {
  const int N = M;
  const int Kmax = 330, local = 50;
  const double zipf_s = 2.1;
  const int64_t dense_target = std::min<int64_t>(150000, N);
  const double p_dense = (double)dense_target / N;
  const uint64_t kl = stream_key(seed, S_LEN), kc = stream_key(seed, S_COLS),
                 kv = stream_key(seed, S_VALS), kd = stream_key(seed, S_DENSE),
                 ks = stream_key(seed, S_SIGN), kp = stream_key(seed, S_PICK);
  // inverse CDF of the truncated Zipf law
  std::vector<double> cdf(Kmax + 1, 0.0);
  for (int k = 1; k <= Kmax; ++k) cdf[k] = cdf[k - 1] + std::pow((double)k, -zipf_s);
  for (int k = 1; k <= Kmax; ++k) cdf[k] /= cdf[Kmax];
  // three distinct dense row/column indices
  std::vector<int> dense;
  for (uint64_t t = 0; (int)dense.size() < std::min(3, N); ++t) {
    int x = (int)vcsr::below(rnd(kp, t), (uint32_t)N);
    if (std::find(dense.begin(), dense.end(), x) == dense.end()) dense.push_back(x);
  }
  auto value = [&](int64_t r, int64_t c) -> float {
    uint64_t id = (uint64_t)r * (uint64_t)N + (uint64_t)c;
    double u1 = 1.0 - vcsr::u01d(rnd(kv, 2 * id));  // (0, 1]
    double u2 = vcsr::u01d(rnd(kv, 2 * id + 1));
    double z = std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2);
    float mag = (float)std::exp(z);
    return (rnd(ks, id) >> 63) ? -mag : mag;
  };
  RowLists rl;
  rl.cols.resize(M);
  rl.vals.resize(M);
#pragma omp parallel for schedule(dynamic, 256)
  for (int r = 0; r < M; ++r) {
    auto &c = rl.cols[r];
    bool is_dense = std::find(dense.begin(), dense.end(), r) != dense.end();
    if (is_dense) {
      for (int j = 0; j < N; ++j)
        if (vcsr::u01d(rnd(kd, (uint64_t)r * (uint64_t)N + j)) < p_dense)
          c.push_back(j);
    } else {
      double u = vcsr::u01d(rnd(kl, (uint64_t)r));
      int L = (int)(std::lower_bound(cdf.begin() + 1, cdf.end(), u) - cdf.begin());
      if (L > Kmax) L = Kmax;
      if (L > N) L = N;
      uint64_t t = 0;
      while ((int)c.size() < L) {
        uint64_t x = rnd(kc, (uint64_t)r * 65536 + t);
        ++t;
        int j;
        if (t <= 8 * (uint64_t)L && vcsr::u01f(x) < 0.7f) {
          int off = (int)vcsr::below(vcsr::vmix64(x), 2 * local + 1) - local;
          j = std::min(std::max(r + off, 0), N - 1);
        } else {
          j = (int)vcsr::below(vcsr::vmix64(x ^ 0x5bd1e995ull), (uint32_t)N);
        }
        if (std::find(c.begin(), c.end(), j) == c.end()) c.push_back(j);
      }
      for (int dcol : dense)  // the dense columns
        if (vcsr::u01d(rnd(kd, ((uint64_t)dcol * (uint64_t)N + (uint64_t)r) ^ (1ull << 62))) <
                p_dense &&
            std::find(c.begin(), c.end(), dcol) == c.end())
          c.push_back(dcol);
    }
    std::sort(c.begin(), c.end());
    rl.vals[r].resize(c.size());
    for (size_t t = 0; t < c.size(); ++t) rl.vals[r][t] = value(r, c[t]);
  }
  return pack_rows(M, N, rl, out);
}

// ------------------------------------------------------------------ rmat
vcsr_status gen_rmat(uint64_t seed, int scale, vcsr_csr *out) {
  if (scale < 1 || scale > 28)
    return fail(VCSR_ERR_INVALID, "rmat scale %d out of [1, 28]", scale);
  const int64_t M = (int64_t)1 << scale;
  const int64_t E = 16 * M;
  // quadrant thresholds of (a, a+b, a+b+c) = (.57, .76, .95) in 16 bits
  const uint32_t ta = 37355, tb = 49807, tc = 62259;
  const uint64_t ke = stream_key(seed, S_EDGE), kv = stream_key(seed, S_VALS);
  std::vector<int> er(E), ec(E);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < E; ++e) {
    uint32_t r = 0, c = 0;
    uint64_t bits = 0;
    for (int l = 0; l < scale; ++l) {
      if ((l & 3) == 0) bits = rnd(ke, (uint64_t)e * 8 + (l >> 2));
      uint32_t u = (uint32_t)(bits & 0xFFFF);
      bits >>= 16;
      uint32_t rb = (u >= tb) ? 1u : 0u;
      uint32_t cb = (u >= ta && u < tb) || (u >= tc) ? 1u : 0u;
      r = (r << 1) | rb;
      c = (c << 1) | cb;
    }
    er[e] = (int)r;
    ec[e] = (int)c;
  }
  std::vector<std::atomic<int>> cnt(M + 1);
  for (auto &x : cnt) x.store(0, std::memory_order_relaxed);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < E; ++e) cnt[er[e] + 1].fetch_add(1, std::memory_order_relaxed);
  std::vector<int64_t> start(M + 1, 0);
  for (int64_t r = 0; r < M; ++r) start[r + 1] = start[r] + cnt[r + 1].load();
  std::vector<int> bucket(E);
  for (int64_t r = 0; r <= M; ++r) cnt[r].store(0, std::memory_order_relaxed);
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < E; ++e) {
    int r = er[e];
    int pos = cnt[r].fetch_add(1, std::memory_order_relaxed);
    bucket[start[r] + pos] = ec[e];
  }
  std::vector<int>().swap(er);
  std::vector<int>().swap(ec);
  std::vector<int64_t> uniq(M + 1, 0);
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t r = 0; r < M; ++r) {
    int *b = bucket.data() + start[r], *e = bucket.data() + start[r + 1];
    std::sort(b, e);
    uniq[r + 1] = std::unique(b, e) - b;
  }
  for (int64_t r = 0; r < M; ++r) uniq[r + 1] += uniq[r];
  if (uniq[M] > INT32_MAX) return fail(VCSR_ERR_UNSUPPORTED, "rmat nnz > int32");
  const int nnz = (int)uniq[M];
  out->row_ptr = (int *)malloc(sizeof(int) * ((size_t)M + 1));
  out->col = (int *)malloc(sizeof(int) * (size_t)(nnz ? nnz : 1));
  out->val = (float *)malloc(sizeof(float) * (size_t)(nnz ? nnz : 1));
  if (!out->row_ptr || !out->col || !out->val) {
    free(out->row_ptr); free(out->col); free(out->val);
    std::memset(out, 0, sizeof *out);
    return fail(VCSR_ERR_ALLOC, "out of host memory");
  }
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t r = 0; r < M; ++r) {
    out->row_ptr[r] = (int)uniq[r];
    const int64_t n = uniq[r + 1] - uniq[r];
    for (int64_t t = 0; t < n; ++t) {
      int c = bucket[start[r] + t];
      out->col[uniq[r] + t] = c;
      out->val[uniq[r] + t] = vcsr::uniform_f(
          rnd(kv, (uint64_t)r * (uint64_t)M + (uint64_t)c), 0.f, 1.f);
    }
  }
  out->row_ptr[M] = nnz;
  out->M = (int)M; out->N = (int)M; out->nnz = nnz;
  return VCSR_OK;
}

// ------------------------------------------------------------ blockdense
vcsr_status gen_blockdense(uint64_t seed, int M, vcsr_csr *out) {
  if (M % 16) return fail(VCSR_ERR_INVALID, "blockdense size must be a multiple of 16");
  const int N = M, nb = M / 16, resid = std::min(8, N);
  const double p_block = 0.01;
  const uint64_t kb = stream_key(seed, S_BLOCK), kc = stream_key(seed, S_COLS),
                 kv = stream_key(seed, S_VALS);
  RowLists rl;
  rl.cols.resize(M);
  rl.vals.resize(M);
#pragma omp parallel for schedule(dynamic, 4)
  for (int bi = 0; bi < nb; ++bi) {
    std::vector<int> blocks;
    for (int bj = 0; bj < nb; ++bj)
      if (vcsr::u01d(rnd(kb, (uint64_t)bi * nb + bj)) < p_block) blocks.push_back(bj);
    for (int k = 0; k < 16; ++k) {
      const int r = bi * 16 + k;
      auto &c = rl.cols[r];
      for (int bj : blocks)
        for (int q = 0; q < 16; ++q) c.push_back(bj * 16 + q);
      std::vector<int> extra;
      uint64_t t = 0;
      while ((int)extra.size() < resid && t < 64 * (uint64_t)resid) {
        int j = (int)vcsr::below(rnd(kc, (uint64_t)r * 4096 + t++), (uint32_t)N);
        if (std::binary_search(blocks.begin(), blocks.end(), j / 16)) continue;
        if (std::find(extra.begin(), extra.end(), j) != extra.end()) continue;
        extra.push_back(j);
      }
      c.insert(c.end(), extra.begin(), extra.end());
      std::sort(c.begin(), c.end());
      rl.vals[r].resize(c.size());
      for (size_t t2 = 0; t2 < c.size(); ++t2)
        rl.vals[r][t2] = vcsr::uniform_f(
            rnd(kv, (uint64_t)r * (uint64_t)N + (uint64_t)c[t2]), -1.f, 1.f);
    }
  }
  return pack_rows(M, N, rl, out);
}

}  // namespace

extern "C" vcsr_status vcsr_gen_csr(const char *config, uint64_t seed,
                                    int size_param, vcsr_csr *out) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!config || !out) return fail(VCSR_ERR_INVALID, "null argument");
    std::memset(out, 0, sizeof *out);
    if (size_param < 0) return fail(VCSR_ERR_INVALID, "negative size_param");
    std::string c(config);
    if (c == "uniform") return gen_uniform(seed, size_param ? size_param : 4096, out);
    if (c == "fem") return gen_fem(seed, size_param ? size_param : 62451, out);
    if (c == "powerlaw")
      return gen_powerlaw(seed, size_param ? size_param : 321821, out);
    if (c == "rmat") return gen_rmat(seed, size_param ? size_param : 22, out);
    if (c == "blockdense")
      return gen_blockdense(seed, size_param ? size_param : 65536, out);
    return fail(VCSR_ERR_INVALID,
                "unknown config '%s' (uniform|fem|powerlaw|rmat|blockdense)", config);
  });
}
