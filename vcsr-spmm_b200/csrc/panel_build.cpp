// panel_build.cpp — host construction of the row-stationary vector panels
// (layout described in panel.h).
#include <algorithm>
#include <cstring>
#include <numeric>
#include <vector>

#include <omp.h>

#include "common.h"
#include "panel.h"

namespace vcsr {

namespace {

// Sorted (column, occurrence) keys of rows [r0, r1): the union of a vector.
void union_keys(const vcsr_csr &csr, int r0, int r1, std::vector<uint64_t> &k) {
  k.clear();
  for (int r = r0; r < r1; ++r) {
    int occ = 0;
    for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) {
      occ = (p > csr.row_ptr[r] && csr.col[p] == csr.col[p - 1]) ? occ + 1 : 0;
      k.push_back(((uint64_t)(uint32_t)csr.col[p] << 32) | (uint32_t)occ);
    }
  }
  std::sort(k.begin(), k.end());
  k.erase(std::unique(k.begin(), k.end()), k.end());
}

}  // namespace

int choose_vec_rows(const vcsr_csr &csr, double *density_out) {
  const int cands[] = {1, 2, 4, 8, 16};
  const int M = csr.M;
  const int windows = (M + 15) / 16;
  const int samples = std::min(windows, 4096);
  if (samples == 0) {
    if (density_out) *density_out = 1.0;
    return 1;
  }
  double unions[5] = {0, 0, 0, 0, 0};
  int64_t nnz_s = 0;
#pragma omp parallel reduction(+ : nnz_s)
  {
    std::vector<uint64_t> k;
    double loc[5] = {0, 0, 0, 0, 0};
#pragma omp for schedule(dynamic, 16)
    for (int s = 0; s < samples; ++s) {
      const int w = (int)((int64_t)s * windows / samples);
      const int r0 = w * 16, r1 = std::min(M, r0 + 16);
      nnz_s += csr.row_ptr[r1] - csr.row_ptr[r0];
      for (int ci = 0; ci < 5; ++ci) {
        const int R = cands[ci];
        for (int v0 = r0; v0 < r1; v0 += R) {
          union_keys(csr, v0, std::min(r1, v0 + R), k);
          loc[ci] += (double)k.size();
        }
      }
    }
#pragma omp critical
    for (int ci = 0; ci < 5; ++ci) unions[ci] += loc[ci];
  }
  // The largest R (up to 8) whose vectors are still at least 60% dense:
  // measured on B200, a denser vector trades one B-row load for more FMAs per
  // union column, while below ~60% density the padded FMAs cost more than the
  // saved loads.  R = 16 is never picked automatically (its 64 float
  // accumulators per lane halve occupancy); callers may still ask for it.
  int best = 1;
  for (int ci = 1; ci < 4; ++ci) {
    const int R = cands[ci];
    const double dens = unions[ci] > 0 ? (double)nnz_s / (unions[ci] * R) : 0.0;
    if (dens >= 0.6) best = R;
  }
  if (density_out) {
    int ci = 0;
    while (cands[ci] != best) ++ci;
    *density_out = unions[ci] > 0 ? (double)nnz_s / (unions[ci] * best) : 1.0;
  }
  return best;
}

vcsr_status build_panel_host(const vcsr_csr &csr, int R, int chunk, int sms,
                             PanelHost *out) {
  if (R != 1 && R != 2 && R != 4 && R != 8 && R != 16)
    return fail(VCSR_ERR_INVALID, "vec_rows must be 1, 2, 4, 8 or 16 (got %d)", R);
  const int M = csr.M;
  const int V = (int)ceil_div(M, R);
  out->R = R;
  out->num_vectors = V;
  out->chunk = chunk;
  out->vec_ptr.assign((size_t)V + 1, 0);
  if (R == 1) {
    std::copy(csr.row_ptr, csr.row_ptr + M + 1, out->vec_ptr.begin());
    out->ucol.assign(csr.col, csr.col + csr.nnz);
    out->uval.assign(csr.val, csr.val + csr.nnz);
  } else {
    std::vector<int64_t> cnt((size_t)V + 1, 0);
#pragma omp parallel
    {
      std::vector<uint64_t> k;
#pragma omp for schedule(dynamic, 64)
      for (int v = 0; v < V; ++v) {
        union_keys(csr, v * R, std::min(M, v * R + R), k);
        cnt[v + 1] = (int64_t)k.size();
      }
    }
    for (int v = 0; v < V; ++v) cnt[v + 1] += cnt[v];
    if (cnt[V] > INT32_MAX || cnt[V] * R > ((int64_t)1 << 40))
      return fail(VCSR_ERR_UNSUPPORTED, "panel layout exceeds 32-bit indexing");
    for (int v = 0; v <= V; ++v) out->vec_ptr[v] = (int)cnt[v];
    out->ucol.assign((size_t)cnt[V], 0);
    out->uval.assign((size_t)cnt[V] * R, 0.f);
    out->umask.assign((size_t)cnt[V], 0u);
#pragma omp parallel
    {
      std::vector<uint64_t> k;
#pragma omp for schedule(dynamic, 64)
      for (int v = 0; v < V; ++v) {
        const int r0 = v * R, r1 = std::min(M, r0 + R);
        union_keys(csr, r0, r1, k);
        const int64_t base = cnt[v];
        for (size_t j = 0; j < k.size(); ++j) out->ucol[base + j] = (int)(k[j] >> 32);
        for (int r = r0; r < r1; ++r) {
          // walk the row against the sorted union (both ordered by key)
          size_t j = 0;
          int occ = 0;
          for (int p = csr.row_ptr[r]; p < csr.row_ptr[r + 1]; ++p) {
            occ = (p > csr.row_ptr[r] && csr.col[p] == csr.col[p - 1]) ? occ + 1 : 0;
            const uint64_t key = ((uint64_t)(uint32_t)csr.col[p] << 32) | (uint32_t)occ;
            while (k[j] < key) ++j;
            out->uval[(size_t)(base + j) * R + (r - r0)] = csr.val[p];
            out->umask[(size_t)(base + j)] |= 1u << (r - r0);
          }
        }
      }
    }
  }
  // nnz-balanced units
  if (chunk <= 0) {
    const int64_t total = out->vec_ptr[V];
    const int64_t per = total / ((int64_t)(sms > 0 ? sms : 148) * 32);
    // Long vectors are split only where they are long compared with the
    // average one: on R-MAT 2^22 at O = 256 (average 15 columns) parts of at
    // most 512 union columns give the hub rows enough warps (2048: 8.1 ms,
    // 512: 6.5 ms), while block-dense (average ~700) stays unsplit.
    const int64_t avg = V > 0 ? total / V : 0;
    const int64_t cap = std::max<int64_t>(512, 2 * avg);
    chunk = (int)std::max<int64_t>(256, std::min<int64_t>(std::min(per, cap), 2048));
  }
  out->chunk = chunk;
  out->units.clear();
  out->parts.clear();
  out->svecs.clear();
  for (int v = 0; v < V; ++v) {
    const int b = out->vec_ptr[v], e = out->vec_ptr[v + 1];
    const int n = e - b;
    const int nparts = n > chunk ? (int)ceil_div(n, chunk) : 1;
    if (nparts == 1) {
      out->units.push_back({v, b, e, -1});
      continue;
    }
    const int sv = (int)out->svecs.size();
    const int first = (int)out->parts.size();
    out->svecs.push_back({first, nparts});
    const int per = (int)ceil_div(n, nparts);
    for (int q = 0; q < nparts; ++q) {
      const int pb = b + q * per, pe = std::min(e, pb + per);
      out->units.push_back({v, pb, pe, first + q});
      out->parts.push_back({sv, q});
    }
  }
  return VCSR_OK;
}

}  // namespace vcsr
