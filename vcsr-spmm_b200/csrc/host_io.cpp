// host_io.cpp — host-side input surface: errors, Matrix Market reader,
// COO -> CSR, container frees, row panels and the nnz-balanced partitioner.
//
// vcsr_read_mtx follows read_matrix_market_coo (include/mmio.hpp:22-45) and
// vcsr_coo_to_csr follows coo_to_csr (include/csr.hpp:16-37); both are
// rewritten for speed (one buffered read, a multi-threaded per-row sort).
#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <omp.h>

#include "common.h"

namespace vcsr {

static thread_local std::string g_error;

vcsr_status fail(vcsr_status s, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return s;
}

void clear_error() { g_error.clear(); }

}  // namespace vcsr

using vcsr::fail;

extern "C" {

const char *vcsr_last_error(void) { return vcsr::g_error.c_str(); }

int vcsr_abi_version(void) { return VCSR_ABI_VERSION; }

const char *vcsr_status_string(vcsr_status s) {
  switch (s) {
    case VCSR_OK: return "ok";
    case VCSR_ERR_INVALID: return "invalid argument";
    case VCSR_ERR_CUDA: return "CUDA error";
    case VCSR_ERR_ALLOC: return "allocation failed";
    case VCSR_ERR_IO: return "I/O error";
    case VCSR_ERR_UNSUPPORTED: return "unsupported";
    case VCSR_ERR_NCCL: return "NCCL error";
    case VCSR_ERR_TIMEOUT: return "timeout";
    case VCSR_ERR_RANGE: return "index out of range";
  }
  return "unknown status";
}

void vcsr_coo_free(vcsr_coo *coo) {
  if (!coo) return;
  free(coo->rows); free(coo->cols); free(coo->vals);
  std::memset(coo, 0, sizeof *coo);
}

// ------------------------------------------------------------ MTX reader

static inline bool is_space(char c) {
  return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\v' ||
         c == '\f';
}

vcsr_status vcsr_read_mtx(const char *path, vcsr_coo *out) {
  vcsr::clear_error();
  if (!path || !out) return fail(VCSR_ERR_INVALID, "null argument");
  std::memset(out, 0, sizeof *out);
  FILE *f = fopen(path, "rb");
  if (!f) return fail(VCSR_ERR_IO, "Failed to open MTX: %s", path);
  std::string buf;
  {
    if (fseek(f, 0, SEEK_END) == 0) {
      long sz = ftell(f);
      if (sz > 0) buf.reserve((size_t)sz + 1);
      fseek(f, 0, SEEK_SET);
    }
    char chunk[1 << 16];
    size_t n;
    while ((n = fread(chunk, 1, sizeof chunk, f)) > 0) buf.append(chunk, n);
    fclose(f);
  }
  const char *p = buf.c_str(), *end = p + buf.size();
  // size line: first line that is neither empty nor starts with '%'
  long long M = -1, N = -1, Z = -1;
  bool found = false;
  while (p < end) {
    const char *eol = (const char *)memchr(p, '\n', end - p);
    if (!eol) eol = end;
    if (eol > p && *p != '%') {
      std::string line(p, eol);
      if (sscanf(line.c_str(), "%lld %lld %lld", &M, &N, &Z) != 3)
        return fail(VCSR_ERR_IO, "Invalid MTX header or empty file");
      p = eol < end ? eol + 1 : end;
      found = true;
      break;
    }
    p = eol < end ? eol + 1 : end;
  }
  if (!found || M < 0 || N < 0 || Z < 0)
    return fail(VCSR_ERR_IO, "Invalid MTX header or empty file");
  if (M > INT32_MAX || N > INT32_MAX || Z > INT32_MAX)
    return fail(VCSR_ERR_UNSUPPORTED, "MTX dimensions exceed 32-bit indexing");
  int *R = (int *)malloc(sizeof(int) * (size_t)(Z ? Z : 1));
  int *Cc = (int *)malloc(sizeof(int) * (size_t)(Z ? Z : 1));
  float *V = (float *)malloc(sizeof(float) * (size_t)(Z ? Z : 1));
  if (!R || !Cc || !V) {
    free(R); free(Cc); free(V);
    return fail(VCSR_ERR_ALLOC, "out of host memory");
  }
  auto bad = [&]() {
    free(R); free(Cc); free(V);
    return fail(VCSR_ERR_IO, "Bad MTX data");
  };
  // tokens, whitespace separated, across line ends (operator>> semantics)
  auto next_tok = [&](const char *&b, const char *&e) -> bool {
    while (p < end && is_space(*p)) ++p;
    if (p >= end) return false;
    b = p;
    while (p < end && !is_space(*p)) ++p;
    e = p;
    return true;
  };
  auto parse_int = [&](int &v) -> bool {
    const char *b, *e;
    if (!next_tok(b, e)) return false;
    std::string t(b, e);
    char *q;
    errno = 0;
    long x = strtol(t.c_str(), &q, 10);
    if (q == t.c_str() || *q || errno || x < INT32_MIN || x > INT32_MAX)
      return false;
    v = (int)x;
    return true;
  };
  auto parse_val = [&](double &v) -> bool {
    const char *b, *e;
    if (!next_tok(b, e)) return false;
    for (const char *q = b; q < e; ++q)
      if (!((*q >= '0' && *q <= '9') || *q == '.' || *q == '+' || *q == '-' ||
            *q == 'e' || *q == 'E'))
        return false;
    std::string t(b, e);
    char *q;
    errno = 0;
    v = strtod(t.c_str(), &q);
    if (q == t.c_str() || *q) return false;
    if (errno == ERANGE && (v == HUGE_VAL || v == -HUGE_VAL)) return false;
    return true;
  };
  bool one_based = true;
  for (long long i = 0; i < Z; ++i) {
    int r, c;
    double v;
    if (!parse_int(r) || !parse_int(c) || !parse_val(v)) return bad();
    if (i == 0 && (r == 0 || c == 0)) one_based = false;
    R[i] = r - (one_based ? 1 : 0);
    Cc[i] = c - (one_based ? 1 : 0);
    V[i] = (float)v;
  }
  out->M = (int)M; out->N = (int)N; out->nnz = (int)Z;
  out->rows = R; out->cols = Cc; out->vals = V;
  return VCSR_OK;
}

// ------------------------------------------------------------ COO -> CSR

vcsr_status vcsr_coo_to_csr(const vcsr_coo *coo, vcsr_csr *out) {
  vcsr::clear_error();
  if (!coo || !out) return fail(VCSR_ERR_INVALID, "null argument");
  std::memset(out, 0, sizeof *out);
  const int M = coo->M, N = coo->N, nnz = coo->nnz;
  if (M < 0 || N < 0 || nnz < 0) return fail(VCSR_ERR_INVALID, "negative size");
  int *rp = (int *)calloc((size_t)M + 1, sizeof(int));
  int *cc = (int *)malloc(sizeof(int) * (size_t)(nnz ? nnz : 1));
  float *vv = (float *)malloc(sizeof(float) * (size_t)(nnz ? nnz : 1));
  if (!rp || !cc || !vv) {
    free(rp); free(cc); free(vv);
    return fail(VCSR_ERR_ALLOC, "out of host memory");
  }
  for (int i = 0; i < nnz; ++i) {
    const int r = coo->rows[i], c = coo->cols[i];
    if (r < 0 || r >= M) {
      free(rp); free(cc); free(vv);
      return fail(VCSR_ERR_RANGE, "row idx out of range (entry %d: row %d, M=%d)",
                  i, r, M);
    }
    if (c < 0 || c >= N) {
      free(rp); free(cc); free(vv);
      return fail(VCSR_ERR_RANGE, "col idx out of range (entry %d: col %d, N=%d)",
                  i, c, N);
    }
    rp[r + 1]++;
  }
  for (int i = 1; i <= M; ++i) rp[i] += rp[i - 1];
  {
    std::vector<int> ctr(rp, rp + M + 1);
    for (int i = 0; i < nnz; ++i) {  // stable: input order within a row
      int d = ctr[coo->rows[i]]++;
      cc[d] = coo->cols[i];
      vv[d] = coo->vals[i];
    }
  }
#pragma omp parallel
  {
    std::vector<std::pair<int, int>> tmp;  // (col, position)
    std::vector<float> tv;
#pragma omp for schedule(dynamic, 256)
    for (int r = 0; r < M; ++r) {
      const int s = rp[r], e = rp[r + 1];
      bool sorted = true;
      for (int q = s + 1; q < e; ++q)
        if (cc[q] < cc[q - 1]) { sorted = false; break; }
      if (sorted) continue;
      tmp.resize(e - s);
      tv.resize(e - s);
      for (int q = s; q < e; ++q) tmp[q - s] = {cc[q], q};
      std::stable_sort(tmp.begin(), tmp.end(),
                       [](const std::pair<int, int> &a,
                          const std::pair<int, int> &b) {
                         return a.first < b.first;
                       });
      for (int q = s; q < e; ++q) tv[q - s] = vv[tmp[q - s].second];
      for (int q = s; q < e; ++q) { cc[q] = tmp[q - s].first; vv[q] = tv[q - s]; }
    }
  }
  out->M = M; out->N = N; out->nnz = nnz;
  out->row_ptr = rp; out->col = cc; out->val = vv;
  return VCSR_OK;
}

// ------------------------------------------------------- partitioning

vcsr_status vcsr_partition_rows(const int *row_ptr, int M, int parts, int align,
                                int *cuts) {
  vcsr::clear_error();
  if (!row_ptr || !cuts || M < 0 || parts <= 0 || align <= 0)
    return fail(VCSR_ERR_INVALID, "bad partition arguments");
  const int64_t nnz = row_ptr[M];
  cuts[0] = 0;
  for (int k = 1; k < parts; ++k) {
    const int64_t target = (nnz * k + parts / 2) / parts;
    // first row r with row_ptr[r] >= target
    int lo = 0, hi = M;
    while (lo < hi) {
      int mid = lo + (hi - lo) / 2;
      if (row_ptr[mid] < target) lo = mid + 1; else hi = mid;
    }
    int r = lo;
    if (r > 0 && target - row_ptr[r - 1] < row_ptr[r] - target) r = r - 1;
    int64_t ra = ((int64_t)r + align / 2) / align * align;
    if (ra > M) ra = M;
    if (ra < cuts[k - 1]) ra = cuts[k - 1];
    cuts[k] = (int)ra;
  }
  cuts[parts] = M;
  return VCSR_OK;
}

vcsr_status vcsr_csr_row_panel(const vcsr_csr *csr, int r0, int r1,
                               vcsr_csr *out) {
  vcsr::clear_error();
  if (!csr || !out || r0 < 0 || r1 < r0 || r1 > csr->M)
    return fail(VCSR_ERR_INVALID, "bad row panel [%d, %d)", r0, r1);
  std::memset(out, 0, sizeof *out);
  const int m = r1 - r0;
  const int b = csr->row_ptr[r0], e = csr->row_ptr[r1];
  const int z = e - b;
  out->row_ptr = (int *)malloc(sizeof(int) * ((size_t)m + 1));
  out->col = (int *)malloc(sizeof(int) * (size_t)(z ? z : 1));
  out->val = (float *)malloc(sizeof(float) * (size_t)(z ? z : 1));
  if (!out->row_ptr || !out->col || !out->val) {
    free(out->row_ptr); free(out->col); free(out->val);
    std::memset(out, 0, sizeof *out);
    return fail(VCSR_ERR_ALLOC, "out of host memory");
  }
  for (int i = 0; i <= m; ++i) out->row_ptr[i] = csr->row_ptr[r0 + i] - b;
  if (z) {
    std::memcpy(out->col, csr->col + b, sizeof(int) * (size_t)z);
    std::memcpy(out->val, csr->val + b, sizeof(float) * (size_t)z);
  }
  out->M = m; out->N = csr->N; out->nnz = z;
  return VCSR_OK;
}

}  // extern "C"
