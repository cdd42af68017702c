// host_io.cpp — host-side input surface: errors, Matrix Market reader,
// COO -> CSR, container frees, row panels and the nnz-balanced partitioner.
//
// vcsr_read_mtx follows read_matrix_market_coo (include/mmio.hpp:22-45) and
// vcsr_coo_to_csr follows coo_to_csr (include/csr.hpp:16-37); both are
// rewritten for speed (one buffered read, a multi-threaded per-row sort).
#include <algorithm>
#include <cerrno>
#include <charconv>
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
  return vcsr::no_throw([&]() -> vcsr_status {
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
  });
}

// --------------------------------------------- MTX reader with the banner

namespace {

struct MtxBanner {
  bool pattern = false, complex_ = false, integer = false;
  int symmetry = 0;  // 0 general, 1 symmetric, 2 skew-symmetric, 3 hermitian
};

bool ieq(const std::string &a, const char *b) {
  size_t n = strlen(b);
  if (a.size() != n) return false;
  for (size_t i = 0; i < n; ++i)
    if (tolower((unsigned char)a[i]) != b[i]) return false;
  return true;
}

// One data line: "r c [v [im]]" -> (r, c, v); false when malformed.
bool parse_entry(const char *b, const char *e, const MtxBanner &mb, long long &r, long long &c,
                 double &v) {
  auto skip = [&](const char *q) {
    while (q < e && is_space(*q)) ++q;
    return q;
  };
  const char *q = skip(b);
  auto ri = std::from_chars(q, e, r);
  if (ri.ec != std::errc() || ri.ptr == q) return false;
  q = skip(ri.ptr);
  auto ci = std::from_chars(q, e, c);
  if (ci.ec != std::errc() || ci.ptr == q) return false;
  q = skip(ci.ptr);
  if (mb.pattern) {
    v = 1.0;
  } else {
    if (*q == '+') ++q;  // from_chars takes no leading '+'
    auto vi = std::from_chars(q, e, v);
    if (vi.ec != std::errc() || vi.ptr == q) return false;
    q = vi.ptr;
    if (mb.complex_) {  // the imaginary part is read and dropped
      q = skip(q);
      if (*q == '+') ++q;
      double im;
      auto ii = std::from_chars(q, e, im);
      if (ii.ec != std::errc() || ii.ptr == q) return false;
      q = ii.ptr;
    }
  }
  return skip(q) == e;
}

}  // namespace

vcsr_status vcsr_read_mtx_ex(const char *path, int flags, vcsr_coo *out) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!path || !out) return fail(VCSR_ERR_INVALID, "null argument");
    if (!(flags & VCSR_MTX_BANNER)) return vcsr_read_mtx(path, out);
    std::memset(out, 0, sizeof *out);
    FILE *f = fopen(path, "rb");
    if (!f) return fail(VCSR_ERR_IO, "Failed to open MTX: %s", path);
    std::string buf;
    if (fseek(f, 0, SEEK_END) == 0) {
      long sz = ftell(f);
      if (sz > 0) buf.resize((size_t)sz);
      fseek(f, 0, SEEK_SET);
      if (sz > 0 && fread(&buf[0], 1, (size_t)sz, f) != (size_t)sz) {
        fclose(f);
        return fail(VCSR_ERR_IO, "Failed to read MTX: %s", path);
      }
    }
    fclose(f);
    const char *p = buf.data(), *end = p + buf.size();
    // banner: %%MatrixMarket matrix coordinate <field> <symmetry>
    MtxBanner mb;
    {
      const char *eol = (const char *)memchr(p, '\n', end - p);
      if (!eol) eol = end;
      std::string line(p, eol);
      char w[5][64] = {{0}};
      if (line.compare(0, 14, "%%MatrixMarket") != 0 ||
          sscanf(line.c_str(), "%63s %63s %63s %63s %63s", w[0], w[1], w[2], w[3], w[4]) != 5)
        return fail(VCSR_ERR_IO, "missing %%%%MatrixMarket banner");
      if (!ieq(w[1], "matrix")) return fail(VCSR_ERR_UNSUPPORTED, "MTX object '%s'", w[1]);
      if (!ieq(w[2], "coordinate"))
        return fail(VCSR_ERR_UNSUPPORTED, "MTX format '%s' (only coordinate)", w[2]);
      const std::string field = w[3], sym = w[4];
      if (ieq(field, "pattern")) mb.pattern = true;
      else if (ieq(field, "complex")) mb.complex_ = true;
      else if (ieq(field, "integer")) mb.integer = true;
      else if (!ieq(field, "real") && !ieq(field, "double"))
        return fail(VCSR_ERR_UNSUPPORTED, "MTX field '%s'", w[3]);
      if (ieq(sym, "general")) mb.symmetry = 0;
      else if (ieq(sym, "symmetric")) mb.symmetry = 1;
      else if (ieq(sym, "skew-symmetric")) mb.symmetry = 2;
      else if (ieq(sym, "hermitian")) mb.symmetry = 3;
      else return fail(VCSR_ERR_UNSUPPORTED, "MTX symmetry '%s'", w[4]);
      p = eol < end ? eol + 1 : end;
    }
    // size line: first line that is neither empty nor a comment
    long long M = -1, N = -1, Z = -1;
    bool found = false;
    while (p < end) {
      const char *eol = (const char *)memchr(p, '\n', end - p);
      if (!eol) eol = end;
      const char *q = p;
      while (q < eol && is_space(*q)) ++q;
      if (q < eol && *q != '%') {
        std::string line(q, eol);
        if (sscanf(line.c_str(), "%lld %lld %lld", &M, &N, &Z) != 3)
          return fail(VCSR_ERR_IO, "Invalid MTX size line");
        p = eol < end ? eol + 1 : end;
        found = true;
        break;
      }
      p = eol < end ? eol + 1 : end;
    }
    if (!found || M < 0 || N < 0 || Z < 0) return fail(VCSR_ERR_IO, "Invalid MTX size line");
    if (M > INT32_MAX || N > INT32_MAX || Z > INT32_MAX)
      return fail(VCSR_ERR_UNSUPPORTED, "MTX dimensions exceed 32-bit indexing");
    if (mb.symmetry && M != N) return fail(VCSR_ERR_IO, "symmetric MTX must be square");
    // data lines (one entry per line, blank and '%' lines skipped), parsed in
    // parallel chunks; each entry is followed by its mirror when the banner
    // says the file holds one triangle
    std::vector<const char *> ls;  // starts of non-empty, non-comment lines
    ls.reserve((size_t)Z + 1);
    while (p < end) {
      const char *eol = (const char *)memchr(p, '\n', end - p);
      if (!eol) eol = end;
      const char *q = p;
      while (q < eol && is_space(*q)) ++q;
      if (q < eol && *q != '%') ls.push_back(p);
      p = eol < end ? eol + 1 : end;
    }
    if ((long long)ls.size() != Z)
      return fail(VCSR_ERR_IO, "MTX has %zu entries, size line says %lld", ls.size(), Z);
    const int T = std::max(1, std::min(omp_get_max_threads(), (int)(Z / 65536) + 1));
    std::vector<long long> cnt(T + 1, 0);
    std::vector<int> bad(T, 0);
    std::vector<unsigned char> mirror((size_t)Z, 0);
    std::vector<int> rr((size_t)Z), cc((size_t)Z);
    std::vector<float> vv((size_t)Z);
  #pragma omp parallel num_threads(T)
    {
      const int t = omp_get_thread_num();
      const long long i0 = Z * t / T, i1 = Z * (t + 1) / T;
      long long extra = 0;
      for (long long i = i0; i < i1; ++i) {
        const char *b = ls[(size_t)i];
        const char *eol = (const char *)memchr(b, '\n', end - b);
        if (!eol) eol = end;
        long long r, c;
        double v;
        if (!parse_entry(b, eol, mb, r, c, v) || r < 1 || c < 1 || r > M || c > N) {
          bad[t] = 1;
          break;
        }
        rr[(size_t)i] = (int)(r - 1);
        cc[(size_t)i] = (int)(c - 1);
        vv[(size_t)i] = (float)v;
        if (mb.symmetry && r != c) {
          mirror[(size_t)i] = 1;
          ++extra;
        }
      }
      cnt[t + 1] = (i1 - i0) + extra;
    }
    for (int t = 0; t < T; ++t)
      if (bad[t]) return fail(VCSR_ERR_IO, "Bad MTX data");
    for (int t = 0; t < T; ++t) cnt[t + 1] += cnt[t];
    const long long total = cnt[T];
    if (total > INT32_MAX) return fail(VCSR_ERR_UNSUPPORTED, "expanded nnz exceeds 32 bits");
    int *R = (int *)malloc(sizeof(int) * (size_t)(total ? total : 1));
    int *C = (int *)malloc(sizeof(int) * (size_t)(total ? total : 1));
    float *V = (float *)malloc(sizeof(float) * (size_t)(total ? total : 1));
    if (!R || !C || !V) {
      free(R); free(C); free(V);
      return fail(VCSR_ERR_ALLOC, "out of host memory");
    }
    const float sign = mb.symmetry == 2 ? -1.f : 1.f;
  #pragma omp parallel num_threads(T)
    {
      const int t = omp_get_thread_num();
      const long long i0 = Z * t / T, i1 = Z * (t + 1) / T;
      long long o = cnt[t];
      for (long long i = i0; i < i1; ++i) {
        R[o] = rr[(size_t)i]; C[o] = cc[(size_t)i]; V[o] = vv[(size_t)i]; ++o;
        if (mirror[(size_t)i]) {
          R[o] = cc[(size_t)i]; C[o] = rr[(size_t)i]; V[o] = sign * vv[(size_t)i]; ++o;
        }
      }
    }
    out->M = (int)M; out->N = (int)N; out->nnz = (int)total;
    out->rows = R; out->cols = C; out->vals = V;
    return VCSR_OK;
  });
}

// ------------------------------------------------------------ COO -> CSR

vcsr_status vcsr_coo_to_csr(const vcsr_coo *coo, vcsr_csr *out) {
  return vcsr::no_throw([&]() -> vcsr_status {
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
  });
}

// ------------------------------------------------------- partitioning

vcsr_status vcsr_partition_rows_weighted(const int *row_ptr, int M, int parts, int align,
                                         double row_weight, int *cuts) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!row_ptr || !cuts || M < 0 || parts <= 0 || align <= 0 || !(row_weight >= 0))
      return fail(VCSR_ERR_INVALID, "bad partition arguments");
    // cost of rows [0, r): row_ptr[r] + row_weight * r, non-decreasing in r
    auto cost = [&](int r) { return (double)row_ptr[r] + row_weight * r; };
    const double total = cost(M);
    cuts[0] = 0;
    for (int k = 1; k < parts; ++k) {
      const double target = total * k / parts;
      int lo = 0, hi = M;  // first row r with cost(r) >= target
      while (lo < hi) {
        int mid = lo + (hi - lo) / 2;
        if (cost(mid) < target) lo = mid + 1; else hi = mid;
      }
      int r = lo;
      if (r > 0 && target - cost(r - 1) < cost(r) - target) r = r - 1;
      int64_t ra = ((int64_t)r + align / 2) / align * align;
      if (ra > M) ra = M;
      if (ra < cuts[k - 1]) ra = cuts[k - 1];
      cuts[k] = (int)ra;
    }
    cuts[parts] = M;
    return VCSR_OK;
  });
}

vcsr_status vcsr_partition_rows(const int *row_ptr, int M, int parts, int align,
                                int *cuts) {
  return vcsr_partition_rows_weighted(row_ptr, M, parts, align, 0.0, cuts);
}

vcsr_status vcsr_csr_row_panel(const vcsr_csr *csr, int r0, int r1,
                               vcsr_csr *out) {
  return vcsr::no_throw([&]() -> vcsr_status {
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
  });
}

}  // extern "C"
