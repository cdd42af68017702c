/*
 * oracle.c — CPU restatement of the MuuSeoTia/VCSR-SPMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product library links, loads or
 * calls this file.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline (the `cpu_baseline` leg and `--impl reference`) use it, and only as
 * the checker / the timed CPU algorithm, never as the measured GPU path.
 *
 * Pinned against the reference itself: tests/golden/ holds outputs of the
 * reference's own include/mmio.hpp, include/csr.hpp and include/vcsr.hpp
 * (compiled from the reference tree by oracle/Makefile into oracle/_ref/),
 * and a GPU test compares oracle_csr_spmm_f32 with the reference's
 * csr_spmm_kernel (src/kernels.cu:15-33) rebuilt for sm_100a.
 *
 * Functions and the reference code they restate:
 *   oracle_read_mtx      include/mmio.hpp:22-45  (read_matrix_market_coo)
 *   oracle_coo_to_csr    include/csr.hpp:16-37   (coo_to_csr)
 *   oracle_csr_spmm_f32  src/kernels.cu:15-33    (csr_spmm_kernel semantics:
 *                        C[r,k] = 0, then C[r,k] += a*B[j,k] in CSR order;
 *                        nvcc contracts the update to one fused multiply-add,
 *                        so the restatement uses fmaf)
 *   oracle_csr_spmm_f64  same order, double accumulation (error budget)
 *   oracle_csr_to_vcsr   include/vcsr.hpp:25-109 (csr_to_vcsr_spmm), with the
 *                        tie order of the per-segment row sort fixed to
 *                        (count descending, row ascending); the reference's
 *                        std::sort leaves ties unspecified.  Memory is
 *                        O(nnz + S + M) instead of the reference's S*M vectors.
 *   oracle_vcsr_spmm     src/kernels.cu:82-101 executed sequentially (group,
 *                        depth, lane, column order), which is the result the
 *                        reference kernel would give without its C data race.
 */
#include <errno.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_OK 0
#define ORC_ERR_IO 4
#define ORC_ERR_RANGE 8
#define ORC_ERR_INVALID 1
#define ORC_ERR_ALLOC 3

static char g_err[512];
const char *oracle_last_error(void) { return g_err; }
static int fail(int code, const char *msg) {
  snprintf(g_err, sizeof g_err, "%s", msg);
  return code;
}

void oracle_free(void *p) { free(p); }

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------ MTX reader */
/* Token reader over a FILE: whitespace-separated like operator>>. */
static int read_token(FILE *f, char *buf, int cap) {
  int c;
  do {
    c = fgetc(f);
  } while (c != EOF && (c == ' ' || c == '\t' || c == '\n' || c == '\r' ||
                        c == '\v' || c == '\f'));
  if (c == EOF) return 0;
  int n = 0;
  while (c != EOF && !(c == ' ' || c == '\t' || c == '\n' || c == '\r' ||
                       c == '\v' || c == '\f')) {
    if (n < cap - 1) buf[n++] = (char)c;
    c = fgetc(f);
  }
  buf[n] = 0;
  return 1;
}

static int parse_int(const char *s, int *out) {
  char *end;
  errno = 0;
  long v = strtol(s, &end, 10);
  if (end == s || *end != 0 || errno || v < -2147483648L || v > 2147483647L)
    return 0;
  *out = (int)v;
  return 1;
}

/* read_matrix_market_coo (include/mmio.hpp:22-45): skip empty and '%' lines,
 * the first other line holds "M N nnz", then nnz triples are read as tokens;
 * 1-based unless the first triple has a zero row or column. */
int oracle_read_mtx(const char *path, int *M, int *N, int *nnz, int **rows,
                    int **cols, float **vals) {
  FILE *f = fopen(path, "r");
  if (!f) return fail(ORC_ERR_IO, "Failed to open MTX");
  char *line = NULL;
  size_t cap = 0;
  ssize_t len;
  int found = 0;
  int m = 0, n = 0, z = 0;
  while ((len = getline(&line, &cap, f)) != -1) {
    /* std::getline strips the '\n' only; an empty line is size 0 */
    if (len > 0 && line[len - 1] == '\n') line[--len] = 0;
    if (len == 0) continue;
    if (line[0] == '%') continue;
    if (sscanf(line, "%d %d %d", &m, &n, &z) != 3) {
      free(line);
      fclose(f);
      return fail(ORC_ERR_IO, "Invalid MTX header or empty file");
    }
    found = 1;
    break;
  }
  free(line);
  if (!found) {
    fclose(f);
    return fail(ORC_ERR_IO, "Invalid MTX header or empty file");
  }
  if (m < 0 || n < 0 || z < 0) {
    fclose(f);
    return fail(ORC_ERR_IO, "Invalid MTX header or empty file");
  }
  int *R = (int *)malloc(sizeof(int) * (size_t)(z ? z : 1));
  int *C = (int *)malloc(sizeof(int) * (size_t)(z ? z : 1));
  float *V = (float *)malloc(sizeof(float) * (size_t)(z ? z : 1));
  if (!R || !C || !V) {
    free(R); free(C); free(V); fclose(f);
    return fail(ORC_ERR_ALLOC, "out of host memory");
  }
  int one_based = 1;
  char tok[256];
  for (int i = 0; i < z; ++i) {
    int r, c;
    char *end;
    if (!read_token(f, tok, sizeof tok) || !parse_int(tok, &r) ||
        !read_token(f, tok, sizeof tok) || !parse_int(tok, &c) ||
        !read_token(f, tok, sizeof tok)) {
      free(R); free(C); free(V); fclose(f);
      return fail(ORC_ERR_IO, "Bad MTX data");
    }
    /* operator>> for double takes [sign] digits [. digits] [e [sign] digits]
     * only (no "inf"/"nan"), and fails on overflow */
    int numeric = 1;
    for (const char *q = tok; *q; ++q)
      if (!((*q >= '0' && *q <= '9') || *q == '.' || *q == '+' || *q == '-' ||
            *q == 'e' || *q == 'E'))
        numeric = 0;
    errno = 0;
    double v = strtod(tok, &end);
    if (!numeric || end == tok || *end != 0 ||
        (errno == ERANGE && (v == HUGE_VAL || v == -HUGE_VAL))) {
      free(R); free(C); free(V); fclose(f);
      return fail(ORC_ERR_IO, "Bad MTX data");
    }
    if (i == 0 && (r == 0 || c == 0)) one_based = 0;
    R[i] = r - (one_based ? 1 : 0);
    C[i] = c - (one_based ? 1 : 0);
    V[i] = (float)v;
  }
  fclose(f);
  *M = m; *N = n; *nnz = z; *rows = R; *cols = C; *vals = V;
  return ORC_OK;
}

/* ---------------------------------------------------------- COO -> CSR */
/* coo_to_csr (include/csr.hpp:16-37): stable counting sort by row, then each
 * row ordered by column (stable for equal columns). */
int oracle_coo_to_csr(int M, int N, int nnz, const int *rows, const int *cols,
                      const float *vals, int **row_ptr_out, int **col_out,
                      float **val_out) {
  (void)N;
  int *rp = (int *)calloc((size_t)M + 1, sizeof(int));
  int *cc = (int *)malloc(sizeof(int) * (size_t)(nnz ? nnz : 1));
  float *vv = (float *)malloc(sizeof(float) * (size_t)(nnz ? nnz : 1));
  int *ctr = (int *)malloc(sizeof(int) * ((size_t)M + 1));
  if (!rp || !cc || !vv || !ctr) {
    free(rp); free(cc); free(vv); free(ctr);
    return fail(ORC_ERR_ALLOC, "out of host memory");
  }
  for (int i = 0; i < nnz; ++i) {
    int r = rows[i];
    if (r < 0 || r >= M) {
      free(rp); free(cc); free(vv); free(ctr);
      return fail(ORC_ERR_RANGE, "row idx out of range");
    }
    rp[r + 1]++;
  }
  for (int i = 1; i <= M; ++i) rp[i] += rp[i - 1];
  memcpy(ctr, rp, sizeof(int) * ((size_t)M + 1));
  for (int i = 0; i < nnz; ++i) {
    int d = ctr[rows[i]]++;
    cc[d] = cols[i];
    vv[d] = vals[i];
  }
  free(ctr);
  /* stable insertion sort per row (rows are short in tests) */
  for (int r = 0; r < M; ++r) {
    for (int p = rp[r] + 1; p < rp[r + 1]; ++p) {
      int c = cc[p];
      float v = vv[p];
      int q = p - 1;
      while (q >= rp[r] && cc[q] > c) {
        cc[q + 1] = cc[q];
        vv[q + 1] = vv[q];
        --q;
      }
      cc[q + 1] = c;
      vv[q + 1] = v;
    }
  }
  *row_ptr_out = rp; *col_out = cc; *val_out = vv;
  return ORC_OK;
}

/* ------------------------------------------------------------- CSR SpMM */
/* csr_spmm_kernel (src/kernels.cu:15-33) semantics, one row per task. */
void oracle_csr_spmm_f32(int M, const int *row_ptr, const int *col,
                         const float *val, const float *B, int64_t ldb, int O,
                         float *C, int64_t ldc, int nthreads) {
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads)
#endif
  for (int r = 0; r < M; ++r) {
    float *Cr = C + (int64_t)r * ldc;
    for (int k = 0; k < O; ++k) Cr[k] = 0.f;
    for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
      const float a = val[p];
      const float *Bj = B + (int64_t)col[p] * ldb;
      for (int k = 0; k < O; ++k) Cr[k] = fmaf(a, Bj[k], Cr[k]);
    }
  }
  (void)nthreads;
}

void oracle_csr_spmm_f64(int M, const int *row_ptr, const int *col,
                         const float *val, const float *B, int64_t ldb, int O,
                         double *C, int64_t ldc, int nthreads) {
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 64) num_threads(nthreads)
#endif
  for (int r = 0; r < M; ++r) {
    double *Cr = C + (int64_t)r * ldc;
    for (int k = 0; k < O; ++k) Cr[k] = 0.0;
    for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
      const double a = val[p];
      const float *Bj = B + (int64_t)col[p] * ldb;
      for (int k = 0; k < O; ++k) Cr[k] += a * (double)Bj[k];
    }
  }
  (void)nthreads;
}

/* ------------------------------------------------------ CSR -> VCSR */
typedef struct {
  int M, N, segw, bundle, num_groups, num_segments;
  int64_t num_slots;
  int *group_ptr, *group_depth, *group_seg_base, *group_rows, *lcol;
  float *val;
  int *segment_group_start;
} oracle_vcsr;

void oracle_vcsr_free(oracle_vcsr *v) {
  free(v->group_ptr); free(v->group_depth); free(v->group_seg_base);
  free(v->group_rows); free(v->lcol); free(v->val);
  free(v->segment_group_start);
  memset(v, 0, sizeof *v);
}

/* csr_to_vcsr_spmm (include/vcsr.hpp:25-109).
 *  - S = ceil(N/segw) segments; an entry of column c goes to segment c/segw
 *    with local column c%segw (vcsr.hpp:28,35-41);
 *  - a (segment,row) entry list keeps column order (vcsr.hpp:43-48);
 *  - per segment, all M rows are ordered by their entry count, descending
 *    (vcsr.hpp:56-59), ties by row ascending (fixed here);
 *  - consecutive chunks of `bundle` rows form groups with depth = the largest
 *    count in the chunk; depth-0 groups are skipped (vcsr.hpp:61-70);
 *  - group metadata and lanes past row M-1 as -1 (vcsr.hpp:72-80);
 *  - slots packed depth-major, lane-minor; missing entries lcol -1, val 0
 *    (vcsr.hpp:82-97). */
int oracle_csr_to_vcsr(int M, int N, const int *row_ptr, const int *col,
                       const float *val, int segw, int bundle,
                       oracle_vcsr *out) {
  memset(out, 0, sizeof *out);
  if (bundle <= 0) return fail(ORC_ERR_INVALID, "bundle must be >0");
  if (segw <= 0) return fail(ORC_ERR_INVALID, "segw must be >0");
  const int S = (N + segw - 1) / segw;
  const int nnz = row_ptr[M];
  /* 1. (row, segment) entry lists: rows' columns are sorted, so a segment's
   *    entries of one row are contiguous. */
  int64_t E = 0;
  for (int r = 0; r < M; ++r)
    for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
      if (col[p] < 0 || col[p] >= N)
        return fail(ORC_ERR_RANGE, "column index out of range");
      if (p > row_ptr[r] && col[p] < col[p - 1])
        return fail(ORC_ERR_INVALID, "CSR row not sorted by column");
      if (p == row_ptr[r] || col[p] / segw != col[p - 1] / segw) ++E;
    }
  int *e_row = (int *)malloc(sizeof(int) * (size_t)(E + 1));
  int *e_seg = (int *)malloc(sizeof(int) * (size_t)(E + 1));
  int *e_start = (int *)malloc(sizeof(int) * (size_t)(E + 1));
  int *e_cnt = (int *)malloc(sizeof(int) * (size_t)(E + 1));
  int *seg_ptr = (int *)calloc((size_t)S + 1, sizeof(int));
  if (!e_row || !e_seg || !e_start || !e_cnt || !seg_ptr) goto oom;
  {
    int64_t e = 0;
    for (int r = 0; r < M; ++r)
      for (int p = row_ptr[r]; p < row_ptr[r + 1]; ++p) {
        if (p == row_ptr[r] || col[p] / segw != col[p - 1] / segw) {
          e_row[e] = r; e_seg[e] = col[p] / segw; e_start[e] = p;
          e_cnt[e] = 0;
          ++e;
        }
        e_cnt[e - 1]++;
      }
  }
  (void)nnz;
  /* 2. stable bucket by segment -> per segment rows ascending */
  for (int64_t e = 0; e < E; ++e) seg_ptr[e_seg[e] + 1]++;
  for (int s = 0; s < S; ++s) seg_ptr[s + 1] += seg_ptr[s];
  int *by_seg = (int *)malloc(sizeof(int) * (size_t)(E + 1));
  int *sorted = (int *)malloc(sizeof(int) * (size_t)(E + 1));
  int *fill = (int *)malloc(sizeof(int) * ((size_t)S + 1));
  if (!by_seg || !sorted || !fill) { free(by_seg); free(sorted); free(fill); goto oom; }
  memcpy(fill, seg_ptr, sizeof(int) * ((size_t)S + 1));
  for (int64_t e = 0; e < E; ++e) by_seg[fill[e_seg[e]]++] = (int)e;
  /* 3. per segment: stable order by count descending */
  int maxc = 0;
  for (int64_t e = 0; e < E; ++e) if (e_cnt[e] > maxc) maxc = e_cnt[e];
  int *cbin = (int *)calloc((size_t)maxc + 2, sizeof(int));
  if (!cbin) { free(by_seg); free(sorted); free(fill); goto oom; }
  int64_t G = 0, P = 0;
  for (int s = 0; s < S; ++s) {
    int b = seg_ptr[s], en = seg_ptr[s + 1];
    memset(cbin, 0, sizeof(int) * ((size_t)maxc + 2));
    for (int i = b; i < en; ++i) cbin[maxc - e_cnt[by_seg[i]] + 1]++;
    for (int c = 0; c <= maxc; ++c) cbin[c + 1] += cbin[c];
    for (int i = b; i < en; ++i) {
      int e = by_seg[i];
      sorted[b + cbin[maxc - e_cnt[e]]++] = e;
    }
    int nz = en - b;
    int ng = (nz + bundle - 1) / bundle;
    G += ng;
    for (int k = 0; k < ng; ++k) P += (int64_t)e_cnt[sorted[b + k * bundle]] * bundle;
  }
  free(cbin);
  if (P > 2147483647LL || G * (int64_t)bundle > 2147483647LL) {
    free(by_seg); free(sorted); free(fill);
    free(e_row); free(e_seg); free(e_start); free(e_cnt); free(seg_ptr);
    return fail(ORC_ERR_INVALID, "VCSR exceeds 32-bit slot indexing");
  }
  out->M = M; out->N = N; out->segw = segw; out->bundle = bundle;
  out->num_groups = (int)G; out->num_segments = S; out->num_slots = P;
  out->group_ptr = (int *)malloc(sizeof(int) * (size_t)(G + 1));
  out->group_depth = (int *)malloc(sizeof(int) * (size_t)(G + 1));
  out->group_seg_base = (int *)malloc(sizeof(int) * (size_t)(G + 1));
  out->group_rows = (int *)malloc(sizeof(int) * (size_t)(G * bundle + 1));
  out->lcol = (int *)malloc(sizeof(int) * (size_t)(P + 1));
  out->val = (float *)malloc(sizeof(float) * (size_t)(P + 1));
  out->segment_group_start = (int *)malloc(sizeof(int) * ((size_t)S + 1));
  if (!out->group_ptr || !out->group_depth || !out->group_seg_base ||
      !out->group_rows || !out->lcol || !out->val || !out->segment_group_start) {
    oracle_vcsr_free(out);
    free(by_seg); free(sorted); free(fill);
    goto oom;
  }
  {
    int64_t g = 0, slot = 0;
    for (int s = 0; s < S; ++s) {
      out->segment_group_start[s] = (int)g;
      int b = seg_ptr[s], en = seg_ptr[s + 1];
      int nz = en - b;
      int ng = (nz + bundle - 1) / bundle;
      /* zero-count rows in ascending order: walk rows against the
       * ascending member list by_seg[b..en) */
      int walk_r = 0, walk_i = b;
      for (int k = 0; k < ng; ++k, ++g) {
        int depth = e_cnt[sorted[b + k * bundle]];
        out->group_ptr[g] = (int)slot;
        out->group_depth[g] = depth;
        out->group_seg_base[g] = s * segw;
        int *rows_g = out->group_rows + g * bundle;
        int *cnt_lane = (int *)malloc(sizeof(int) * (size_t)bundle);
        int *start_lane = (int *)malloc(sizeof(int) * (size_t)bundle);
        if (!cnt_lane || !start_lane) {
          free(cnt_lane); free(start_lane);
          oracle_vcsr_free(out);
          free(by_seg); free(sorted); free(fill);
          goto oom;
        }
        for (int lane = 0; lane < bundle; ++lane) {
          int64_t pos = (int64_t)k * bundle + lane;
          if (pos < nz) {
            int e = sorted[b + pos];
            rows_g[lane] = e_row[e]; cnt_lane[lane] = e_cnt[e];
            start_lane[lane] = e_start[e];
          } else if (pos < M) {
            /* next row (ascending) that has no entry in segment s */
            while (walk_i < en && e_row[by_seg[walk_i]] < walk_r) ++walk_i;
            while (walk_i < en && e_row[by_seg[walk_i]] == walk_r) {
              ++walk_i; ++walk_r;
            }
            rows_g[lane] = walk_r++;
            cnt_lane[lane] = 0; start_lane[lane] = 0;
          } else {
            rows_g[lane] = -1; cnt_lane[lane] = 0; start_lane[lane] = 0;
          }
        }
        for (int d = 0; d < depth; ++d)
          for (int lane = 0; lane < bundle; ++lane, ++slot) {
            if (d < cnt_lane[lane]) {
              int p = start_lane[lane] + d;
              out->lcol[slot] = col[p] - s * segw;
              out->val[slot] = val[p];
            } else {
              out->lcol[slot] = -1;
              out->val[slot] = 0.f;
            }
          }
        free(cnt_lane); free(start_lane);
      }
    }
    out->segment_group_start[S] = (int)g;
    out->group_ptr[G] = (int)slot;
  }
  free(by_seg); free(sorted); free(fill);
  free(e_row); free(e_seg); free(e_start); free(e_cnt); free(seg_ptr);
  return ORC_OK;
oom:
  free(e_row); free(e_seg); free(e_start); free(e_cnt); free(seg_ptr);
  return fail(ORC_ERR_ALLOC, "out of host memory");
}

/* Sequential execution of vcsr_spmm_kernel's update (src/kernels.cu:82-101):
 * C[row][k] += a * B[seg_base+lc][k] for groups, depths, lanes, columns in
 * order.  C is accumulated (the reference caller zeroes it first). */
void oracle_vcsr_spmm(const oracle_vcsr *v, const float *B, int O, float *C) {
  for (int g = 0; g < v->num_groups; ++g) {
    int base = v->group_ptr[g], depth = v->group_depth[g];
    int sb = v->group_seg_base[g];
    for (int d = 0; d < depth; ++d)
      for (int lane = 0; lane < v->bundle; ++lane) {
        int row = v->group_rows[g * v->bundle + lane];
        if (row < 0) continue;
        int idx = base + d * v->bundle + lane;
        int lc = v->lcol[idx];
        if (lc < 0 || lc >= v->segw) continue;
        float a = v->val[idx];
        const float *Bj = B + (int64_t)(sb + lc) * O;
        float *Cr = C + (int64_t)row * O;
        for (int k = 0; k < O; ++k) Cr[k] = fmaf(a, Bj[k], Cr[k]);
      }
  }
}

/* ------------------------------------------------------------ inputs
 * The benchmark's seeded inputs restated for the CPU reference arm, so that
 * arm builds them without loading the engine library: the R-MAT matrix and
 * the dense fill of the engine's generators (vcsr-spmm_b200/csrc/gen.cpp
 * gen_rmat, csrc/memory.cu vcsr_gen_dense).  Random numbers: SplitMix64's
 * output function (Steele, Lea & Flood, OOPSLA 2014) on key + index, with
 * key = mix(seed * 0xD1B54A32D192ED03 ^ mix(stream)).  Pinned bit for bit
 * against the library by tests/test_oracle_golden.py. */
static inline uint64_t og_mix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
static inline uint64_t og_key(uint64_t seed, uint64_t stream) {
  return og_mix(seed * 0xD1B54A32D192ED03ull ^ og_mix(stream));
}
static inline float og_u01f(uint64_t x) {
  return (float)(uint32_t)(x >> 40) * (1.0f / 16777216.0f);
}

/* rows x cols row-major: element i = lo + (hi - lo) * u01(mix(key + i)). */
void oracle_gen_dense(float *out, int64_t rows, int64_t cols, uint64_t seed, float lo,
                      float hi) {
  const uint64_t key = og_key(seed, 0xB0B0ull);
  const int64_t n = rows * cols;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = lo + (hi - lo) * og_u01f(og_mix(key + (uint64_t)i));
}

static int og_cmp_int(const void *a, const void *b) {
  const int x = *(const int *)a, y = *(const int *)b;
  return (x > y) - (x < y);
}

/* R-MAT 2^scale x 2^scale with 16 * 2^scale edges: per edge and level a
 * 16-bit draw picks a quadrant with thresholds (a, a+b, a+b+c) = (.57, .76,
 * .95); duplicates merged, columns ascending, values u01(mix(kv + r*M + c)).
 * Arrays are malloc'd (free with oracle_free).  Returns 0 or -1. */
int oracle_gen_rmat(int scale, uint64_t seed, int *M_out, int **row_ptr, int **col,
                    float **val, int *nnz_out) {
  if (scale < 1 || scale > 28) return fail(-1, "rmat scale out of [1, 28]");
  const int64_t M = (int64_t)1 << scale, E = 16 * M;
  const uint32_t ta = 37355, tb = 49807, tc = 62259;
  const uint64_t ke = og_key(seed, 3), kv = og_key(seed, 2);
  int *er = (int *)malloc(sizeof(int) * (size_t)E), *ec = (int *)malloc(sizeof(int) * (size_t)E);
  int *cnt = (int *)calloc((size_t)M + 1, sizeof(int));
  int64_t *start = (int64_t *)malloc(sizeof(int64_t) * ((size_t)M + 1));
  int *bucket = (int *)malloc(sizeof(int) * (size_t)E);
  int64_t *uniq = (int64_t *)malloc(sizeof(int64_t) * ((size_t)M + 1));
  if (!er || !ec || !cnt || !start || !bucket || !uniq) {
    free(er); free(ec); free(cnt); free(start); free(bucket); free(uniq);
    return fail(-1, "out of host memory");
  }
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < E; ++e) {
    uint32_t r = 0, c = 0;
    uint64_t bits = 0;
    for (int l = 0; l < scale; ++l) {
      if ((l & 3) == 0) bits = og_mix(ke + (uint64_t)e * 8 + (uint64_t)(l >> 2));
      const uint32_t u = (uint32_t)(bits & 0xFFFF);
      bits >>= 16;
      r = (r << 1) | (u >= tb ? 1u : 0u);
      c = (c << 1) | (((u >= ta && u < tb) || u >= tc) ? 1u : 0u);
    }
    er[e] = (int)r;
    ec[e] = (int)c;
  }
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < E; ++e) __atomic_fetch_add(&cnt[er[e] + 1], 1, __ATOMIC_RELAXED);
  start[0] = 0;
  for (int64_t r = 0; r < M; ++r) start[r + 1] = start[r] + cnt[r + 1];
  memset(cnt, 0, sizeof(int) * ((size_t)M + 1));
#pragma omp parallel for schedule(static)
  for (int64_t e = 0; e < E; ++e) {
    const int r = er[e];
    const int pos = __atomic_fetch_add(&cnt[r], 1, __ATOMIC_RELAXED);
    bucket[start[r] + pos] = ec[e];
  }
  free(er);
  free(ec);
  uniq[0] = 0;
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t r = 0; r < M; ++r) {
    int *b = bucket + start[r];
    const int64_t n = start[r + 1] - start[r];
    qsort(b, (size_t)n, sizeof(int), og_cmp_int);
    int64_t u = 0;
    for (int64_t i = 0; i < n; ++i)
      if (i == 0 || b[i] != b[i - 1]) b[u++] = b[i];
    uniq[r + 1] = u;
  }
  for (int64_t r = 0; r < M; ++r) uniq[r + 1] += uniq[r];
  if (uniq[M] > INT32_MAX) {
    free(cnt); free(start); free(bucket); free(uniq);
    return fail(-1, "rmat nnz exceeds int32");
  }
  const int nnz = (int)uniq[M];
  int *rp = (int *)malloc(sizeof(int) * ((size_t)M + 1));
  int *cc = (int *)malloc(sizeof(int) * (size_t)(nnz ? nnz : 1));
  float *vv = (float *)malloc(sizeof(float) * (size_t)(nnz ? nnz : 1));
  if (!rp || !cc || !vv) {
    free(rp); free(cc); free(vv); free(cnt); free(start); free(bucket); free(uniq);
    return fail(-1, "out of host memory");
  }
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t r = 0; r < M; ++r) {
    rp[r] = (int)uniq[r];
    for (int64_t t = 0; t < uniq[r + 1] - uniq[r]; ++t) {
      const int c = bucket[start[r] + t];
      cc[uniq[r] + t] = c;
      vv[uniq[r] + t] = og_u01f(og_mix(kv + (uint64_t)r * (uint64_t)M + (uint64_t)c));
    }
  }
  rp[M] = nnz;
  free(cnt); free(start); free(bucket); free(uniq);
  *M_out = (int)M;
  *row_ptr = rp;
  *col = cc;
  *val = vv;
  *nnz_out = nnz;
  return 0;
}
