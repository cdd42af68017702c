/*
 * vcsr_spmm.h — C ABI of the B200 (sm_100a) VCSR SpMM engine.
 *
 * One job: C[M x O] = A[M x N, sparse] * B[N x O, dense row-major], FP32.
 *
 * Every entry point is extern "C", takes plain pointers and sizes and returns a
 * vcsr_status.  No entry point exits the process; on failure the thread-local
 * message behind vcsr_last_error() says what went wrong.  All device work is
 * enqueued on the caller's stream (a cudaStream_t passed as void*, NULL = the
 * legacy default stream) with no implicit device synchronisation, except where
 * an entry point says it synchronises.
 *
 * Reference interfaces each group replaces are cited as file:line inside the
 * MuuSeoTia/VCSR-SPMM tree.
 */
#ifndef VCSR_SPMM_H
#define VCSR_SPMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VCSR_ABI_VERSION 3

typedef void *vcsr_stream_t; /* a cudaStream_t */

typedef enum vcsr_status {
  VCSR_OK = 0,
  VCSR_ERR_INVALID = 1,     /* bad argument / malformed input */
  VCSR_ERR_CUDA = 2,        /* a CUDA runtime/driver call failed */
  VCSR_ERR_ALLOC = 3,       /* host or device allocation failed */
  VCSR_ERR_IO = 4,          /* file could not be opened / parsed */
  VCSR_ERR_UNSUPPORTED = 5, /* valid request this build cannot serve */
  VCSR_ERR_NCCL = 6,        /* an NCCL call failed */
  VCSR_ERR_TIMEOUT = 7,     /* a bounded wait ran out */
  VCSR_ERR_RANGE = 8        /* index out of range (e.g. COO row >= M) */
} vcsr_status;

/* Where a structure's arrays live. */
#define VCSR_HOST 0
#define VCSR_DEVICE 1

/* ------------------------------------------------------------------ errors */

/* Thread-local text of the last failure (never NULL; "" when none). */
const char *vcsr_last_error(void);
const char *vcsr_status_string(vcsr_status s);
int vcsr_abi_version(void);

/* ------------------------------------------------------- matrix containers */

/* COO triplets; replaces struct COO (include/mmio.hpp:15-19). */
typedef struct vcsr_coo {
  int M, N;
  int nnz;
  int *rows; /* 0-based */
  int *cols; /* 0-based */
  float *vals;
} vcsr_coo;

/* CSR; replaces struct CSR (include/csr.hpp:8-13).  row_ptr has M+1 entries. */
typedef struct vcsr_csr {
  int M, N, nnz;
  int *row_ptr;
  int *col;
  float *val;
} vcsr_csr;

/* Segment-major VCSR; field for field struct VCSRSpMM (include/vcsr.hpp:12-23).
 * num_groups = G, num_slots = P = group_ptr[G].  group_rows has G*bundle
 * entries (-1 pads lanes past row M-1), lcol/val have P entries (lcol -1 and
 * val 0 mark padding slots).  Slot of (group g, depth d, lane l) is
 * group_ptr[g] + d*bundle + l.  segment_group_start (S+1 entries, S =
 * ceil(N/segw)) gives the first group of each column segment (the
 * VCSRSeg::segment_group_start of src/vcsr_seg.cu:21,53,109). */
typedef struct vcsr_vcsr {
  int M, N, segw, bundle;
  int num_groups;
  int num_segments;
  int64_t num_slots;
  int *group_ptr;
  int *group_depth;
  int *group_seg_base;
  int *group_rows;
  int *lcol;
  float *val;
  int *segment_group_start;
} vcsr_vcsr;

void vcsr_coo_free(vcsr_coo *coo);          /* host arrays from this library */
void vcsr_csr_free(vcsr_csr *csr, int where);
void vcsr_vcsr_free(vcsr_vcsr *v, int where);

/* --------------------------------------------------------- host-side input */

/* Matrix Market reader; replaces read_matrix_market_coo (include/mmio.hpp:22-45).
 * Same semantics: '%' lines and empty lines before the size line are skipped,
 * the size line gives M N nnz, then nnz "r c v" triples follow as
 * whitespace-separated tokens; indices are 1-based unless the first triple has
 * a 0 row or column; values are read as double and stored as float; no
 * symmetric expansion; duplicates kept.  Errors: VCSR_ERR_IO for an unopenable
 * file, a missing size line or a short/garbled data section. */
vcsr_status vcsr_read_mtx(const char *path, vcsr_coo *out);

/* Options of vcsr_read_mtx_ex. */
#define VCSR_MTX_BANNER 1 /* read the %%MatrixMarket banner and follow the standard */

/* Matrix Market reader that follows the format's banner (no counterpart in
 * the reference, whose reader ignores it: include/mmio.hpp:22-45).  Without
 * VCSR_MTX_BANNER it is vcsr_read_mtx.  With it: the first line must be
 * "%%MatrixMarket matrix coordinate <field> <symmetry>"; indices are 1-based;
 * one entry per line; field real/double/integer as values, pattern entries
 * get 1, complex keeps the real part; symmetry symmetric / skew-symmetric /
 * hermitian stores one triangle and every off-diagonal entry is followed by
 * its mirror (negated for skew-symmetric, the real part for hermitian).
 * Entries keep file order.  Lines are parsed by all host threads.  Errors:
 * VCSR_ERR_IO (no banner, bad size line, wrong entry count, bad entry or
 * index out of range), VCSR_ERR_UNSUPPORTED (array format, other objects,
 * unknown field or symmetry). */
vcsr_status vcsr_read_mtx_ex(const char *path, int flags, vcsr_coo *out);

/* COO -> CSR; replaces coo_to_csr (include/csr.hpp:16-37).  Rows are placed by
 * a stable counting sort, then each row's entries are ordered by column; equal
 * columns keep input order.  A row index outside [0,M) is VCSR_ERR_RANGE like
 * the reference's "row idx out of range"; a column outside [0,N) is also
 * rejected (the reference leaves it unchecked). */
vcsr_status vcsr_coo_to_csr(const vcsr_coo *coo, vcsr_csr *out);

/* Deterministic synthetic matrices (host, multi-threaded).  config is one of
 * "uniform", "fem", "powerlaw", "rmat", "blockdense"; size_param overrides the
 * config's row count (0 = the configured size; for "rmat" it is the scale,
 * log2 of the row count).  The same (config, seed, size_param) always gives
 * the same CSR, bit for bit. */
vcsr_status vcsr_gen_csr(const char *config, uint64_t seed, int size_param,
                         vcsr_csr *out);

/* Fill a rows x cols row-major matrix (leading dimension ld) with values
 * lo + (hi-lo)*u, u a 24-bit uniform drawn from (seed, element index).  Host
 * and device fills give identical bits.  where = VCSR_HOST | VCSR_DEVICE. */
vcsr_status vcsr_gen_dense(float *out, int64_t rows, int64_t cols, int64_t ld,
                           uint64_t seed, float lo, float hi, int where,
                           vcsr_stream_t stream);

/* Copy a CSR between host and device (dst arrays allocated by the library). */
vcsr_status vcsr_csr_to_device(const vcsr_csr *host, vcsr_csr *dev,
                               vcsr_stream_t stream);

/* ------------------------------------------------ VCSR format construction */

/* Build the segment-major VCSR of a device-resident CSR on the GPU (segmented
 * scan, stable radix sort, pack); replaces csr_to_vcsr_spmm
 * (include/vcsr.hpp:25-109).  Output arrays are device allocations owned by
 * *out (free with vcsr_vcsr_free(out, VCSR_DEVICE)).  Rows inside a segment
 * are ordered by per-segment count descending and, on ties, by row ascending
 * (the reference's std::sort leaves tie order unspecified). Synchronises the
 * stream once to size the outputs. */
vcsr_status vcsr_build_vcsr(const vcsr_csr *dev_csr, int segw, int bundle,
                            vcsr_vcsr *out, vcsr_stream_t stream);

/* Copy a device VCSR to host arrays (allocated by the library). */
vcsr_status vcsr_vcsr_to_host(const vcsr_vcsr *dev, vcsr_vcsr *host);

/* ------------------------------------------------------------- SpMM plans */

typedef struct vcsr_plan vcsr_plan;

#define VCSR_PLAN_REFERENCE_FORMAT 1 /* also keep the segment-major VCSR */
/* Run dense 16x16 blocks of A (>= panel_min_nnz entries) on the tensor cores
 * in TF32 (tcgen05.mma kind::tf32, FP32 accumulation): the reference's
 * tensor-core variant (src/vcsr_tc.cu:122-195, FP16 WMMA) on B200.  Results
 * then match the FP32 CSR sum to about 1e-3 relative L2 instead of 1e-5.
 * Needs O and ldb multiples of 4 and a 16-byte aligned B at call time
 * (VCSR_ERR_UNSUPPORTED otherwise). */
#define VCSR_PLAN_TF32_PANELS 2
/* Build the plan's layout on the host (OpenMP) instead of with the GPU
 * kernels that build it by default.  The layout is the same, bit for bit;
 * the flag exists to check the GPU builder against the host one. */
#define VCSR_PLAN_HOST_BUILD 4
/* Run A's column runs on the tensor cores at FP32 accuracy: every 16 rows
 * (a row block) the union of their columns is cut into runs of consecutive
 * columns, each run's B rows come into shared memory by TMA (the
 * reference's B-tile-per-segment idea, src/kernels.cu:37-103), and
 * tcgen05.mma kind::tf32 multiplies them by the row block's dense values with
 * every value split into a TF32 high part and a TF32 remainder (three MMAs
 * per step): results within about 1e-6 relative L2 of the CSR sum, and any
 * output left non-finite is recomputed as the CSR sum is.  Runs shorter
 * than seg_min_run columns stay on the FP32 kernel.  Pays where rows come
 * in runs of consecutive columns (banded FEM matrices, dense blocks).
 * Needs O and ldb multiples of 4 and a 16-byte aligned B at call time;
 * built on the GPU only; excludes VCSR_PLAN_TF32_PANELS. */
#define VCSR_PLAN_TC_SEGMENTS 8

typedef struct vcsr_plan_params {
  int segw;     /* column segment width (--segw) */
  int bundle;   /* rows per VCSR group (--bundle) */
  int tileK;    /* O columns per tile (--tileK); 0 = choose per call */
  int max_O;    /* largest O the plan will serve; sizes split-row scratch */
  int vec_rows; /* rows per panel vector: 0 = choose from the pattern,
                   else 1, 2, 4, 8 or 16 */
  int chunk;    /* max union columns per work unit; 0 = choose */
  int flags;    /* VCSR_PLAN_* */
  int panel_min_nnz; /* entries that make a 16x16 block a TF32 panel
                        (1..256; 0 = 128) */
  int target_O; /* the O the plan will mostly serve (0 = not given); with
                   vec_rows = 0 and target_O > 128 an 8-row choice becomes 4
                   rows (wider O: an 8-row vector's sums take 64 registers per
                   lane; measured 13-16% faster on FEM at O >= 192) */
  int seg_min_run; /* VCSR_PLAN_TC_SEGMENTS: shortest column run on the tensor
                      cores (0 = choose: runs under 8 columns are padded to 8
                      while their padded rows stay below M, else left to the
                      FP32 kernel) */
} vcsr_plan_params;

typedef struct vcsr_plan_info {
  int M, N, nnz;
  int vec_rows;       /* chosen rows per panel vector */
  int num_vectors;    /* ceil(M / vec_rows) */
  int64_t num_union;  /* union columns over all vectors */
  int num_units;      /* nnz-balanced work units */
  int num_split_vectors;
  int num_split_units;
  int num_long_units;  /* units walked by a whole warp (>= 128 union columns) */
  int64_t panel_bytes; /* device bytes of the panel layout */
  int has_reference_format;
  double build_ms;    /* wall time of vcsr_plan_create */
  int num_panel_blocks;     /* dense 16x16 blocks on the TF32 path */
  int num_panel_row_blocks; /* row blocks holding them */
  int64_t panel_nnz;        /* entries of A on the tensor cores */
  int num_seg_row_blocks;   /* VCSR_PLAN_TC_SEGMENTS: row blocks with runs */
  int num_seg_pieces;       /* pieces of at most 32 columns */
  int64_t seg_rows;         /* B rows the pieces read (padding included) */
  int seg_only;             /* 1: no residual; the segment kernel writes C alone */
} vcsr_plan_info;

void vcsr_plan_params_default(vcsr_plan_params *p);

/* Build a plan for A.  csr_where = VCSR_HOST or VCSR_DEVICE.  The plan owns
 * every device array it needs; the caller's CSR may be freed afterwards.
 * Replaces the format build + upload half of run_vcsr_spmm_gpu
 * (src/kernels.cu:120-151), done once instead of per call. */
vcsr_status vcsr_plan_create(const vcsr_csr *csr, int csr_where,
                             const vcsr_plan_params *params, vcsr_plan **out,
                             vcsr_stream_t stream);
/* Build a plan for the matrix a segment-major VCSR holds (the reference's
 * VCSRSpMM, include/vcsr.hpp:12-23, as host or device arrays by `where`):
 * the slots with a row >= 0 and an lcol >= 0 become entries (row, column
 * group_seg_base + lcol, value) on the GPU, rows in slot order, and the plan
 * is built from them as vcsr_plan_create builds a device CSR.  This lets a
 * caller of the reference's launcher, which receives this format
 * (src/kernels.cu:120-167), run the engine.  Errors: VCSR_ERR_INVALID when
 * group_ptr does not match group_depth * bundle and num_slots or a segment
 * base is outside [0, N); VCSR_ERR_RANGE for a row outside [-1, M) or an
 * lcol outside [-1, segw) or past column N. */
vcsr_status vcsr_plan_from_vcsr(const vcsr_vcsr *v, int where, const vcsr_plan_params *params,
                                vcsr_plan **out, vcsr_stream_t stream);
vcsr_status vcsr_plan_get_info(const vcsr_plan *plan, vcsr_plan_info *info);
/* Host copy of the plan's segment-major VCSR (needs VCSR_PLAN_REFERENCE_FORMAT). */
vcsr_status vcsr_plan_export(const vcsr_plan *plan, vcsr_vcsr *host_out);
void vcsr_plan_destroy(vcsr_plan *plan);

/* Plans on disk, so that a matrix's layout is built once.  vcsr_plan_save
 * writes every array the plan holds (and the segment-major VCSR when the plan
 * keeps it) with a checksum; vcsr_plan_load reads such a file onto the
 * current device, on `stream`.  The load checks the checksum, the sizes and
 * every index the kernels follow before it allocates anything on the device:
 * VCSR_ERR_IO for a missing, damaged or inconsistent file,
 * VCSR_ERR_UNSUPPORTED for another file version.  The reference rebuilds its
 * format on every run (src/main.cpp:113-118); no counterpart there. */
vcsr_status vcsr_plan_save(const vcsr_plan *plan, const char *path);
vcsr_status vcsr_plan_load(const char *path, vcsr_plan **out, vcsr_stream_t stream);

/* C = A * B (C written, not accumulated: beta = 0 semantics, the zeroing the
 * reference does with cudaMemset is fused).  B is N x O with leading dimension
 * ldb >= O, C is M x O with ldc >= O, both device pointers.  Replaces the
 * launch half of run_vcsr_spmm_gpu (src/kernels.cu:153-160); timing is left to
 * the caller.  Calls on one plan must not overlap on the GPU (split rows share
 * the plan's scratch).  Reports the kernel launches it made through
 * *launches when launches != NULL. */
vcsr_status vcsr_spmm(const vcsr_plan *plan, const float *dB, int ldb,
                      float *dC, int ldc, int O, vcsr_stream_t stream,
                      int *launches);
/* C += A * B: vcsr_spmm's product added into C, the contract of the
 * reference's launcher (src/kernels.cu:120-167, whose kernel adds into a C
 * the caller zeroed).  Each value of C is read and written once, by one
 * thread (no atomics: the result does not depend on the schedule); rows of A
 * without entries leave C as it was.  Same other rules as vcsr_spmm. */
vcsr_status vcsr_spmm_accumulate(const vcsr_plan *plan, const float *dB, int ldb,
                                 float *dC, int ldc, int O, vcsr_stream_t stream,
                                 int *launches);

/* Row panels of a plan (about equal nnz; at most 8), for callers that
 * schedule the product themselves, e.g. behind a chunked broadcast of B: on
 * input *count is the length of the arrays (any may be NULL; all NULL asks
 * only for the count), on output the number of panels; panel j covers rows
 * [row0[j], row1[j]) and reads B rows up to col_max[j] (-1: no entries).
 * Plans with TF32 panels and small plans (M < 8192 or nnz < 2^20) have
 * none.  No counterpart in the reference. */
vcsr_status vcsr_plan_row_panels(const vcsr_plan *plan, int *count, int *row0, int *row1,
                                 int *col_max);
/* C rows of one row panel: C[row0[j]:row1[j]) = A[those rows] * B, with the
 * contract of vcsr_spmm (the other rows of C are not touched).  The panels
 * together are vcsr_spmm. */
vcsr_status vcsr_spmm_row_panel(const vcsr_plan *plan, int panel, const float *dB, int ldb,
                                float *dC, int ldc, int O, vcsr_stream_t stream,
                                int *launches);

/* C = A * B with B in BF16 (bfloat16 bits, N x O, leading dimension ldb);
 * each B value is widened to FP32 as it is loaded (exact) and the sums are the
 * FP32 path's, so C equals, bit for bit, vcsr_spmm on the widened B.  B traffic
 * is half of FP32's (gather-bound matrices such as R-MAT gain most).  Not for
 * plans with TF32 panels (VCSR_ERR_UNSUPPORTED); same other rules as
 * vcsr_spmm.  The reference's only reduced-precision path is its FP16 WMMA
 * kernel (src/vcsr_tc.cu); no direct counterpart. */
vcsr_status vcsr_spmm_bf16(const vcsr_plan *plan, const void *dB, int ldb,
                           float *dC, int ldc, int O, vcsr_stream_t stream,
                           int *launches);

/* The same with B in FP16 (IEEE binary16 bits): each value is widened to FP32
 * as it is loaded (exact, subnormals included), FP32 sums, so C equals, bit for
 * bit, vcsr_spmm on the widened B.  Same rules as vcsr_spmm_bf16.  The
 * reference's FP16 kernel (src/vcsr_tc.cu:122-195) rounds A to FP16 as well
 * and sums on the tensor cores; this one keeps A in FP32. */
vcsr_status vcsr_spmm_f16(const vcsr_plan *plan, const void *dB, int ldb,
                          float *dC, int ldc, int O, vcsr_stream_t stream,
                          int *launches);

/* The same product with host buffers: copies hB (N x O, ld = O) to the device,
 * runs vcsr_spmm, copies C back to hC (M x O, ld = O) and synchronises the
 * stream.  Replaces the upload/launch/download sequence of the reference's
 * main (src/main.cpp:104-161) as one call.  With more than 8 MB of B and C
 * the transfers overlap the work: for banded matrices (no row panel reads B
 * rows beyond the next 1/8 of B) B goes up in row chunks cut at the highest
 * column of each row panel, each row panel runs as soon as its chunk is on
 * the device and its C rows come back while later chunks go up; otherwise,
 * with O >= 128, up to four column
 * chunks form the pipeline (chunk k comes back while chunk k+1 goes up).
 * Downloads and products run on plan-owned streams; the call returns after
 * all of them.  Host buffers should be pinned for full PCIe speed and for
 * the overlap. */
vcsr_status vcsr_spmm_host(vcsr_plan *plan, const float *hB, float *hC, int O,
                           vcsr_stream_t stream);

/* Rows vcsr_spmm_host moves across PCIe per call when hB and hC are
 * page-locked and 64-byte aligned, O is a multiple of 16 and B and C exceed
 * 8 MB: *b_rows B rows up and *c_rows C rows down.  A product reads only the
 * B rows of columns that hold an entry, and only the C rows that hold an
 * entry are non-zero; when these lists save more than 1/8 of B or of C
 * (graph matrices: R-MAT 2^22 touches 48% of its columns and 52% of its rows
 * are empty), the entry point moves just those rows (copy kernels reading
 * and writing the mapped host buffers, up to four column chunks overlapped
 * as above) and zeroes the empty C rows on host threads; otherwise, and for
 * plans with tensor-core blocks, *b_rows = N and *c_rows = M.  Builds the row
 * lists on first use (synchronises `stream`).  No counterpart in the
 * reference (its main copies all of B and C). */
vcsr_status vcsr_plan_host_rows(vcsr_plan *plan, int *b_rows, int *c_rows,
                                vcsr_stream_t stream);

/* Synchronises `stream` and reports a failure that the plan's kernels
 * recorded on the device since the last check (the tensor-core panel kernel
 * bounds every wait on its pipeline barriers and records the first one that
 * ran out): VCSR_ERR_TIMEOUT with the barrier named in vcsr_last_error(); the
 * record is cleared.  vcsr_spmm_host checks on its own.  No counterpart in
 * the reference (its kernels have no waits). */
vcsr_status vcsr_plan_check(vcsr_plan *plan, vcsr_stream_t stream);

/* Test hook for the failure path above, not for production use: the next
 * TF32 panel launch of `plan` withholds one barrier signal in its first block
 * (the accumulator-ready signal of that block's first item), so the block's
 * epilogue wait for it runs out after a short bounded poll; the block stops
 * its other roles, waits for its own copies and MMAs, frees its tensor
 * memory and records the site, and vcsr_plan_check then returns
 * VCSR_ERR_TIMEOUT ("accumulator-full ... block 0").  C is incomplete for
 * that call only; the hook is one-shot.  Nothing faults or hangs.
 * VCSR_ERR_UNSUPPORTED for a plan without TF32 panels.  No counterpart in the
 * reference. */
vcsr_status vcsr_plan_test_withhold_signal(vcsr_plan *plan);

/* ------------------------------------------------------------ peer paths */

/* Race-free SpMM straight on a device VCSR; same contract as
 * run_vcsr_spmm_gpu (src/kernels.cu:120): C += A*B (C must hold zeros, or the
 * partial sum to add to), ld = O for B and C.  Each group keeps its rows' sums
 * in registers over its depth and adds them to C with vector atomics. */
vcsr_status vcsr_spmm_segmented(const vcsr_vcsr *dev, const float *dB, int O,
                                int tileK, float *dC, vcsr_stream_t stream);

/* CSR row-wise SpMM on device arrays; same contract as run_csr_spmm_gpu
 * (src/kernels.cu:107-118): C = A*B with ld = O. */
vcsr_status vcsr_csr_spmm(int M, const int *d_row_ptr, const int *d_col,
                          const float *d_val, const float *dB, int O,
                          float *dC, vcsr_stream_t stream);

/* CSR SpMM that allocates nothing (no cudaMalloc, cudaFree or allocating
 * library call).  No counterpart in the reference.  For callers that cannot
 * allocate device memory: a solver embedded in an application whose framework
 * hands all free device memory to its own caching pool at start-up (a
 * cudaMalloc would then fail, or take memory the pool counts on), or a code
 * path that has a fixed device-memory budget.  Same contract as vcsr_csr_spmm
 * (C = A*B, ld = O, device pointers), but rows longer than
 * VCSR_NOALLOC_SPLIT entries are cut into parts walked by separate warps, and
 * the bookkeeping and partial sums of those parts live in one
 * VCSR_NOALLOC_SCRATCH_BYTES array compiled into the library (every GPU that
 * loads the library holds it until the process exits).  Limits, rejected
 * with VCSR_ERR_RANGE and a message: O <= VCSR_NOALLOC_MAX_O; at most
 * VCSR_NOALLOC_MAX_LONG_ROWS long rows; at most VCSR_NOALLOC_MAX_PARTS parts
 * over all long rows (the last two are detected on the device, and C is then
 * incomplete).  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  Each call clears the counters it needs,
 * synchronises `stream` once to read the overflow flag, and shares the one
 * array: calls that overlap on the GPU (other streams, other threads) race. */
#define VCSR_NOALLOC_MAX_O 512
#define VCSR_NOALLOC_MAX_LONG_ROWS 1024
#define VCSR_NOALLOC_MAX_PARTS 2048
#define VCSR_NOALLOC_SPLIT 4096
#define VCSR_NOALLOC_SCRATCH_BYTES 6320384
vcsr_status vcsr_csr_spmm_noalloc(int M, const int *d_row_ptr, const int *d_col,
                                  const float *d_val, const float *dB, int O,
                                  float *dC, vcsr_stream_t stream);

/* cuSPARSE SpMM with the handle, descriptors, buffer and preprocessing made
 * once; replaces run_cusparse_spmm (src/kernels.cu:170-235).  alg: 0 =
 * CUSPARSE_SPMM_ALG_DEFAULT, 1 = CSR_ALG1, 2 = CSR_ALG2, 3 = CSR_ALG3. */
typedef struct vcsr_cusparse vcsr_cusparse;
vcsr_status vcsr_cusparse_create(int M, int N, int nnz, const int *d_row_ptr,
                                 const int *d_col, const float *d_val,
                                 const float *dB, int O, float *dC, int alg,
                                 vcsr_stream_t stream, vcsr_cusparse **out);
vcsr_status vcsr_cusparse_run(vcsr_cusparse *h, vcsr_stream_t stream);
void vcsr_cusparse_destroy(vcsr_cusparse *h);

/* -------------------------------------------------------------- multi-GPU */

/* nnz-balanced row panels: cuts[0] = 0, cuts[parts] = M, cut k is the row
 * nearest to k*nnz/parts (binary search of row_ptr) rounded to a multiple of
 * align (rows), kept non-decreasing.  Host-only. */
vcsr_status vcsr_partition_rows(const int *row_ptr, int M, int parts,
                                int align, int *cuts);
/* The same with a per-row cost: row r weighs (its nnz + row_weight), so
 * panels of many short rows get fewer rows (each row also costs a C row write
 * and its own setup).  row_weight = 0 is vcsr_partition_rows. */
vcsr_status vcsr_partition_rows_weighted(const int *row_ptr, int M, int parts, int align,
                                         double row_weight, int *cuts);

/* Extract rows [r0, r1) of a host CSR as a new host CSR (row ids local). */
vcsr_status vcsr_csr_row_panel(const vcsr_csr *csr, int r0, int r1,
                               vcsr_csr *out);

/* Row panels of A on several GPUs of one process.  No reference counterpart
 * (the reference runs on device 0 only, src/kernels.cu:129); the survey's
 * multi-GPU design: nnz-balanced row panels (vcsr_partition_rows, align =
 * bundle), one plan per device, B replicated by one ncclBroadcast over
 * NVLink, disjoint C panels (no reduction).  NCCL is loaded at run time
 * (libnccl.so.2); every wait on a collective is bounded (60 s), after which
 * the communicators are aborted and VCSR_ERR_TIMEOUT is returned. */
typedef struct vcsr_mgpu vcsr_mgpu;
vcsr_status vcsr_mgpu_create(const vcsr_csr *host_csr, int ngpus,
                             const int *devices, const vcsr_plan_params *params,
                             vcsr_mgpu **out);
/* Copy host B (N x O, ld = O) to the first device and broadcast it to all;
 * *bcast_ms = time of the broadcast (max over devices). */
vcsr_status vcsr_mgpu_set_b(vcsr_mgpu *m, const float *hB, int O,
                            float *bcast_ms);
/* Every device computes its C panel; *ms = max over devices of the kernel
 * time measured with CUDA events. */
vcsr_status vcsr_mgpu_spmm(vcsr_mgpu *m, int O, float *ms);
/* Copy the C panels to host C (M x O, ld = O). */
vcsr_status vcsr_mgpu_gather_c(vcsr_mgpu *m, float *hC);
/* Row cut points (ngpus + 1 entries) of the panels. */
vcsr_status vcsr_mgpu_cuts(const vcsr_mgpu *m, int *cuts);
void vcsr_mgpu_destroy(vcsr_mgpu *m);

#ifdef __cplusplus
}
#endif

#endif /* VCSR_SPMM_H */
