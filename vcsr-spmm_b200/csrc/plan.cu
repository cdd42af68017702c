// plan.cu — SpMM plans: build once (layout + upload), run many times.
//
// vcsr_plan_create is the format-build-and-upload half of run_vcsr_spmm_gpu
// (src/kernels.cu:120-151) done once per matrix instead of per call;
// vcsr_spmm is its launch half (src/kernels.cu:153-160) with C written
// instead of accumulated into a caller-zeroed buffer.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <vector>
#if defined(__SSE2__)
#include <emmintrin.h>
#endif

#include "common.h"
#include "host_transfer.h"
#include "panel.h"
#include "panel_gpu.h"
#include "plan_impl.h"
#include "panel_tc.h"
#include "spmm_kernels.h"
#include "seg_tc.h"
#include "spmm_tc.h"

using vcsr::fail;
using vcsr::upload;

namespace vcsr {

void plan_release(vcsr_plan *p) {
  cudaFree(p->d_ucol); cudaFree(p->d_uval); cudaFree(p->d_umask); cudaFree(p->d_units);
  cudaFree(p->d_batches); cudaFree(p->d_long); cudaFree(p->d_long_col);
  cudaFree(p->d_vec_ptr);
  cudaFree(p->d_parts); cudaFree(p->d_svecs); cudaFree(p->d_partials);
  cudaFree(p->d_counters); cudaFree(p->d_stage_B); cudaFree(p->d_stage_C);
  cudaFree(p->d_xcols); cudaFree(p->d_xrows);
  if (p->has_ref) vcsr_vcsr_free(&p->ref, VCSR_DEVICE);
  cudaFree(p->d_rb_row); cudaFree(p->d_rb_ptr); cudaFree(p->d_blk_col);
  cudaFree(p->d_blk_val); cudaFree(p->d_err);
  cudaFree(p->d_seg_rb_row); cudaFree(p->d_seg_pp); cudaFree(p->d_seg_pieces);
  cudaFree(p->d_seg_a); cudaFree(p->d_seg_rp); cudaFree(p->d_seg_col); cudaFree(p->d_seg_val);
  if (p->side) cudaStreamDestroy(p->side);
  if (p->down) cudaStreamDestroy(p->down);
  if (p->comp) cudaStreamDestroy(p->comp);
  for (cudaEvent_t e : p->chunk_done) cudaEventDestroy(e);
  if (p->fork) cudaEventDestroy(p->fork);
  if (p->join) cudaEventDestroy(p->join);
}

vcsr_status plan_finish(vcsr_plan *p, cudaStream_t st) {
  VCSR_TRY(order_long_by_column(p, st));
  if (p->n_long > 0 && p->n_batches > 0) {
    cudaError_t e = cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->fork, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->join, cudaEventDisableTiming);
    if (e != cudaSuccess) return fail(VCSR_ERR_CUDA, "side stream: %s", cudaGetErrorString(e));
  }
  if (p->n_split_units > 0) {
    const size_t pbytes = sizeof(float) * (size_t)p->n_split_units * p->R * p->pstride;
    const size_t cbytes = sizeof(int) * (size_t)p->n_split_vectors * p->counter_stride;
    cudaError_t e = cudaMalloc(&p->d_partials, pbytes);
    if (e == cudaSuccess) e = cudaMalloc(&p->d_counters, cbytes);
    if (e == cudaSuccess) e = cudaMemsetAsync(p->d_counters, 0, cbytes, st);
    if (e != cudaSuccess) return fail(VCSR_ERR_CUDA, "split scratch: %s", cudaGetErrorString(e));
    p->panel_bytes += (int64_t)(pbytes + cbytes);
  }
  return VCSR_OK;
}

}  // namespace vcsr

namespace {

vcsr::PanelDevView view(const vcsr_plan *p) {
  vcsr::PanelDevView v;
  v.ucol = p->d_ucol;
  v.uval = p->d_uval;
  v.umask = p->R > 1 ? p->d_umask : nullptr;
  v.units = p->d_units;
  v.n_units = p->n_units;
  v.batches = p->d_batches;
  v.n_batches = p->n_batches;
  v.vec_ptr = p->d_vec_ptr;
  v.long_idx = p->d_long;
  v.n_long = p->n_long;
  v.parts = p->d_parts;
  v.svecs = p->d_svecs;
  v.partials = p->d_partials;
  v.counters = p->d_counters;
  v.pstride = p->pstride;
  v.counter_stride = p->counter_stride;
  v.n_split_units = p->n_split_units;
  v.M = p->M;
  v.R = p->R;
  return v;
}

// The view for a launch over the whole matrix: long units in column order.
vcsr::PanelDevView view_all(const vcsr_plan *p) {
  vcsr::PanelDevView v = view(p);
  if (p->d_long_col) v.long_idx = p->d_long_col;
  return v;
}

// Host copy of a CSR whose rows are sorted by column (stable); *owned says
// whether the copy must be freed.
vcsr_status host_sorted_csr(const vcsr_csr *in, int where, vcsr_csr *out,
                            bool *owned) {
  *owned = false;
  vcsr_csr h = *in;
  if (where == VCSR_DEVICE) {
    h.row_ptr = (int *)malloc(sizeof(int) * ((size_t)in->M + 1));
    h.col = (int *)malloc(sizeof(int) * (size_t)(in->nnz ? in->nnz : 1));
    h.val = (float *)malloc(sizeof(float) * (size_t)(in->nnz ? in->nnz : 1));
    *owned = true;
    if (!h.row_ptr || !h.col || !h.val) {
      vcsr_csr_free(&h, VCSR_HOST);
      return fail(VCSR_ERR_ALLOC, "out of host memory");
    }
    VCSR_CUDA(cudaMemcpy(h.row_ptr, in->row_ptr, sizeof(int) * ((size_t)in->M + 1),
                         cudaMemcpyDeviceToHost));
    if (in->nnz) {
      VCSR_CUDA(cudaMemcpy(h.col, in->col, sizeof(int) * (size_t)in->nnz,
                           cudaMemcpyDeviceToHost));
      VCSR_CUDA(cudaMemcpy(h.val, in->val, sizeof(float) * (size_t)in->nnz,
                           cudaMemcpyDeviceToHost));
    }
  }
  // validate
  if (h.row_ptr[0] != 0 || h.row_ptr[h.M] != h.nnz) {
    if (*owned) vcsr_csr_free(&h, VCSR_HOST);
    return fail(VCSR_ERR_INVALID, "row_ptr must start at 0 and end at nnz");
  }
  bool sorted = true;
  for (int r = 0; r < h.M; ++r) {
    if (h.row_ptr[r + 1] < h.row_ptr[r]) {
      if (*owned) vcsr_csr_free(&h, VCSR_HOST);
      return fail(VCSR_ERR_INVALID, "row_ptr decreases at row %d", r);
    }
    for (int p = h.row_ptr[r]; p < h.row_ptr[r + 1]; ++p) {
      if (h.col[p] < 0 || h.col[p] >= h.N) {
        if (*owned) vcsr_csr_free(&h, VCSR_HOST);
        return fail(VCSR_ERR_RANGE, "column %d of entry %d outside [0, %d)",
                    h.col[p], p, h.N);
      }
      if (p > h.row_ptr[r] && h.col[p] < h.col[p - 1]) sorted = false;
    }
  }
  if (!sorted) {  // stable per-row sort of a private copy
    vcsr_csr s = h;
    s.row_ptr = (int *)malloc(sizeof(int) * ((size_t)h.M + 1));
    s.col = (int *)malloc(sizeof(int) * (size_t)(h.nnz ? h.nnz : 1));
    s.val = (float *)malloc(sizeof(float) * (size_t)(h.nnz ? h.nnz : 1));
    if (!s.row_ptr || !s.col || !s.val) {
      vcsr_csr_free(&s, VCSR_HOST);
      if (*owned) vcsr_csr_free(&h, VCSR_HOST);
      return fail(VCSR_ERR_ALLOC, "out of host memory");
    }
    std::memcpy(s.row_ptr, h.row_ptr, sizeof(int) * ((size_t)h.M + 1));
#pragma omp parallel for schedule(dynamic, 256)
    for (int r = 0; r < h.M; ++r) {
      const int b = h.row_ptr[r], e = h.row_ptr[r + 1];
      std::vector<int> idx(e - b);
      for (int q = 0; q < e - b; ++q) idx[q] = b + q;
      std::stable_sort(idx.begin(), idx.end(),
                       [&](int a, int c) { return h.col[a] < h.col[c]; });
      for (int q = 0; q < e - b; ++q) {
        s.col[b + q] = h.col[idx[q]];
        s.val[b + q] = h.val[idx[q]];
      }
    }
    if (*owned) vcsr_csr_free(&h, VCSR_HOST);
    h = s;
    *owned = true;
  }
  *out = h;
  return VCSR_OK;
}

// The default build: the CSR goes to (or stays on) the device, is validated
// and, if needed, row-sorted there, and every array of the layout is built
// by device kernels (panel_gpu_build.cu); the host reads back only totals.
vcsr_status create_on_device(vcsr_plan *p, const vcsr_csr *csr, int where, int sms,
                             cudaStream_t st) {
  vcsr_csr din = *csr, up{}, sorted{};
  bool up_owned = false, sorted_owned = false;
  vcsr_status s = VCSR_OK;
  int zero = 0;
  if (where == VCSR_HOST || csr->M == 0) {  // to the device (M = 0: a valid row_ptr)
    vcsr_csr h = *csr;
    if (csr->M == 0) h.row_ptr = &zero;
    s = vcsr_csr_to_device(&h, &up, st);
    up_owned = s == VCSR_OK;
    din = up;
  }
  if (s == VCSR_OK) s = vcsr::device_sorted_csr(din, &sorted, &sorted_owned, st);
  if (s == VCSR_OK) s = vcsr::build_plan_layout_device(p, sorted, sms, st);
  if (s == VCSR_OK) s = vcsr::plan_finish(p, st);
  if (s == VCSR_OK && (p->params.flags & VCSR_PLAN_REFERENCE_FORMAT)) {
    s = vcsr_build_vcsr(&sorted, p->params.segw, p->params.bundle, &p->ref, st);
    p->has_ref = s == VCSR_OK;
  }
  const cudaError_t e = cudaStreamSynchronize(st);  // the temporaries die here
  if (sorted_owned) vcsr_csr_free(&sorted, VCSR_DEVICE);
  if (up_owned) vcsr_csr_free(&up, VCSR_DEVICE);
  if (s != VCSR_OK) return s;
  if (e != cudaSuccess) return fail(VCSR_ERR_CUDA, "plan build: %s", cudaGetErrorString(e));
  return VCSR_OK;
}

}  // namespace

extern "C" {

void vcsr_plan_params_default(vcsr_plan_params *p) {
  if (!p) return;
  p->segw = 4;
  p->bundle = 32;
  p->tileK = 0;
  p->max_O = 512;
  p->vec_rows = 0;
  p->chunk = 0;
  p->flags = 0;
  p->panel_min_nnz = 0;
  p->target_O = 0;
  p->seg_min_run = 0;
}

vcsr_status vcsr_plan_create(const vcsr_csr *csr, int csr_where,
                             const vcsr_plan_params *params, vcsr_plan **out,
                             vcsr_stream_t stream) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!csr || !params || !out) return fail(VCSR_ERR_INVALID, "null argument");
    *out = nullptr;
    if (csr->M < 0 || csr->N < 0 || csr->nnz < 0)
      return fail(VCSR_ERR_INVALID, "negative matrix size");
    if (params->segw <= 0 || params->bundle <= 0)
      return fail(VCSR_ERR_INVALID, "segw and bundle must be > 0");
    if (params->max_O < 0 || params->tileK < 0)
      return fail(VCSR_ERR_INVALID, "negative max_O or tileK");
    if (csr->M > 0 && !csr->row_ptr) return fail(VCSR_ERR_INVALID, "null row_ptr");
    if (csr->nnz > 0 && (!csr->col || !csr->val))
      return fail(VCSR_ERR_INVALID, "null col/val");
    const auto t0 = std::chrono::steady_clock::now();
    cudaStream_t st = (cudaStream_t)stream;
    vcsr_plan *p = new (std::nothrow) vcsr_plan();
    if (!p) return fail(VCSR_ERR_ALLOC, "out of host memory");
    p->M = csr->M; p->N = csr->N; p->nnz = csr->nnz;
    p->params = *params;
    cudaGetDevice(&p->device);
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device);
    if (!(params->flags & VCSR_PLAN_HOST_BUILD)) {  // the layout built by GPU kernels
      const vcsr_status s = create_on_device(p, csr, csr_where, sms, st);
      if (s != VCSR_OK) {
        vcsr::plan_release(p);
        delete p;
        return s;
      }
      p->build_ms = std::chrono::duration<double, std::milli>(
                        std::chrono::steady_clock::now() - t0).count();
      *out = p;
      return VCSR_OK;
    }

    if (params->flags & VCSR_PLAN_TC_SEGMENTS) {
      delete p;
      return fail(VCSR_ERR_UNSUPPORTED, "tensor-core segments are built on the GPU only");
    }
    vcsr_csr h{};
    bool owned = false;
    vcsr_csr empty_rp{};
    std::vector<int> zero_rp;
    if (csr->M == 0) {  // nothing to read; keep a valid row_ptr
      zero_rp.assign(1, 0);
      empty_rp = *csr;
      empty_rp.row_ptr = zero_rp.data();
      h = empty_rp;
    } else {
      vcsr_status s = host_sorted_csr(csr, csr_where, &h, &owned);
      if (s != VCSR_OK) { delete p; return s; }
    }

    // TF32 panels: the dense 16x16 blocks go to the tensor-core path, the
    // rest (the residual) to the row-stationary layout below
    vcsr::TcHost tc;
    std::vector<int> r_rp, r_col;
    std::vector<float> r_val;
    vcsr_csr work = h;
    if ((params->flags & VCSR_PLAN_TF32_PANELS) && h.M > 0) {
      if (params->panel_min_nnz < 0 || params->panel_min_nnz > 256) {
        if (owned) vcsr_csr_free(&h, VCSR_HOST);
        delete p;
        return fail(VCSR_ERR_INVALID, "panel_min_nnz must be in [0, 256]");
      }
      const int min_nnz = params->panel_min_nnz > 0 ? params->panel_min_nnz : 128;
      vcsr_status s0 = vcsr::split_dense_panels(h, min_nnz, &tc, r_rp, r_col, r_val);
      if (s0 != VCSR_OK) {
        if (owned) vcsr_csr_free(&h, VCSR_HOST);
        delete p;
        return s0;
      }
      work.nnz = r_rp.back();
      work.row_ptr = r_rp.data();
      work.col = r_col.data();
      work.val = r_val.data();
      p->n_panel_rb = (int)tc.rb_row.size();
      p->n_panel_blocks = (int)tc.blk_col.size();
      p->panel_nnz = (int64_t)h.nnz - work.nnz;
    }
    vcsr::PanelHost ph;
    int R = params->vec_rows;
    if (R == 0) {
      R = vcsr::choose_vec_rows(work, nullptr);
      if (R == 8 && params->target_O > 128) R = 4;
    }
    vcsr_status s = vcsr::build_panel_host(work, R, params->chunk, sms, &ph);
    if (s != VCSR_OK) {
      if (owned) vcsr_csr_free(&h, VCSR_HOST);
      delete p;
      return s;
    }
    p->R = ph.R;
    p->num_vectors = ph.num_vectors;
    p->num_union = (int64_t)ph.ucol.size();
    p->chunk = ph.chunk;
    p->n_units = (int)ph.units.size();
    p->n_split_units = (int)ph.parts.size();
    p->n_split_vectors = (int)ph.svecs.size();
    p->pstride = std::max(params->max_O, 1);
    p->counter_stride = std::max(params->max_O, 1);
    static_assert(sizeof(vcsr::Unit) == sizeof(int4), "Unit must match int4");
    static_assert(sizeof(vcsr::SplitPart) == sizeof(int2), "SplitPart must match int2");
    static_assert(sizeof(vcsr::SplitVec) == sizeof(int2), "SplitVec must match int2");
    std::vector<int4> units(ph.units.size());
    std::memcpy(units.data(), ph.units.data(), sizeof(int4) * units.size());
    // Split parts and units of at least kLongUnit union columns are walked by a
    // whole warp (its sub-warps split the columns).  The other vectors are
    // packed, in order, into batches of consecutive vectors walked by one
    // sub-warp each: a batch starts after a long unit, at every 64th short
    // unit, and where the short units' running column count crosses a
    // multiple of `batch_cols`, chosen so that there are ~64 batches per SM
    // (the rule the GPU builder applies in parallel, panel_gpu_build.cu).
    // With R > 2 a batch is one vector (vectors are long enough on their own).
    constexpr int kLongUnit = 128, kMaxBatchVecs = 64;
    std::vector<int> long_idx;
    std::vector<int4> batches;
    int64_t short_cols = 0;
    for (const auto &u : ph.units)
      if (u.slot < 0 && u.end - u.begin < kLongUnit) short_cols += u.end - u.begin;
    const int64_t batch_cols =
        std::max<int64_t>(16, std::min<int64_t>(256, short_cols / ((int64_t)sms * 64)));
    {
      int4 cur = make_int4(-1, -1, 0, 0);
      auto close = [&]() {
        if (cur.x >= 0) batches.push_back(cur);
        cur.x = -1;
      };
      // short units so far; the exclusive column prefix at this short unit
      // and at the previous one
      int64_t k = 0, C = 0, prevC = 0;
      for (size_t u = 0; u < ph.units.size(); ++u) {
        const auto &un = ph.units[u];
        const int len = un.end - un.begin;
        if (un.slot >= 0 || len >= kLongUnit) {
          long_idx.push_back((int)u);
          close();
          continue;
        }
        if (cur.x >= 0 && (ph.R > 2 || k % kMaxBatchVecs == 0 ||
                           C / batch_cols != prevC / batch_cols))
          close();
        if (cur.x < 0) cur = make_int4(un.vec, un.vec, un.begin, un.begin);
        cur.y = un.vec + 1;
        cur.w = un.end;
        prevC = C;
        C += len;
        ++k;
      }
      close();
    }
    p->n_batches = (int)batches.size();
    p->n_long = (int)long_idx.size();
    // Row panels (cut at vectors where a batch or a long unit starts) for the
    // host entry point's row pipeline; not with TF32 panels, whose kernel
    // covers all rows at once.  Cuts at 1/32, 1/6, ..., 5/6 and 31/32 of the
    // entries: the small first and last panels shorten the pipeline's fill
    // (the first upload before any product) and drain (the last download
    // after the last upload); measured on FEM at O = 32 / 128 / 512 against
    // eight equal panels: -16% / -2% / -1% per call (more panels cost more
    // per-panel overhead than they save).
    if (p->n_panel_rb == 0 && work.M >= 8192 && work.nnz >= (1 << 20)) {
      constexpr int kRowPanels = 8;
      constexpr double kCut[kRowPanels - 1] = {1.0 / 32, 1.0 / 6, 2.0 / 6, 3.0 / 6,
                                               4.0 / 6,  5.0 / 6, 31.0 / 32};
      std::vector<int> cuts;  // vector indices where a panel may start
      for (const int4 &b : batches) cuts.push_back(b.x);
      for (int u : long_idx) cuts.push_back(ph.units[u].vec);
      std::sort(cuts.begin(), cuts.end());
      cuts.erase(std::unique(cuts.begin(), cuts.end()), cuts.end());
      std::vector<int> vb{0};
      for (int j = 1; j < kRowPanels; ++j) {
        const int64_t target = (int64_t)(work.nnz * kCut[j - 1]);
        const int row = (int)(std::lower_bound(work.row_ptr, work.row_ptr + work.M + 1, target) -
                              work.row_ptr);
        auto it = std::lower_bound(cuts.begin(), cuts.end(), row / ph.R);
        if (it != cuts.end() && *it > vb.back()) vb.push_back(*it);
      }
      vb.push_back(ph.num_vectors);
      std::vector<int> lvec(long_idx.size());
      for (size_t i = 0; i < long_idx.size(); ++i) lvec[i] = ph.units[long_idx[i]].vec;
      std::vector<int> bvec(batches.size());
      for (size_t i = 0; i < batches.size(); ++i) bvec[i] = batches[i].x;
      for (size_t j = 0; j + 1 < vb.size(); ++j) {
        vcsr_plan::RowPanel rp;
        rp.row0 = vb[j] * ph.R;
        rp.row1 = std::min(work.M, vb[j + 1] * ph.R);
        rp.b0 = (int)(std::lower_bound(bvec.begin(), bvec.end(), vb[j]) - bvec.begin());
        rp.b1 = (int)(std::lower_bound(bvec.begin(), bvec.end(), vb[j + 1]) - bvec.begin());
        rp.l0 = (int)(std::lower_bound(lvec.begin(), lvec.end(), vb[j]) - lvec.begin());
        rp.l1 = (int)(std::lower_bound(lvec.begin(), lvec.end(), vb[j + 1]) - lvec.begin());
        rp.col_max = -1;
        for (int r = rp.row0; r < rp.row1; ++r)
          if (work.row_ptr[r + 1] > work.row_ptr[r])
            rp.col_max = std::max(rp.col_max, work.col[work.row_ptr[r + 1] - 1]);
        p->rpanels.push_back(rp);
      }
    }
    std::vector<int2> parts(ph.parts.size()), svecs(ph.svecs.size());
    std::memcpy(parts.data(), ph.parts.data(), sizeof(int2) * parts.size());
    std::memcpy(svecs.data(), ph.svecs.data(), sizeof(int2) * svecs.size());
    if ((s = upload(&p->d_ucol, ph.ucol, st, &p->panel_bytes)) ||
        (s = upload(&p->d_uval, ph.uval, st, &p->panel_bytes)) ||
        (s = upload(&p->d_umask, ph.umask, st, &p->panel_bytes)) ||
        (s = upload(&p->d_units, units, st, &p->panel_bytes)) ||
        (s = upload(&p->d_parts, parts, st, &p->panel_bytes)) ||
        (s = upload(&p->d_svecs, svecs, st, &p->panel_bytes)) ||
        (s = upload(&p->d_batches, batches, st, &p->panel_bytes)) ||
        (s = upload(&p->d_long, long_idx, st, &p->panel_bytes)) ||
        (s = upload(&p->d_vec_ptr, ph.vec_ptr, st, &p->panel_bytes))) {
      if (owned) vcsr_csr_free(&h, VCSR_HOST);
      vcsr::plan_release(p);
      delete p;
      return s;
    }
    if (p->n_panel_rb > 0) {
      std::vector<int> zero1(1, 0);
      if ((s = upload(&p->d_rb_row, tc.rb_row, st, &p->panel_bytes)) ||
          (s = upload(&p->d_rb_ptr, tc.rb_ptr, st, &p->panel_bytes)) ||
          (s = upload(&p->d_blk_col, tc.blk_col, st, &p->panel_bytes)) ||
          (s = upload(&p->d_blk_val, tc.blk_val, st, &p->panel_bytes)) ||
          (s = upload(&p->d_err, zero1, st, &p->panel_bytes))) {
        if (owned) vcsr_csr_free(&h, VCSR_HOST);
        vcsr::plan_release(p);
        delete p;
        return s;
      }
    }
    if ((s = vcsr::plan_finish(p, st)) != VCSR_OK) {
      if (owned) vcsr_csr_free(&h, VCSR_HOST);
      vcsr::plan_release(p);
      delete p;
      return s;
    }
    if (params->flags & VCSR_PLAN_REFERENCE_FORMAT) {
      vcsr_csr d{};
      s = vcsr_csr_to_device(&h, &d, stream);
      if (s == VCSR_OK) s = vcsr_build_vcsr(&d, params->segw, params->bundle, &p->ref, stream);
      if (d.row_ptr) {
        cudaStreamSynchronize(st);
        vcsr_csr_free(&d, VCSR_DEVICE);
      }
      if (s != VCSR_OK) {
        if (owned) vcsr_csr_free(&h, VCSR_HOST);
        vcsr::plan_release(p);
        delete p;
        return s;
      }
      p->has_ref = true;
    }
    cudaError_t e = cudaStreamSynchronize(st);  // host vectors die here
    if (owned) vcsr_csr_free(&h, VCSR_HOST);
    if (e != cudaSuccess) {
      vcsr::plan_release(p);
      delete p;
      return fail(VCSR_ERR_CUDA, "plan upload: %s", cudaGetErrorString(e));
    }
    p->build_ms = std::chrono::duration<double, std::milli>(
                      std::chrono::steady_clock::now() - t0).count();
    *out = p;
    return VCSR_OK;
  });
}

vcsr_status vcsr_plan_get_info(const vcsr_plan *p, vcsr_plan_info *info) {
  vcsr::clear_error();
  if (!p || !info) return fail(VCSR_ERR_INVALID, "null argument");
  info->M = p->M; info->N = p->N; info->nnz = p->nnz;
  info->vec_rows = p->R;
  info->num_vectors = p->num_vectors;
  info->num_union = p->num_union;
  info->num_units = p->n_units;
  info->num_split_vectors = p->n_split_vectors;
  info->num_split_units = p->n_split_units;
  info->num_long_units = p->n_long;
  info->panel_bytes = p->panel_bytes;
  info->has_reference_format = p->has_ref ? 1 : 0;
  info->build_ms = p->build_ms;
  info->num_panel_blocks = p->n_panel_blocks;
  info->num_panel_row_blocks = p->n_panel_rb;
  info->panel_nnz = p->panel_nnz;
  info->num_seg_row_blocks = p->n_seg_rb;
  info->num_seg_pieces = p->n_seg_pieces;
  info->seg_rows = p->seg_rows;
  info->seg_only = p->seg_only ? 1 : 0;
  return VCSR_OK;
}

vcsr_status vcsr_plan_export(const vcsr_plan *p, vcsr_vcsr *host_out) {
  vcsr::clear_error();
  if (!p || !host_out) return fail(VCSR_ERR_INVALID, "null argument");
  if (!p->has_ref)
    return fail(VCSR_ERR_INVALID,
                "plan was built without VCSR_PLAN_REFERENCE_FORMAT");
  return vcsr_vcsr_to_host(&p->ref, host_out);
}

void vcsr_plan_destroy(vcsr_plan *p) {
  if (!p) return;
  vcsr::plan_release(p);
  delete p;
}

namespace {

// C = A * B, or C += A * B with `accumulate`: every kernel of the plan then
// adds into C (the FP32 kernels load, add and store each finished value; the
// tensor-core kernels add their product after the FP32 residual).
vcsr_status spmm_impl(const vcsr_plan *p, const float *dB, int ldb, float *dC, int ldc, int O,
                      vcsr_stream_t stream, int *launches, bool accumulate) {
  vcsr::clear_error();
  if (launches) *launches = 0;
  if (!p) return fail(VCSR_ERR_INVALID, "null plan");
  if (O < 0 || ldb < O || ldc < O)
    return fail(VCSR_ERR_INVALID, "need 0 <= O <= ldb, ldc (O=%d ldb=%d ldc=%d)",
                O, ldb, ldc);
  if (O == 0 || p->M == 0) return VCSR_OK;
  if (!dC || (!dB && p->N > 0)) return fail(VCSR_ERR_INVALID, "null B or C");
  if (p->n_split_units > 0 && O > p->pstride)
    return fail(VCSR_ERR_INVALID,
                "O=%d exceeds the plan's max_O=%d (split rows need scratch)", O,
                p->pstride);
  int n1 = 0, n2 = 0;
  vcsr::PanelDevView pv = view_all(p);
  pv.accumulate = accumulate ? 1 : 0;
  if (p->n_seg_rb > 0) {  // tensor-core segments; the residual (if any) first
    if (!p->seg_only)
      VCSR_TRY(vcsr::launch_panel_spmm(pv, false, dB, ldb, dC, ldc, O,
                                       (cudaStream_t)stream, &n1, p->side, p->fork, p->join));
    vcsr::SegView sv;
    sv.n_rb = p->n_seg_rb;
    sv.rb_row = p->d_seg_rb_row;
    sv.pp = p->d_seg_pp;
    sv.pieces = p->d_seg_pieces;
    sv.a = p->d_seg_a;
    sv.rp = p->d_seg_rp;
    sv.col = p->d_seg_col;
    sv.val = p->d_seg_val;
    sv.M = p->M;
    sv.accumulate = (p->seg_only && !accumulate) ? 0 : 1;
    sv.err = p->d_err;
    VCSR_TRY(vcsr::launch_seg_tc(sv, dB, p->N, ldb, dC, ldc, O, (cudaStream_t)stream, &n2));
    if (launches) *launches = n1 + n2;
    return VCSR_OK;
  }
  // Single-row vectors with no long or split rows and at least 8 entries per
  // row on average (uniform-degree matrices): one sub-warp per row, straight
  // from the row offsets (vec_ptr is the CSR's row_ptr when R = 1), one
  // dependent load fewer than a batch record and its vector offsets.
  // Measured on B200, uniform 16 entries per row at O = 32: 4,096 rows
  // 10.1 -> 8.3 us, 65,536 rows 28.6 -> 25.6 us, 2^20 rows 462 -> 436 us;
  // O = 128 unchanged; the sums are the same (each row in CSR order).
  const bool by_rows = p->R == 1 && p->n_long == 0 && p->n_split_units == 0 &&
                       p->n_panel_rb == 0 && p->num_union >= 8LL * p->M;
  if (by_rows) {
    pv.row_ptr = p->d_vec_ptr;
    pv.n_units = p->M;
  }
  VCSR_TRY(vcsr::launch_panel_spmm(pv, by_rows, dB, ldb, dC, ldc, O, (cudaStream_t)stream,
                                   &n1, p->side, p->fork, p->join));
  if (p->n_panel_rb > 0) {  // C += dense panels * B on the tensor cores
    vcsr::TcView tv;
    tv.n_rb = p->n_panel_rb;
    tv.rb_row = p->d_rb_row;
    tv.rb_ptr = p->d_rb_ptr;
    tv.blk_col = p->d_blk_col;
    tv.blk_val = p->d_blk_val;
    tv.M = p->M;
    tv.err = p->d_err;
    tv.inject = p->tc_inject.exchange(0);
    VCSR_TRY(vcsr::launch_tc_panels(tv, dB, p->N, ldb, dC, ldc, O, (cudaStream_t)stream, &n2));
  }
  if (launches) *launches = n1 + n2;
  return VCSR_OK;
}

}  // namespace

vcsr_status vcsr_spmm(const vcsr_plan *p, const float *dB, int ldb, float *dC,
                      int ldc, int O, vcsr_stream_t stream, int *launches) {
  return spmm_impl(p, dB, ldb, dC, ldc, O, stream, launches, false);
}

vcsr_status vcsr_spmm_accumulate(const vcsr_plan *p, const float *dB, int ldb, float *dC,
                                 int ldc, int O, vcsr_stream_t stream, int *launches) {
  return spmm_impl(p, dB, ldb, dC, ldc, O, stream, launches, true);
}

vcsr_status vcsr_plan_row_panels(const vcsr_plan *p, int *count, int *row0, int *row1,
                                 int *col_max) {
  vcsr::clear_error();
  if (!p || !count) return fail(VCSR_ERR_INVALID, "null argument");
  const int n = (int)p->rpanels.size();
  if (row0 || row1 || col_max) {
    if (*count < n) return fail(VCSR_ERR_INVALID, "arrays hold %d panels, the plan has %d", *count, n);
    for (int j = 0; j < n; ++j) {
      if (row0) row0[j] = p->rpanels[j].row0;
      if (row1) row1[j] = p->rpanels[j].row1;
      if (col_max) col_max[j] = p->rpanels[j].col_max;
    }
  }
  *count = n;
  return VCSR_OK;
}

vcsr_status vcsr_spmm_row_panel(const vcsr_plan *p, int panel, const float *dB, int ldb,
                                float *dC, int ldc, int O, vcsr_stream_t stream,
                                int *launches) {
  vcsr::clear_error();
  if (launches) *launches = 0;
  if (!p) return fail(VCSR_ERR_INVALID, "null plan");
  if (panel < 0 || panel >= (int)p->rpanels.size())
    return fail(VCSR_ERR_RANGE, "row panel %d of %d", panel, (int)p->rpanels.size());
  if (O < 0 || ldb < O || ldc < O)
    return fail(VCSR_ERR_INVALID, "need 0 <= O <= ldb, ldc (O=%d ldb=%d ldc=%d)", O, ldb, ldc);
  if (O == 0) return VCSR_OK;
  if (!dC || !dB) return fail(VCSR_ERR_INVALID, "null B or C");
  if (p->n_split_units > 0 && O > p->pstride)
    return fail(VCSR_ERR_INVALID,
                "O=%d exceeds the plan's max_O=%d (split rows need scratch)", O, p->pstride);
  const auto &rp = p->rpanels[panel];
  vcsr::PanelDevView v = view(p);
  v.batches += rp.b0;
  v.n_batches = rp.b1 - rp.b0;
  v.long_idx += rp.l0;
  v.n_long = rp.l1 - rp.l0;
  return vcsr::launch_panel_spmm(v, false, dB, ldb, dC, ldc, O, (cudaStream_t)stream, launches,
                                 p->side, p->fork, p->join);
}

namespace {

// vcsr_spmm with B of a 16-bit element type (bt), widened as it is loaded.
vcsr_status spmm_16bit(const vcsr_plan *p, const void *dB, int ldb, float *dC, int ldc, int O,
                       vcsr_stream_t stream, int *launches, vcsr::BType bt, const char *name) {
  vcsr::clear_error();
  if (launches) *launches = 0;
  if (!p) return fail(VCSR_ERR_INVALID, "null plan");
  if (O < 0 || ldb < O || ldc < O)
    return fail(VCSR_ERR_INVALID, "need 0 <= O <= ldb, ldc (O=%d ldb=%d ldc=%d)", O, ldb, ldc);
  if (O == 0 || p->M == 0) return VCSR_OK;
  if (!dC || (!dB && p->N > 0)) return fail(VCSR_ERR_INVALID, "null B or C");
  if (p->n_panel_rb > 0 || p->n_seg_rb > 0)
    return fail(VCSR_ERR_UNSUPPORTED,
                "a plan with tensor-core panels or segments reads B in FP32");
  if ((uintptr_t)dB % 2) return fail(VCSR_ERR_INVALID, "%s B must be 2-byte aligned", name);
  if (p->n_split_units > 0 && O > p->pstride)
    return fail(VCSR_ERR_INVALID,
                "O=%d exceeds the plan's max_O=%d (split rows need scratch)", O, p->pstride);
  return vcsr::launch_panel_spmm(view_all(p), false, dB, ldb, dC, ldc, O, (cudaStream_t)stream,
                                 launches, p->side, p->fork, p->join, bt);
}

}  // namespace

vcsr_status vcsr_spmm_bf16(const vcsr_plan *p, const void *dB, int ldb, float *dC, int ldc,
                           int O, vcsr_stream_t stream, int *launches) {
  return spmm_16bit(p, dB, ldb, dC, ldc, O, stream, launches, vcsr::BType::kBF16, "BF16");
}

vcsr_status vcsr_spmm_f16(const vcsr_plan *p, const void *dB, int ldb, float *dC, int ldc,
                          int O, vcsr_stream_t stream, int *launches) {
  return spmm_16bit(p, dB, ldb, dC, ldc, O, stream, launches, vcsr::BType::kF16, "FP16");
}

namespace {

// Device address of a page-locked (pinned or registered) host buffer, or null
// for pageable memory.
const void *mapped_host(const void *h) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, h) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

// Whether the host entry point moves only the touched B rows and the C rows
// holding entries: page-locked buffers aligned to 64 bytes, O a multiple of
// 16 (whole 64-byte lines per row), no tensor-core blocks (their rows are not
// in the row lists), and more than 1/8 of B or C to save.
bool rows_worth_moving(const vcsr_plan *p) {
  return p->n_xcols * 8LL <= p->N * 7LL || p->n_xrows * 8LL <= p->M * 7LL;
}

// Zeroes rows [r0, r1) of every range of the row-major M x O buffer c (O a
// multiple of 16, c 64-byte aligned) on all host threads, with streaming
// stores: a plain store first reads each line into the cache, doubling the
// memory traffic that competes with the PCIe copies.
void zero_rows(float *c, int O, const std::vector<std::pair<int, int>> &ranges) {
#pragma omp parallel
  {
#pragma omp for schedule(dynamic, 1024)
    for (long i = 0; i < (long)ranges.size(); ++i) {
      float *q = c + (size_t)ranges[i].first * O;
      const size_t n = (size_t)(ranges[i].second - ranges[i].first) * O;
#if defined(__SSE2__)
      const __m128i z = _mm_setzero_si128();
      for (size_t k = 0; k < n; k += 4) _mm_stream_si128(reinterpret_cast<__m128i *>(q + k), z);
#else
      std::memset(q, 0, sizeof(float) * n);
#endif
    }
#if defined(__SSE2__)
    _mm_sfence();  // this thread's streaming stores are visible before the call returns
#endif
  }
}

// The host entry point for graph matrices: a copy kernel reads the touched B
// rows from the mapped host buffer, the product runs, another copy kernel
// writes the C rows that hold entries into the mapped host buffer, and host
// threads zero the empty C rows meanwhile.  O is cut into up to four column
// chunks as in the column pipeline, so chunk k's C rows go down while chunk
// k+1's B rows come up.  The copy kernels hold up to half of the SMs; the
// products' grids leave those SMs room, so none of their blocks waits for a
// copy to end.  Measured on one B200 host (R-MAT 2^22, O = 256, 2.06 GB each
// way instead of 4.29 GB): 79-83 ms per call against 108-119 ms for full
// copies on the copy engines; the uploads run at ~43 GB/s alone and ~32 GB/s
// beside the downloads.  *used = false (nothing done) when the conditions of
// rows_worth_moving do not hold.
vcsr_status host_rows_pipeline(vcsr_plan *p, const float *hB, float *hC, int O,
                               cudaStream_t st, bool *used) {
  *used = false;
  if (O % 16 != 0 || p->n_panel_blocks > 0 || p->n_seg_rb > 0 || p->M <= 0 || p->N <= 0 ||
      ((uintptr_t)hB % 64) != 0 || ((uintptr_t)hC % 64) != 0)
    return VCSR_OK;
  const float *dB_host = static_cast<const float *>(mapped_host(hB));
  float *dC_host = static_cast<float *>(const_cast<void *>(mapped_host(hC)));
  if (!dB_host || !dC_host) return VCSR_OK;
  VCSR_TRY(vcsr::host_transfer_lists(p, st));
  if (!rows_worth_moving(p)) return VCSR_OK;
  *used = true;
  if (!p->down) VCSR_CUDA(cudaStreamCreateWithFlags(&p->down, cudaStreamNonBlocking));
  if (!p->comp) VCSR_CUDA(cudaStreamCreateWithFlags(&p->comp, cudaStreamNonBlocking));
  int W = O;
  if (O >= 128) {
    const int nch = std::min(4, O / 64);
    W = (((O + nch - 1) / nch) + 15) & ~15;
  }
  const int n_chunks = (O + W - 1) / W;
  while ((int)p->chunk_done.size() < 2 * n_chunks) {
    cudaEvent_t e;
    VCSR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    p->chunk_done.push_back(e);
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, p->device);
  const int copy_blocks = std::max(1, sms / 2);  // blocks per copy kernel
  const int reserve = std::min(2 * copy_blocks, sms / 2);
  vcsr_status status = VCSR_OK;
  for (int k = 0; k < n_chunks && status == VCSR_OK; ++k) {  // B rows up, back to back
    const int o0 = k * W, w = std::min(W, O - o0);
    status = vcsr::copy_rows(dB_host, p->d_stage_B, O, p->d_xcols, p->n_xcols, o0, w,
                             copy_blocks, st);
    if (status == VCSR_OK) {
      const cudaError_t e = cudaEventRecord(p->chunk_done[k], st);
      if (e != cudaSuccess) status = fail(VCSR_ERR_CUDA, "row upload: %s", cudaGetErrorString(e));
    }
  }
  for (int k = 0; k < n_chunks && status == VCSR_OK; ++k) {
    const int o0 = k * W, w = std::min(W, O - o0);
    cudaError_t e = cudaStreamWaitEvent(p->comp, p->chunk_done[k], 0);
    if (e != cudaSuccess) {
      status = fail(VCSR_ERR_CUDA, "chunk wait: %s", cudaGetErrorString(e));
      break;
    }
    status = vcsr::launch_panel_spmm(view_all(p), false, p->d_stage_B + o0, O, p->d_stage_C + o0, O,
                                     w, p->comp, nullptr, p->side, p->fork, p->join,
                                     vcsr::BType::kF32, reserve);
    if (status != VCSR_OK) break;
    e = cudaEventRecord(p->chunk_done[n_chunks + k], p->comp);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->down, p->chunk_done[n_chunks + k], 0);
    if (e != cudaSuccess) {
      status = fail(VCSR_ERR_CUDA, "chunk download: %s", cudaGetErrorString(e));
      break;
    }
    status = vcsr::copy_rows(p->d_stage_C, dC_host, O, p->d_xrows, p->n_xrows, o0, w,
                             copy_blocks, p->down);
  }
  zero_rows(hC, O, p->empty_rows);  // on the host while the device works
  // every stream drains before returning, also after an error
  const cudaError_t e0 = cudaStreamSynchronize(p->comp);
  const cudaError_t e1 = cudaStreamSynchronize(p->down), e2 = cudaStreamSynchronize(st);
  if (status != VCSR_OK) return status;
  if (e0 != cudaSuccess || e1 != cudaSuccess || e2 != cudaSuccess)
    return fail(VCSR_ERR_CUDA, "host rows pipeline: %s",
                cudaGetErrorString(e0 != cudaSuccess ? e0 : (e1 != cudaSuccess ? e1 : e2)));
  return p->d_err ? vcsr_plan_check(p, (vcsr_stream_t)st) : VCSR_OK;
}

}  // namespace

vcsr_status vcsr_spmm_host(vcsr_plan *p, const float *hB, float *hC, int O,
                           vcsr_stream_t stream) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!p || !hC || (!hB && p->N > 0 && O > 0))
      return fail(VCSR_ERR_INVALID, "null argument");
    if (O < 0) return fail(VCSR_ERR_INVALID, "negative O");
    cudaStream_t st = (cudaStream_t)stream;
    const size_t nb = sizeof(float) * (size_t)p->N * O;
    const size_t nc = sizeof(float) * (size_t)p->M * O;
    if (nb > p->stage_B) {
      cudaFree(p->d_stage_B);
      p->d_stage_B = nullptr;
      p->stage_B = 0;
      VCSR_CUDA(cudaMalloc(&p->d_stage_B, nb));
      p->stage_B = nb;
    }
    if (nc > p->stage_C) {
      cudaFree(p->d_stage_C);
      p->d_stage_C = nullptr;
      p->stage_C = 0;
      VCSR_CUDA(cudaMalloc(&p->d_stage_C, nc));
      p->stage_C = nc;
    }
    constexpr size_t kPipelineBytes = (size_t)8 << 20;
    if (O > 0 && nb + nc >= kPipelineBytes && !(p->n_split_units > 0 && O > p->pstride)) {
      bool used = false;
      VCSR_TRY(host_rows_pipeline(p, hB, hC, O, st, &used));
      if (used) return VCSR_OK;
    }
    if (O > 0 && p->N > 0 && p->M > 0 && nb + nc >= kPipelineBytes && !p->rpanels.empty() &&
        !(p->n_split_units > 0 && O > p->pstride)) {
      // Row pipeline for banded matrices: B goes up in P contiguous row chunks
      // on `stream`, chunk j ending at the highest column that row panels
      // 0..j read (the last one at N); row panel j runs on the plan's compute
      // stream as soon as chunk j is up, and its C rows go back on the
      // download stream.  Used when no panel reads B rows beyond the next
      // equal 1/P share of B, so that the chunks stay balanced and uploads,
      // products and downloads overlap.
      const int P = (int)p->rpanels.size();
      const int per = (p->N + P - 1) / P;
      bool banded = true;
      std::vector<int> cend(P);
      for (int j = 0, c = 0; j < P; ++j) {
        const int cm = p->rpanels[j].col_max;
        if (j + 1 < P && cm >= 0 && cm / per > j + 1) banded = false;
        c = std::max(c, std::min(p->N, cm + 1));
        cend[j] = j == P - 1 ? p->N : c;
      }
      if (banded) {
        if (!p->down) VCSR_CUDA(cudaStreamCreateWithFlags(&p->down, cudaStreamNonBlocking));
        if (!p->comp) VCSR_CUDA(cudaStreamCreateWithFlags(&p->comp, cudaStreamNonBlocking));
        while ((int)p->chunk_done.size() < 2 * P) {
          cudaEvent_t e;
          VCSR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
          p->chunk_done.push_back(e);
        }
        const size_t row_b = sizeof(float) * (size_t)O;
        vcsr_status status = VCSR_OK;
        cudaError_t e = cudaSuccess;
        for (int i = 0; i < P && e == cudaSuccess; ++i) {
          const int r0 = i == 0 ? 0 : cend[i - 1], r1 = cend[i];
          if (r1 > r0)
            e = cudaMemcpyAsync(p->d_stage_B + (size_t)r0 * O, hB + (size_t)r0 * O,
                                row_b * (r1 - r0), cudaMemcpyHostToDevice, st);
          if (e == cudaSuccess) e = cudaEventRecord(p->chunk_done[i], st);
        }
        if (e != cudaSuccess) status = fail(VCSR_ERR_CUDA, "row upload: %s", cudaGetErrorString(e));
        for (int j = 0; j < P && status == VCSR_OK; ++j) {
          const auto &rp = p->rpanels[j];
          e = cudaStreamWaitEvent(p->comp, p->chunk_done[j], 0);
          if (e != cudaSuccess) {
            status = fail(VCSR_ERR_CUDA, "row panel wait: %s", cudaGetErrorString(e));
            break;
          }
          vcsr::PanelDevView v = view(p);
          v.batches += rp.b0;
          v.n_batches = rp.b1 - rp.b0;
          v.long_idx += rp.l0;
          v.n_long = rp.l1 - rp.l0;
          status = vcsr::launch_panel_spmm(v, false, p->d_stage_B, O, p->d_stage_C, O, O, p->comp,
                                           nullptr, p->side, p->fork, p->join);
          if (status != VCSR_OK) break;
          e = cudaEventRecord(p->chunk_done[P + j], p->comp);
          if (e == cudaSuccess) e = cudaStreamWaitEvent(p->down, p->chunk_done[P + j], 0);
          if (e == cudaSuccess && rp.row1 > rp.row0)
            e = cudaMemcpyAsync(hC + (size_t)rp.row0 * O, p->d_stage_C + (size_t)rp.row0 * O,
                                row_b * (rp.row1 - rp.row0), cudaMemcpyDeviceToHost, p->down);
          if (e != cudaSuccess) status = fail(VCSR_ERR_CUDA, "row download: %s", cudaGetErrorString(e));
        }
        // every stream drains before returning, also after an error
        const cudaError_t e1 = cudaStreamSynchronize(p->down), e2 = cudaStreamSynchronize(p->comp),
                          e3 = cudaStreamSynchronize(st);
        if (status != VCSR_OK) return status;
        if (e1 != cudaSuccess || e2 != cudaSuccess || e3 != cudaSuccess)
          return fail(VCSR_ERR_CUDA, "row pipeline: %s",
                      cudaGetErrorString(e1 != cudaSuccess ? e1 : (e2 != cudaSuccess ? e2 : e3)));
        return VCSR_OK;
      }
    }
    // Columns of B and C split into chunks are independent products
    // (C[:, chunk] = A * B[:, chunk]).  With large buffers the call runs as a
    // pipeline of up to four chunks: the chunks go up back to back on
    // `stream`, chunk k is multiplied on the plan's compute stream once it is
    // up and downloaded on the plan's download stream once multiplied, so the
    // two PCIe directions overlap and no upload waits for a product.  Chunk
    // copies are 2-D
    // (w floats out of every row of O); measured on B200 hosts, rows of at
    // least 256 bytes keep both directions at full speed (128-byte rows lose
    // a third), so a chunk is at least 64 floats wide.
    int W = O;
    if (O >= 128 && nb + nc >= kPipelineBytes) {
      const int nch = std::min(4, O / 64);
      W = (int)(((O + nch - 1) / nch + 3) & ~3);
    }
    const int n_chunks = O > 0 ? (O + W - 1) / W : 0;
    if (n_chunks <= 1) {
      if (nb) VCSR_CUDA(cudaMemcpyAsync(p->d_stage_B, hB, nb, cudaMemcpyHostToDevice, st));
      VCSR_TRY(vcsr_spmm(p, p->d_stage_B, O, p->d_stage_C, O, O, stream, nullptr));
      if (nc) VCSR_CUDA(cudaMemcpyAsync(hC, p->d_stage_C, nc, cudaMemcpyDeviceToHost, st));
      VCSR_CUDA(cudaStreamSynchronize(st));
      return p->d_err ? vcsr_plan_check(p, stream) : VCSR_OK;
    }
    if (!p->down) VCSR_CUDA(cudaStreamCreateWithFlags(&p->down, cudaStreamNonBlocking));
    if (!p->comp) VCSR_CUDA(cudaStreamCreateWithFlags(&p->comp, cudaStreamNonBlocking));
    while ((int)p->chunk_done.size() < 2 * n_chunks) {
      cudaEvent_t e;
      VCSR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
      p->chunk_done.push_back(e);
    }
    const size_t pitch = sizeof(float) * (size_t)O;
    vcsr_status status = VCSR_OK;
    cudaError_t e = cudaSuccess;
    for (int k = 0; k < n_chunks && e == cudaSuccess; ++k) {  // uploads, back to back
      const int o0 = k * W, w = std::min(W, O - o0);
      if (p->N > 0)
        e = cudaMemcpy2DAsync(p->d_stage_B + o0, pitch, hB + o0, pitch, sizeof(float) * w,
                              (size_t)p->N, cudaMemcpyHostToDevice, st);
      if (e == cudaSuccess) e = cudaEventRecord(p->chunk_done[k], st);
    }
    if (e != cudaSuccess) status = fail(VCSR_ERR_CUDA, "chunk upload: %s", cudaGetErrorString(e));
    for (int k = 0; k < n_chunks && status == VCSR_OK; ++k) {
      const int o0 = k * W, w = std::min(W, O - o0);
      e = cudaStreamWaitEvent(p->comp, p->chunk_done[k], 0);
      if (e != cudaSuccess) {
        status = fail(VCSR_ERR_CUDA, "chunk wait: %s", cudaGetErrorString(e));
        break;
      }
      status = vcsr_spmm(p, p->d_stage_B + o0, O, p->d_stage_C + o0, O, w, p->comp, nullptr);
      if (status != VCSR_OK) break;
      e = cudaEventRecord(p->chunk_done[n_chunks + k], p->comp);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(p->down, p->chunk_done[n_chunks + k], 0);
      if (e == cudaSuccess && p->M > 0)
        e = cudaMemcpy2DAsync(hC + o0, pitch, p->d_stage_C + o0, pitch, sizeof(float) * w,
                              (size_t)p->M, cudaMemcpyDeviceToHost, p->down);
      if (e != cudaSuccess) status = fail(VCSR_ERR_CUDA, "chunk download: %s", cudaGetErrorString(e));
    }
    // every stream drains before returning, also after an error
    const cudaError_t e0 = cudaStreamSynchronize(p->comp);
    const cudaError_t e1 = cudaStreamSynchronize(p->down), e2 = cudaStreamSynchronize(st);
    if (status != VCSR_OK) return status;
    if (e0 != cudaSuccess || e1 != cudaSuccess || e2 != cudaSuccess)
      return fail(VCSR_ERR_CUDA, "host entry point: %s",
                  cudaGetErrorString(e0 != cudaSuccess ? e0 : (e1 != cudaSuccess ? e1 : e2)));
    return p->d_err ? vcsr_plan_check(p, stream) : VCSR_OK;
  });
}

vcsr_status vcsr_plan_host_rows(vcsr_plan *p, int *b_rows, int *c_rows,
                                vcsr_stream_t stream) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!p || !b_rows || !c_rows) return fail(VCSR_ERR_INVALID, "null argument");
    *b_rows = p->N;
    *c_rows = p->M;
    if (p->n_panel_blocks > 0 || p->n_seg_rb > 0 || p->M <= 0 || p->N <= 0) return VCSR_OK;
    VCSR_TRY(vcsr::host_transfer_lists(p, (cudaStream_t)stream));
    if (!rows_worth_moving(p)) return VCSR_OK;
    *b_rows = p->n_xcols;
    *c_rows = p->n_xrows;
    return VCSR_OK;
  });
}

vcsr_status vcsr_plan_test_withhold_signal(vcsr_plan *p) {
  vcsr::clear_error();
  if (!p) return fail(VCSR_ERR_INVALID, "null plan");
  if (p->n_panel_rb == 0)
    return fail(VCSR_ERR_UNSUPPORTED, "the plan has no TF32 panels (no barrier waits)");
  p->tc_inject.store(1);
  return VCSR_OK;
}

vcsr_status vcsr_plan_check(vcsr_plan *p, vcsr_stream_t stream) {
  vcsr::clear_error();
  if (!p) return fail(VCSR_ERR_INVALID, "null plan");
  cudaStream_t st = (cudaStream_t)stream;
  VCSR_CUDA(cudaStreamSynchronize(st));
  if (!p->d_err) return VCSR_OK;
  int word = 0;
  VCSR_CUDA(cudaMemcpyAsync(&word, p->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  if (!word) return VCSR_OK;
  VCSR_CUDA(cudaMemsetAsync(p->d_err, 0, sizeof(int), st));
  VCSR_CUDA(cudaStreamSynchronize(st));
  char msg[160];
  vcsr::describe_tc_error(word, msg, sizeof msg);
  return fail(VCSR_ERR_TIMEOUT, "%s", msg);
}

}  // extern "C"
