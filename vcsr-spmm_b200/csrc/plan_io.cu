// plan_io.cu — plans saved to and loaded from disk, so that a matrix's
// layout is built once (vcsr_plan_save / vcsr_plan_load).
//
// File: the 8 bytes "VCSRPLAN", then little-endian int64 header fields, then
// every array as (int64 byte count, bytes), then the FNV-1a 64-bit hash of
// everything before it.  A load checks the hash, the header, every array's
// size and every index the kernels follow (columns < N, unit and batch
// bounds, split slots, dense-panel bounds) before it touches the device, so
// a damaged or hand-made file is an error, not an out-of-bounds read.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "common.h"
#include "panel.h"
#include "plan_impl.h"

using vcsr::fail;

namespace {

constexpr char kMagic[8] = {'V', 'C', 'S', 'R', 'P', 'L', 'A', 'N'};
constexpr int64_t kVersion = 4;

uint64_t fnv1a(const unsigned char *p, size_t n) {
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

struct Writer {
  std::vector<unsigned char> buf;
  void raw(const void *p, size_t n) {
    const unsigned char *b = static_cast<const unsigned char *>(p);
    buf.insert(buf.end(), b, b + n);
  }
  void i64(int64_t v) { raw(&v, 8); }
  template <class T>
  void arr(const std::vector<T> &v) {
    i64((int64_t)(v.size() * sizeof(T)));
    raw(v.data(), v.size() * sizeof(T));
  }
};

struct Reader {
  const unsigned char *p, *end;
  bool ok = true;
  int64_t i64() {
    int64_t v = 0;
    if (end - p < 8) { ok = false; return 0; }
    std::memcpy(&v, p, 8);
    p += 8;
    return v;
  }
  // reads an array that must hold exactly n elements
  template <class T>
  std::vector<T> arr(int64_t n) {
    std::vector<T> v;
    const int64_t bytes = i64();
    if (!ok || n < 0 || bytes != n * (int64_t)sizeof(T) || end - p < bytes) {
      ok = false;
      return v;
    }
    v.resize((size_t)n);
    if (bytes) std::memcpy(v.data(), p, (size_t)bytes);
    p += bytes;
    return v;
  }
};

template <class T>
vcsr_status download(std::vector<T> &out, const T *d, int64_t n) {
  out.resize((size_t)(n > 0 ? n : 0));
  if (n > 0) VCSR_CUDA(cudaMemcpy(out.data(), d, sizeof(T) * (size_t)n, cudaMemcpyDeviceToHost));
  return VCSR_OK;
}

// Device copy of n host elements (plain allocation, for the VCSR arrays).
template <class T>
vcsr_status upload_n(T **dst, const std::vector<T> &src, cudaStream_t st) {
  VCSR_CUDA(cudaMalloc((void **)dst, sizeof(T) * (src.size() ? src.size() : 1)));
  if (!src.empty())
    VCSR_CUDA(cudaMemcpyAsync(*dst, src.data(), sizeof(T) * src.size(), cudaMemcpyHostToDevice,
                              st));
  return VCSR_OK;
}

// Everything a plan holds, on the host.
struct HostPlan {
  std::vector<int> ucol, long_idx, vec_ptr, rb_row, rb_ptr, blk_col, rpan;
  std::vector<unsigned> umask;
  std::vector<int> seg_rb, seg_pp, seg_rp, seg_col;
  std::vector<int4> seg_pieces;
  std::vector<float> seg_a, seg_val;
  std::vector<float> uval, blk_val;
  std::vector<int4> units, batches;
  std::vector<int2> parts, svecs;
  std::vector<int> g_ptr, g_depth, g_seg, g_rows, g_lcol, g_sgs;
  std::vector<float> g_val;
};

}  // namespace

extern "C" {

vcsr_status vcsr_plan_save(const vcsr_plan *p, const char *path) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!p || !path) return fail(VCSR_ERR_INVALID, "null argument");
    HostPlan h;
    VCSR_TRY(download(h.ucol, p->d_ucol, p->num_union));
    VCSR_TRY(download(h.uval, p->d_uval, p->num_union * p->R));
    if (p->R > 1) VCSR_TRY(download(h.umask, p->d_umask, p->num_union));
    VCSR_TRY(download(h.units, p->d_units, p->n_units));
    VCSR_TRY(download(h.batches, p->d_batches, p->n_batches));
    VCSR_TRY(download(h.long_idx, p->d_long, p->n_long));
    VCSR_TRY(download(h.vec_ptr, p->d_vec_ptr, (int64_t)p->num_vectors + 1));
    VCSR_TRY(download(h.parts, p->d_parts, p->n_split_units));
    VCSR_TRY(download(h.svecs, p->d_svecs, p->n_split_vectors));
    if (p->n_panel_rb > 0) {
      VCSR_TRY(download(h.rb_row, p->d_rb_row, p->n_panel_rb));
      VCSR_TRY(download(h.rb_ptr, p->d_rb_ptr, (int64_t)p->n_panel_rb + 1));
      VCSR_TRY(download(h.blk_col, p->d_blk_col, p->n_panel_blocks));
      VCSR_TRY(download(h.blk_val, p->d_blk_val, (int64_t)p->n_panel_blocks * 256));
    }
    if (p->n_seg_rb > 0) {
    VCSR_TRY(download(h.seg_rb, p->d_seg_rb_row, p->n_seg_rb));
    VCSR_TRY(download(h.seg_pp, p->d_seg_pp, (int64_t)p->n_seg_rb + 1));
    VCSR_TRY(download(h.seg_pieces, p->d_seg_pieces, p->n_seg_pieces));
    VCSR_TRY(download(h.seg_a, p->d_seg_a, (int64_t)p->seg_rows * 16));
    VCSR_TRY(download(h.seg_rp, p->d_seg_rp, (int64_t)p->M + 1));
    VCSR_TRY(download(h.seg_col, p->d_seg_col, p->nnz));
    VCSR_TRY(download(h.seg_val, p->d_seg_val, p->nnz));
  }
  for (const auto &r : p->rpanels)
      for (int v : {r.row0, r.row1, r.b0, r.b1, r.l0, r.l1, r.col_max}) h.rpan.push_back(v);
    const vcsr_vcsr &g = p->ref;
    if (p->has_ref) {
      VCSR_TRY(download(h.g_ptr, g.group_ptr, (int64_t)g.num_groups + 1));
      VCSR_TRY(download(h.g_depth, g.group_depth, g.num_groups));
      VCSR_TRY(download(h.g_seg, g.group_seg_base, g.num_groups));
      VCSR_TRY(download(h.g_rows, g.group_rows, (int64_t)g.num_groups * g.bundle));
      VCSR_TRY(download(h.g_lcol, g.lcol, g.num_slots));
      VCSR_TRY(download(h.g_val, g.val, g.num_slots));
      VCSR_TRY(download(h.g_sgs, g.segment_group_start, (int64_t)g.num_segments + 1));
    }
    Writer w;
    w.raw(kMagic, 8);
    const vcsr_plan_params &q = p->params;
    for (int64_t v :
         {kVersion, (int64_t)VCSR_ABI_VERSION, (int64_t)p->M, (int64_t)p->N, (int64_t)p->nnz,
          (int64_t)p->R, (int64_t)p->num_vectors, p->num_union, (int64_t)p->chunk,
          (int64_t)p->n_units, (int64_t)p->n_split_units, (int64_t)p->n_split_vectors,
          (int64_t)p->n_batches, (int64_t)p->n_long, (int64_t)p->pstride,
          (int64_t)p->counter_stride, (int64_t)p->n_panel_rb, (int64_t)p->n_panel_blocks,
          p->panel_nnz, (int64_t)p->rpanels.size(), (int64_t)q.segw, (int64_t)q.bundle,
          (int64_t)q.tileK, (int64_t)q.max_O, (int64_t)q.vec_rows, (int64_t)q.chunk,
          (int64_t)(q.flags & ~VCSR_PLAN_HOST_BUILD), (int64_t)q.panel_min_nnz, (int64_t)(p->has_ref ? 1 : 0),
          (int64_t)g.M, (int64_t)g.N, (int64_t)g.segw, (int64_t)g.bundle, (int64_t)g.num_groups,
          (int64_t)g.num_segments, g.num_slots, (int64_t)q.target_O, (int64_t)q.seg_min_run,
        (int64_t)p->n_seg_rb, (int64_t)p->n_seg_pieces, (int64_t)p->seg_rows,
        (int64_t)p->seg_min_run, (int64_t)(p->seg_only ? 1 : 0)})
      w.i64(v);
    w.arr(h.ucol); w.arr(h.uval); w.arr(h.umask); w.arr(h.units); w.arr(h.batches); w.arr(h.long_idx);
    w.arr(h.vec_ptr); w.arr(h.parts); w.arr(h.svecs); w.arr(h.rb_row); w.arr(h.rb_ptr);
    w.arr(h.blk_col); w.arr(h.blk_val); w.arr(h.rpan);
    w.arr(h.g_ptr); w.arr(h.g_depth); w.arr(h.g_seg); w.arr(h.g_rows); w.arr(h.g_lcol);
    w.arr(h.g_val); w.arr(h.g_sgs);
  w.arr(h.seg_rb); w.arr(h.seg_pp); w.arr(h.seg_pieces); w.arr(h.seg_a); w.arr(h.seg_rp);
  w.arr(h.seg_col); w.arr(h.seg_val);
    const uint64_t hash = fnv1a(w.buf.data(), w.buf.size());
    w.raw(&hash, 8);
    // write beside the target, then rename: a reader never sees half a file
    const std::string tmp = std::string(path) + ".tmp";
    FILE *f = fopen(tmp.c_str(), "wb");
    if (!f) return fail(VCSR_ERR_IO, "cannot write %s", tmp.c_str());
    const size_t n = fwrite(w.buf.data(), 1, w.buf.size(), f);
    const int c = fclose(f);
    if (n != w.buf.size() || c != 0 || rename(tmp.c_str(), path) != 0) {
      remove(tmp.c_str());
      return fail(VCSR_ERR_IO, "cannot write %s", path);
    }
    return VCSR_OK;
  });
}

vcsr_status vcsr_plan_load(const char *path, vcsr_plan **out, vcsr_stream_t stream) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!path || !out) return fail(VCSR_ERR_INVALID, "null argument");
    *out = nullptr;
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<unsigned char> buf;
    {
      FILE *f = fopen(path, "rb");
      if (!f) return fail(VCSR_ERR_IO, "cannot open plan file %s", path);
      unsigned char chunk[1 << 16];
      size_t n;
      while ((n = fread(chunk, 1, sizeof chunk, f)) > 0) buf.insert(buf.end(), chunk, chunk + n);
      fclose(f);
    }
    if (buf.size() < 16 || std::memcmp(buf.data(), kMagic, 8) != 0)
      return fail(VCSR_ERR_IO, "%s is not a plan file", path);
    uint64_t hash;
    std::memcpy(&hash, buf.data() + buf.size() - 8, 8);
    if (fnv1a(buf.data(), buf.size() - 8) != hash)
      return fail(VCSR_ERR_IO, "plan file %s is damaged (checksum)", path);
    Reader r{buf.data() + 8, buf.data() + buf.size() - 8};
    const int64_t version = r.i64(), abi = r.i64();
    if (!r.ok || version != kVersion || abi != VCSR_ABI_VERSION)
      return fail(VCSR_ERR_UNSUPPORTED, "plan file version %lld (ABI %lld); this library reads %lld (ABI %d)",
                  (long long)version, (long long)abi, (long long)kVersion, VCSR_ABI_VERSION);
    int64_t hv[41];
    for (int64_t &v : hv) v = r.i64();
    if (!r.ok) return fail(VCSR_ERR_IO, "plan file %s is truncated", path);
    const int64_t M = hv[0], N = hv[1], nnz = hv[2], R = hv[3], nv = hv[4], nu = hv[5],
                  chunk = hv[6], n_units = hv[7], n_su = hv[8], n_sv = hv[9], n_b = hv[10],
                  n_l = hv[11], pstride = hv[12], cstride = hv[13], n_rb = hv[14],
                  n_blk = hv[15], panel_nnz = hv[16], n_rp = hv[17];
    const int64_t has_ref = hv[26];
  const int64_t s_rb = hv[36], s_np = hv[37], s_rows = hv[38], s_min = hv[39], s_only = hv[40];
    const int64_t gM = hv[27], gN = hv[28], g_segw = hv[29], g_bundle = hv[30], g_G = hv[31],
                  g_S = hv[32], g_P = hv[33];
    const int64_t i32 = INT32_MAX;
    bool ok = M >= 0 && M <= i32 && N >= 0 && N <= i32 && nnz >= 0 && nnz <= i32 &&
              (R == 1 || R == 2 || R == 4 || R == 8 || R == 16) && nv == (M + R - 1) / R &&
              nu >= 0 && nu * R <= (int64_t)1 << 40 && n_units >= nv && n_units <= i32 &&
              n_su >= 0 && n_su <= n_units && n_sv >= 0 && n_sv <= n_su && n_b >= 0 &&
              n_l >= 0 && n_l <= n_units && pstride >= 1 && pstride <= i32 && cstride >= 1 &&
              cstride <= i32 && n_rb >= 0 && n_rb <= (M + 15) / 16 && n_blk >= n_rb &&
              n_blk <= i32 && panel_nnz >= 0 && n_rp >= 0 && n_rp <= 1024 && chunk >= 0 &&
              (has_ref == 0 || has_ref == 1) && s_rb >= 0 && s_rb <= (M + 15) / 16 &&
            s_np >= s_rb && s_np <= i32 && s_rows >= 0 && s_rows * 16 <= i32 && s_min >= 0 &&
            (s_only == 0 || s_only == 1) && !(s_rb > 0 && n_rb > 0);
    if (has_ref)
      ok = ok && gM == M && gN == N && g_segw > 0 && g_bundle > 0 && g_G >= 0 && g_G <= i32 &&
           g_S >= 0 && g_S <= i32 && g_P >= 0 && g_P <= i32;
    if (!ok) return fail(VCSR_ERR_IO, "plan file %s has an invalid header", path);
    HostPlan h;
    h.ucol = r.arr<int>(nu);
    h.uval = r.arr<float>(nu * R);
    h.umask = r.arr<unsigned>(R > 1 ? nu : 0);
    h.units = r.arr<int4>(n_units);
    h.batches = r.arr<int4>(n_b);
    h.long_idx = r.arr<int>(n_l);
    h.vec_ptr = r.arr<int>(nv + 1);
    h.parts = r.arr<int2>(n_su);
    h.svecs = r.arr<int2>(n_sv);
    h.rb_row = r.arr<int>(n_rb);
    h.rb_ptr = r.arr<int>(n_rb ? n_rb + 1 : 0);
    h.blk_col = r.arr<int>(n_rb ? n_blk : 0);
    h.blk_val = r.arr<float>(n_rb ? n_blk * 256 : 0);
    h.rpan = r.arr<int>(n_rp * 7);
    h.g_ptr = r.arr<int>(has_ref ? g_G + 1 : 0);
    h.g_depth = r.arr<int>(has_ref ? g_G : 0);
    h.g_seg = r.arr<int>(has_ref ? g_G : 0);
    h.g_rows = r.arr<int>(has_ref ? g_G * g_bundle : 0);
    h.g_lcol = r.arr<int>(has_ref ? g_P : 0);
    h.g_val = r.arr<float>(has_ref ? g_P : 0);
    h.g_sgs = r.arr<int>(has_ref ? g_S + 1 : 0);
  h.seg_rb = r.arr<int>(s_rb);
  h.seg_pp = r.arr<int>(s_rb ? s_rb + 1 : 0);
  h.seg_pieces = r.arr<int4>(s_rb ? s_np : 0);
  h.seg_a = r.arr<float>(s_rb ? s_rows * 16 : 0);
  h.seg_rp = r.arr<int>(s_rb ? M + 1 : 0);
  h.seg_col = r.arr<int>(s_rb ? nnz : 0);
  h.seg_val = r.arr<float>(s_rb ? nnz : 0);
    if (!r.ok || r.p != r.end) return fail(VCSR_ERR_IO, "plan file %s has bad array sizes", path);
    // every index the kernels follow
    for (int c : h.ucol) ok = ok && c >= 0 && c < N;
    for (unsigned m : h.umask) ok = ok && m != 0 && (m >> R) == 0;
    ok = ok && h.vec_ptr[0] == 0 && h.vec_ptr[(size_t)nv] == nu;
    for (int64_t v = 0; v < nv && ok; ++v) ok = h.vec_ptr[(size_t)v] <= h.vec_ptr[(size_t)v + 1];
    for (const int4 &u : h.units)
      ok = ok && u.x >= 0 && u.x < nv && u.y >= h.vec_ptr[(size_t)u.x] && u.y <= u.z &&
           u.z <= h.vec_ptr[(size_t)u.x + 1] && u.w >= -1 && u.w < n_su;
    for (const int4 &b : h.batches)
      ok = ok && b.x >= 0 && b.x < b.y && b.y <= nv && b.y - b.x <= 64 &&
           b.z == h.vec_ptr[(size_t)b.x] && b.w == h.vec_ptr[(size_t)b.y];
    for (int u : h.long_idx) ok = ok && u >= 0 && u < n_units;
    for (const int2 &q : h.parts) ok = ok && q.x >= 0 && q.x < n_sv && q.y >= 0;
    for (const int2 &q : h.svecs) ok = ok && q.x >= 0 && q.y >= 1 && q.x + q.y <= n_su;
    if (n_rb) {
      ok = ok && h.rb_ptr[0] == 0 && h.rb_ptr[(size_t)n_rb] == n_blk;
      for (int64_t k = 0; k < n_rb && ok; ++k)
        ok = h.rb_row[(size_t)k] >= 0 && h.rb_row[(size_t)k] < M && h.rb_row[(size_t)k] % 16 == 0 &&
             h.rb_ptr[(size_t)k] < h.rb_ptr[(size_t)k + 1];
      for (int c : h.blk_col) ok = ok && c >= 0 && (int64_t)c * 16 < N;
    }
    for (int64_t j = 0; j < n_rp && ok; ++j) {
      const int *q = &h.rpan[(size_t)j * 7];
      ok = q[0] >= 0 && q[0] <= q[1] && q[1] <= M && q[2] >= 0 && q[2] <= q[3] && q[3] <= n_b &&
           q[4] >= 0 && q[4] <= q[5] && q[5] <= n_l && q[6] >= -1 && q[6] < N;
    }
    if (has_ref) {
      ok = ok && h.g_ptr[0] == 0 && h.g_ptr[(size_t)g_G] == g_P;
      for (int64_t k = 0; k < g_G && ok; ++k)
        ok = h.g_ptr[(size_t)k] <= h.g_ptr[(size_t)k + 1] && h.g_depth[(size_t)k] >= 0 &&
             h.g_seg[(size_t)k] >= 0 && h.g_seg[(size_t)k] < N;
      for (int x : h.g_rows) ok = ok && x >= -1 && x < M;
      for (int x : h.g_lcol) ok = ok && x >= -1 && x < g_segw;
      for (int x : h.g_sgs) ok = ok && x >= 0 && x <= g_G;
    }
    if (s_rb) {
    ok = ok && h.seg_pp[0] == 0 && h.seg_pp[(size_t)s_rb] == s_np;
    for (int64_t k = 0; k < s_rb && ok; ++k)
      ok = h.seg_rb[(size_t)k] >= 0 && h.seg_rb[(size_t)k] < M && h.seg_rb[(size_t)k] % 16 == 0 &&
           h.seg_pp[(size_t)k] < h.seg_pp[(size_t)k + 1];
    for (const int4 &q : h.seg_pieces)
      ok = ok && q.x >= 0 && q.x < N && q.y >= 8 && q.y <= 32 && q.y % 8 == 0 && q.z >= 0 &&
           q.z % 8 == 0 && (int64_t)q.z + q.y <= s_rows;
    ok = ok && h.seg_rp[0] == 0 && h.seg_rp[(size_t)M] == nnz;
    for (int64_t k = 0; k < M && ok; ++k) ok = h.seg_rp[(size_t)k] <= h.seg_rp[(size_t)k + 1];
    for (int c : h.seg_col) ok = ok && c >= 0 && c < N;
  }
  if (!ok) return fail(VCSR_ERR_IO, "plan file %s has out-of-range indices", path);

    // the device side
    vcsr_plan *p = new (std::nothrow) vcsr_plan();
    if (!p) return fail(VCSR_ERR_ALLOC, "out of host memory");
    cudaStream_t st = (cudaStream_t)stream;
    p->M = (int)M; p->N = (int)N; p->nnz = (int)nnz; p->R = (int)R;
    p->num_vectors = (int)nv; p->num_union = nu; p->chunk = (int)chunk;
    p->n_units = (int)n_units; p->n_split_units = (int)n_su; p->n_split_vectors = (int)n_sv;
    p->n_batches = (int)n_b; p->n_long = (int)n_l;
    p->pstride = (int)pstride; p->counter_stride = (int)cstride;
    p->n_panel_rb = (int)n_rb; p->n_panel_blocks = n_rb ? (int)n_blk : 0; p->panel_nnz = panel_nnz;
    p->params.segw = (int)hv[18]; p->params.bundle = (int)hv[19]; p->params.tileK = (int)hv[20];
    p->params.max_O = (int)hv[21]; p->params.vec_rows = (int)hv[22]; p->params.chunk = (int)hv[23];
    p->params.flags = (int)hv[24]; p->params.panel_min_nnz = (int)hv[25];
    p->params.target_O = (int)hv[34];
  p->params.seg_min_run = (int)hv[35];
  p->n_seg_rb = (int)s_rb;
  p->n_seg_pieces = s_rb ? (int)s_np : 0;
  p->seg_rows = s_rb ? (int)s_rows : 0;
  p->seg_min_run = (int)s_min;
  p->seg_only = s_only == 1;
    cudaGetDevice(&p->device);
    for (int64_t j = 0; j < n_rp; ++j) {
      const int *q = &h.rpan[(size_t)j * 7];
      p->rpanels.push_back({q[0], q[1], q[2], q[3], q[4], q[5], q[6]});
    }
    vcsr_status s;
    std::vector<int> zero1(1, 0);
    if ((s = vcsr::upload(&p->d_ucol, h.ucol, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_uval, h.uval, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_umask, h.umask, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_units, h.units, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_parts, h.parts, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_svecs, h.svecs, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_batches, h.batches, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_long, h.long_idx, st, &p->panel_bytes)) ||
        (s = vcsr::upload(&p->d_vec_ptr, h.vec_ptr, st, &p->panel_bytes)) ||
        (n_rb && ((s = vcsr::upload(&p->d_rb_row, h.rb_row, st, &p->panel_bytes)) ||
                  (s = vcsr::upload(&p->d_rb_ptr, h.rb_ptr, st, &p->panel_bytes)) ||
                  (s = vcsr::upload(&p->d_blk_col, h.blk_col, st, &p->panel_bytes)) ||
                  (s = vcsr::upload(&p->d_blk_val, h.blk_val, st, &p->panel_bytes)) ||
                  (s = vcsr::upload(&p->d_err, zero1, st, &p->panel_bytes)))) ||
      (s_rb && ((s = vcsr::upload(&p->d_seg_rb_row, h.seg_rb, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_seg_pp, h.seg_pp, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_seg_pieces, h.seg_pieces, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_seg_a, h.seg_a, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_seg_rp, h.seg_rp, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_seg_col, h.seg_col, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_seg_val, h.seg_val, st, &p->panel_bytes)) ||
                (s = vcsr::upload(&p->d_err, zero1, st, nullptr)))) ||
        (s = vcsr::plan_finish(p, st))) {
      vcsr::plan_release(p);
      delete p;
      return s;
    }
    if (has_ref) {
      vcsr_vcsr &g = p->ref;
      g.M = (int)gM; g.N = (int)gN; g.segw = (int)g_segw; g.bundle = (int)g_bundle;
      g.num_groups = (int)g_G; g.num_segments = (int)g_S; g.num_slots = g_P;
      p->has_ref = true;  // freed with the plan from here on
      if ((s = upload_n(&g.group_ptr, h.g_ptr, st)) || (s = upload_n(&g.group_depth, h.g_depth, st)) ||
          (s = upload_n(&g.group_seg_base, h.g_seg, st)) || (s = upload_n(&g.group_rows, h.g_rows, st)) ||
          (s = upload_n(&g.lcol, h.g_lcol, st)) || (s = upload_n(&g.val, h.g_val, st)) ||
          (s = upload_n(&g.segment_group_start, h.g_sgs, st))) {
        cudaStreamSynchronize(st);
        vcsr::plan_release(p);
        delete p;
        return s;
      }
    }
    const cudaError_t e = cudaStreamSynchronize(st);  // the host copies die here
    if (e != cudaSuccess) {
      vcsr::plan_release(p);
      delete p;
      return fail(VCSR_ERR_CUDA, "plan upload: %s", cudaGetErrorString(e));
    }
    p->build_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0)
                      .count();
    *out = p;
    return VCSR_OK;
  });
}

}  // extern "C"
