// mgpu.cu — row panels of A on several GPUs of one process.
//
// The reference has no multi-GPU path (it pins device 0, src/kernels.cu:129).
// Here A is cut into nnz-balanced row panels (vcsr_partition_rows, cuts
// aligned to `bundle` rows), each GPU gets its own plan for its panel, B is
// replicated by one ncclBroadcast from the first GPU over NVLink, and each
// GPU writes its own rows of C (disjoint, so nothing is reduced).  Each GPU
// reads B only from its own HBM copy.
//
// NCCL is resolved at run time from libnccl.so.2 (whichever copy the process
// already has, e.g. PyTorch's, or the system one), so linking the library
// does not pin an NCCL build.  Every wait on NCCL work is a polling loop with
// a 60 s limit; on expiry the communicators are aborted and the call returns
// VCSR_ERR_TIMEOUT.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "common.h"

using vcsr::fail;

namespace {

struct NcclApi {
  void *h = nullptr;
  ncclResult_t (*CommInitAll)(ncclComm_t *, int, const int *) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int,
                            ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

vcsr_status load_nccl(NcclApi &a) {
  if (a.h) return VCSR_OK;
  a.h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!a.h) a.h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!a.h) return fail(VCSR_ERR_NCCL, "cannot load libnccl.so.2: %s", dlerror());
#define LOAD(f)                                                               \
  a.f = reinterpret_cast<decltype(a.f)>(dlsym(a.h, "nccl" #f));               \
  if (!a.f) return fail(VCSR_ERR_NCCL, "libnccl lacks nccl" #f);
  LOAD(CommInitAll) LOAD(CommDestroy) LOAD(CommAbort) LOAD(Broadcast)
  LOAD(GroupStart) LOAD(GroupEnd) LOAD(GetErrorString)
#undef LOAD
  return VCSR_OK;
}

constexpr double kWaitLimitS = 60.0;

}  // namespace

struct vcsr_mgpu {
  NcclApi nccl;
  int n = 0;
  int M = 0, N = 0, nnz = 0;
  std::vector<int> devs, cuts;
  std::vector<vcsr_plan *> plans;
  std::vector<ncclComm_t> comms;
  std::vector<cudaStream_t> streams;
  std::vector<float *> dB, dC;
  std::vector<cudaEvent_t> ev0, ev1;
  int O = 0;
};

namespace {

// Poll every stream until idle or the limit passes; abort NCCL on expiry.
vcsr_status wait_all(vcsr_mgpu *m, bool abort_on_timeout) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    bool busy = false;
    for (int i = 0; i < m->n; ++i) {
      cudaSetDevice(m->devs[i]);
      cudaError_t e = cudaStreamQuery(m->streams[i]);
      if (e == cudaErrorNotReady) busy = true;
      else if (e != cudaSuccess)
        return fail(VCSR_ERR_CUDA, "device %d: %s", m->devs[i], cudaGetErrorString(e));
    }
    if (!busy) return VCSR_OK;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
        kWaitLimitS) {
      if (abort_on_timeout)
        for (auto c : m->comms)
          if (c) m->nccl.CommAbort(c);
      m->comms.assign(m->comms.size(), nullptr);
      return fail(VCSR_ERR_TIMEOUT, "multi-GPU wait exceeded %.0f s; NCCL aborted",
                  kWaitLimitS);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void release(vcsr_mgpu *m) {
  for (int i = 0; i < m->n; ++i) {
    cudaSetDevice(m->devs[i]);
    if (i < (int)m->plans.size() && m->plans[i]) vcsr_plan_destroy(m->plans[i]);
    if (i < (int)m->dB.size()) cudaFree(m->dB[i]);
    if (i < (int)m->dC.size()) cudaFree(m->dC[i]);
    if (i < (int)m->ev0.size() && m->ev0[i]) cudaEventDestroy(m->ev0[i]);
    if (i < (int)m->ev1.size() && m->ev1[i]) cudaEventDestroy(m->ev1[i]);
    if (i < (int)m->streams.size() && m->streams[i]) cudaStreamDestroy(m->streams[i]);
    if (i < (int)m->comms.size() && m->comms[i]) m->nccl.CommDestroy(m->comms[i]);
  }
}

}  // namespace

extern "C" {

vcsr_status vcsr_mgpu_create(const vcsr_csr *csr, int ngpus, const int *devices,
                             const vcsr_plan_params *params, vcsr_mgpu **out) {
  return vcsr::no_throw([&]() -> vcsr_status {
    vcsr::clear_error();
    if (!csr || !params || !out || ngpus <= 0) return fail(VCSR_ERR_INVALID, "bad arguments");
    *out = nullptr;
    int ndev = 0;
    VCSR_CUDA(cudaGetDeviceCount(&ndev));
    auto *m = new vcsr_mgpu();
    m->n = ngpus;
    m->M = csr->M; m->N = csr->N; m->nnz = csr->nnz;
    for (int i = 0; i < ngpus; ++i) {
      const int d = devices ? devices[i] : i;
      if (d < 0 || d >= ndev) {
        delete m;
        return fail(VCSR_ERR_INVALID, "device %d not visible (%d devices)", d, ndev);
      }
      m->devs.push_back(d);
    }
    vcsr_status s = load_nccl(m->nccl);
    if (s != VCSR_OK) { delete m; return s; }
    m->cuts.assign(ngpus + 1, 0);
    s = vcsr_partition_rows(csr->row_ptr, csr->M, ngpus, params->bundle, m->cuts.data());
    if (s != VCSR_OK) { delete m; return s; }
    m->plans.assign(ngpus, nullptr);
    m->streams.assign(ngpus, nullptr);
    m->ev0.assign(ngpus, nullptr);
    m->ev1.assign(ngpus, nullptr);
    m->dB.assign(ngpus, nullptr);
    m->dC.assign(ngpus, nullptr);
    m->comms.assign(ngpus, nullptr);
    for (int i = 0; i < ngpus; ++i) {
      cudaSetDevice(m->devs[i]);
      cudaError_t e = cudaStreamCreateWithFlags(&m->streams[i], cudaStreamNonBlocking);
      if (e == cudaSuccess) e = cudaEventCreate(&m->ev0[i]);
      if (e == cudaSuccess) e = cudaEventCreate(&m->ev1[i]);
      if (e != cudaSuccess) {
        release(m); delete m;
        return fail(VCSR_ERR_CUDA, "%s", cudaGetErrorString(e));
      }
      vcsr_csr panel{};
      s = vcsr_csr_row_panel(csr, m->cuts[i], m->cuts[i + 1], &panel);
      if (s == VCSR_OK) s = vcsr_plan_create(&panel, VCSR_HOST, params, &m->plans[i],
                                             m->streams[i]);
      vcsr_csr_free(&panel, VCSR_HOST);
      if (s != VCSR_OK) { release(m); delete m; return s; }
    }
    ncclResult_t r = m->nccl.CommInitAll(m->comms.data(), ngpus, m->devs.data());
    if (r != ncclSuccess) {
      m->comms.assign(ngpus, nullptr);
      release(m); delete m;
      return fail(VCSR_ERR_NCCL, "ncclCommInitAll: %s", m->nccl.GetErrorString(r));
    }
    *out = m;
    return VCSR_OK;
  });
}

namespace {

// One grouped broadcast of B (nb floats) from device 0 to every device, each
// enqueue's result checked: a failed ncclBroadcast ends the group and is
// reported with NCCL's message.
vcsr_status broadcast_b(vcsr_mgpu *m, size_t nb) {
  ncclResult_t r = m->nccl.GroupStart();
  if (r != ncclSuccess) return fail(VCSR_ERR_NCCL, "ncclGroupStart: %s", m->nccl.GetErrorString(r));
  for (int i = 0; i < m->n; ++i) {
    cudaSetDevice(m->devs[i]);
    r = m->nccl.Broadcast(m->dB[i], m->dB[i], nb, ncclFloat, 0, m->comms[i], m->streams[i]);
    if (r != ncclSuccess) {
      m->nccl.GroupEnd();
      return fail(VCSR_ERR_NCCL, "ncclBroadcast: %s", m->nccl.GetErrorString(r));
    }
  }
  r = m->nccl.GroupEnd();
  if (r != ncclSuccess) return fail(VCSR_ERR_NCCL, "ncclGroupEnd: %s", m->nccl.GetErrorString(r));
  return VCSR_OK;
}

}  // namespace

vcsr_status vcsr_mgpu_set_b(vcsr_mgpu *m, const float *hB, int O, float *bcast_ms) {
  vcsr::clear_error();
  if (!m || O <= 0 || (!hB && m->N > 0)) return fail(VCSR_ERR_INVALID, "bad arguments");
  const size_t nb = (size_t)m->N * O;
  for (int i = 0; i < m->n; ++i) {
    cudaSetDevice(m->devs[i]);
    cudaFree(m->dB[i]);
    cudaFree(m->dC[i]);
    m->dB[i] = m->dC[i] = nullptr;
    const size_t rows = (size_t)(m->cuts[i + 1] - m->cuts[i]);
    VCSR_CUDA(cudaMalloc(&m->dB[i], sizeof(float) * (nb ? nb : 1)));
    VCSR_CUDA(cudaMalloc(&m->dC[i], sizeof(float) * (rows * O ? rows * O : 1)));
  }
  m->O = O;
  cudaSetDevice(m->devs[0]);
  VCSR_CUDA(cudaMemcpyAsync(m->dB[0], hB, sizeof(float) * nb, cudaMemcpyHostToDevice,
                            m->streams[0]));
  VCSR_CUDA(cudaStreamSynchronize(m->streams[0]));
  // the first broadcast on a buffer carries NCCL's set-up; run it untimed
  VCSR_TRY(broadcast_b(m, nb));
  VCSR_TRY(wait_all(m, true));
  for (int i = 0; i < m->n; ++i) {
    cudaSetDevice(m->devs[i]);
    VCSR_CUDA(cudaEventRecord(m->ev0[i], m->streams[i]));
  }
  VCSR_TRY(broadcast_b(m, nb));
  for (int i = 0; i < m->n; ++i) {
    cudaSetDevice(m->devs[i]);
    VCSR_CUDA(cudaEventRecord(m->ev1[i], m->streams[i]));
  }
  VCSR_TRY(wait_all(m, true));
  float mx = 0.f;
  for (int i = 0; i < m->n; ++i) {
    float t = 0.f;
    cudaSetDevice(m->devs[i]);
    VCSR_CUDA(cudaEventElapsedTime(&t, m->ev0[i], m->ev1[i]));
    mx = t > mx ? t : mx;
  }
  if (bcast_ms) *bcast_ms = mx;
  return VCSR_OK;
}

vcsr_status vcsr_mgpu_spmm(vcsr_mgpu *m, int O, float *ms) {
  vcsr::clear_error();
  if (!m || O != m->O) return fail(VCSR_ERR_INVALID, "call vcsr_mgpu_set_b with this O first");
  for (int i = 0; i < m->n; ++i) {
    cudaSetDevice(m->devs[i]);
    VCSR_CUDA(cudaEventRecord(m->ev0[i], m->streams[i]));
    VCSR_TRY(vcsr_spmm(m->plans[i], m->dB[i], O, m->dC[i], O, O, m->streams[i], nullptr));
    VCSR_CUDA(cudaEventRecord(m->ev1[i], m->streams[i]));
  }
  VCSR_TRY(wait_all(m, false));
  float mx = 0.f;
  for (int i = 0; i < m->n; ++i) {
    float t = 0.f;
    cudaSetDevice(m->devs[i]);
    VCSR_CUDA(cudaEventElapsedTime(&t, m->ev0[i], m->ev1[i]));
    mx = t > mx ? t : mx;
  }
  if (ms) *ms = mx;
  return VCSR_OK;
}

vcsr_status vcsr_mgpu_gather_c(vcsr_mgpu *m, float *hC) {
  vcsr::clear_error();
  if (!m || !hC || m->O <= 0) return fail(VCSR_ERR_INVALID, "bad arguments");
  for (int i = 0; i < m->n; ++i) {
    const size_t rows = (size_t)(m->cuts[i + 1] - m->cuts[i]);
    if (!rows) continue;
    cudaSetDevice(m->devs[i]);
    VCSR_CUDA(cudaMemcpyAsync(hC + (size_t)m->cuts[i] * m->O, m->dC[i],
                              sizeof(float) * rows * m->O, cudaMemcpyDeviceToHost,
                              m->streams[i]));
  }
  return wait_all(m, false);
}

vcsr_status vcsr_mgpu_cuts(const vcsr_mgpu *m, int *cuts) {
  vcsr::clear_error();
  if (!m || !cuts) return fail(VCSR_ERR_INVALID, "null argument");
  std::memcpy(cuts, m->cuts.data(), sizeof(int) * m->cuts.size());
  return VCSR_OK;
}

void vcsr_mgpu_destroy(vcsr_mgpu *m) {
  if (!m) return;
  release(m);
  delete m;
}

}  // extern "C"
