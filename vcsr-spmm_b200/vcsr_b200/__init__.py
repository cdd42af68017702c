"""Python front end of the B200 VCSR SpMM engine (ctypes over the C ABI in
include/vcsr_spmm.h, implemented by lib/libvcsr_b200.so).

The names mirror the reference's C++ interface so that tests read like the
reference's own call sites:

    read_matrix_market_coo   include/mmio.hpp:22      -> vcsr_read_mtx
    coo_to_csr               include/csr.hpp:16       -> vcsr_coo_to_csr
    csr_to_vcsr_spmm         include/vcsr.hpp:25      -> vcsr_build_vcsr (GPU)
    run_vcsr_spmm_gpu        src/kernels.cu:120       -> vcsr_plan_from_vcsr +
                                                       vcsr_spmm_accumulate
    run_csr_spmm_gpu         src/kernels.cu:107       -> vcsr_csr_spmm
    run_cusparse_spmm        src/kernels.cu:170       -> CuSparse
and Plan (vcsr_plan_*) is the engine's own build-once / run-many operator.

There is no CPU fallback: if the library is missing, importing this module
works but every call raises VcsrError.  Device buffers are torch CUDA tensors
(or raw device pointers); streams are torch.cuda.Stream objects or raw
cudaStream_t integers.
"""
from __future__ import annotations

import ctypes as C
import os
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "lib", "libvcsr_b200.so")

_i32p = C.POINTER(C.c_int)
_f32p = C.POINTER(C.c_float)

STATUS = {0: "ok", 1: "invalid", 2: "cuda", 3: "alloc", 4: "io",
          5: "unsupported", 6: "nccl", 7: "timeout", 8: "range"}
HOST, DEVICE = 0, 1
PLAN_REFERENCE_FORMAT = 1
PLAN_TF32_PANELS = 2
PLAN_HOST_BUILD = 4
PLAN_TC_SEGMENTS = 8
MTX_BANNER = 1


class VcsrError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status
        self.msg = msg


class _Coo(C.Structure):
    _fields_ = [("M", C.c_int), ("N", C.c_int), ("nnz", C.c_int),
                ("rows", _i32p), ("cols", _i32p), ("vals", _f32p)]


class _Csr(C.Structure):
    _fields_ = [("M", C.c_int), ("N", C.c_int), ("nnz", C.c_int),
                ("row_ptr", C.c_void_p), ("col", C.c_void_p), ("val", C.c_void_p)]


class _Vcsr(C.Structure):
    _fields_ = [("M", C.c_int), ("N", C.c_int), ("segw", C.c_int),
                ("bundle", C.c_int), ("num_groups", C.c_int),
                ("num_segments", C.c_int), ("num_slots", C.c_int64),
                ("group_ptr", C.c_void_p), ("group_depth", C.c_void_p),
                ("group_seg_base", C.c_void_p), ("group_rows", C.c_void_p),
                ("lcol", C.c_void_p), ("val", C.c_void_p),
                ("segment_group_start", C.c_void_p)]


class _PlanParams(C.Structure):
    _fields_ = [("segw", C.c_int), ("bundle", C.c_int), ("tileK", C.c_int),
                ("max_O", C.c_int), ("vec_rows", C.c_int), ("chunk", C.c_int),
                ("flags", C.c_int), ("panel_min_nnz", C.c_int), ("target_O", C.c_int),
                ("seg_min_run", C.c_int)]


class _PlanInfo(C.Structure):
    _fields_ = [("M", C.c_int), ("N", C.c_int), ("nnz", C.c_int),
                ("vec_rows", C.c_int), ("num_vectors", C.c_int),
                ("num_union", C.c_int64), ("num_units", C.c_int),
                ("num_split_vectors", C.c_int), ("num_split_units", C.c_int),
                ("num_long_units", C.c_int), ("panel_bytes", C.c_int64), ("has_reference_format", C.c_int),
                ("build_ms", C.c_double), ("num_panel_blocks", C.c_int),
                ("num_panel_row_blocks", C.c_int), ("panel_nnz", C.c_int64),
                ("num_seg_row_blocks", C.c_int), ("num_seg_pieces", C.c_int),
                ("seg_rows", C.c_int64), ("seg_only", C.c_int)]


_LIB = None

# every function of include/vcsr_spmm.h with its ctypes signature
_SIGS = {
    "vcsr_last_error": (C.c_char_p, []),
    "vcsr_status_string": (C.c_char_p, [C.c_int]),
    "vcsr_abi_version": (C.c_int, []),
    "vcsr_coo_free": (None, [C.POINTER(_Coo)]),
    "vcsr_csr_free": (None, [C.POINTER(_Csr), C.c_int]),
    "vcsr_vcsr_free": (None, [C.POINTER(_Vcsr), C.c_int]),
    "vcsr_read_mtx": (C.c_int, [C.c_char_p, C.POINTER(_Coo)]),
    "vcsr_read_mtx_ex": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(_Coo)]),
    "vcsr_coo_to_csr": (C.c_int, [C.POINTER(_Coo), C.POINTER(_Csr)]),
    "vcsr_gen_csr": (C.c_int, [C.c_char_p, C.c_uint64, C.c_int, C.POINTER(_Csr)]),
    "vcsr_gen_dense": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                 C.c_uint64, C.c_float, C.c_float, C.c_int,
                                 C.c_void_p]),
    "vcsr_csr_to_device": (C.c_int, [C.POINTER(_Csr), C.POINTER(_Csr), C.c_void_p]),
    "vcsr_build_vcsr": (C.c_int, [C.POINTER(_Csr), C.c_int, C.c_int,
                                  C.POINTER(_Vcsr), C.c_void_p]),
    "vcsr_vcsr_to_host": (C.c_int, [C.POINTER(_Vcsr), C.POINTER(_Vcsr)]),
    "vcsr_plan_params_default": (None, [C.POINTER(_PlanParams)]),
    "vcsr_plan_create": (C.c_int, [C.POINTER(_Csr), C.c_int, C.POINTER(_PlanParams),
                                   C.POINTER(C.c_void_p), C.c_void_p]),
    "vcsr_plan_get_info": (C.c_int, [C.c_void_p, C.POINTER(_PlanInfo)]),
    "vcsr_plan_export": (C.c_int, [C.c_void_p, C.POINTER(_Vcsr)]),
    "vcsr_plan_destroy": (None, [C.c_void_p]),
    "vcsr_spmm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                            C.c_int, C.c_void_p, C.POINTER(C.c_int)]),
    "vcsr_spmm_accumulate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p,
                                       C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int)]),
    "vcsr_plan_from_vcsr": (C.c_int, [C.POINTER(_Vcsr), C.c_int, C.POINTER(_PlanParams),
                                      C.POINTER(C.c_void_p), C.c_void_p]),
    "vcsr_spmm_host": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                 C.c_void_p]),
    "vcsr_plan_check": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vcsr_plan_host_rows": (C.c_int, [C.c_void_p, _i32p, _i32p, C.c_void_p]),
    "vcsr_plan_test_withhold_signal": (C.c_int, [C.c_void_p]),
    "vcsr_plan_row_panels": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.c_void_p,
                                       C.c_void_p, C.c_void_p]),
    "vcsr_spmm_row_panel": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p,
                                      C.c_int, C.c_int, C.c_void_p, C.POINTER(C.c_int)]),
    "vcsr_spmm_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                 C.c_int, C.c_void_p, C.POINTER(C.c_int)]),
    "vcsr_spmm_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int,
                                C.c_int, C.c_void_p, C.POINTER(C.c_int)]),
    "vcsr_plan_save": (C.c_int, [C.c_void_p, C.c_char_p]),
    "vcsr_plan_load": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p), C.c_void_p]),
    "vcsr_spmm_segmented": (C.c_int, [C.POINTER(_Vcsr), C.c_void_p, C.c_int, C.c_int,
                                      C.c_void_p, C.c_void_p]),
    "vcsr_csr_spmm": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "vcsr_csr_spmm_noalloc": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "vcsr_cusparse_create": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_void_p, C.c_int, C.c_void_p,
                                       C.POINTER(C.c_void_p)]),
    "vcsr_cusparse_run": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vcsr_cusparse_destroy": (None, [C.c_void_p]),
    "vcsr_partition_rows": (C.c_int, [_i32p, C.c_int, C.c_int, C.c_int, _i32p]),
    "vcsr_partition_rows_weighted": (C.c_int, [_i32p, C.c_int, C.c_int, C.c_int, C.c_double,
                                               _i32p]),
    "vcsr_csr_row_panel": (C.c_int, [C.POINTER(_Csr), C.c_int, C.c_int,
                                     C.POINTER(_Csr)]),
    "vcsr_mgpu_create": (C.c_int, [C.POINTER(_Csr), C.c_int, _i32p,
                                   C.POINTER(_PlanParams), C.POINTER(C.c_void_p)]),
    "vcsr_mgpu_set_b": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int,
                                  C.POINTER(C.c_float)]),
    "vcsr_mgpu_spmm": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_float)]),
    "vcsr_mgpu_gather_c": (C.c_int, [C.c_void_p, C.c_void_p]),
    "vcsr_mgpu_cuts": (C.c_int, [C.c_void_p, _i32p]),
    "vcsr_mgpu_destroy": (None, [C.c_void_p]),
}


def lib():
    """Load the engine library (raises VcsrError if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise VcsrError(5, f"{LIB_PATH} is missing: build it with "
                               "`make -C vcsr-spmm_b200` (no CPU fallback)")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _LIB = L
    return _LIB


def exported_names():
    return list(_SIGS)


def _check(st):
    if st != 0:
        raise VcsrError(st, lib().vcsr_last_error().decode())


def _stream(s):
    if s is None:
        try:
            import torch
            if torch.cuda.is_available():
                return C.c_void_p(torch.cuda.current_stream().cuda_stream)
        except ImportError:
            pass
        return C.c_void_p(0)
    if isinstance(s, int):
        return C.c_void_p(s)
    return C.c_void_p(s.cuda_stream)


def _ptr(x):
    if x is None:
        return C.c_void_p(0)
    if isinstance(x, int):
        return C.c_void_p(x)
    if isinstance(x, np.ndarray):
        return x.ctypes.data_as(C.c_void_p)
    return C.c_void_p(x.data_ptr())


def _take(ptr, n, dtype):
    if n == 0 or not ptr:
        return np.zeros(0, dtype)
    ct = {np.int32: C.c_int, np.float32: C.c_float}[dtype]
    arr = C.cast(ptr, C.POINTER(ct))
    return np.ctypeslib.as_array(arr, shape=(n,)).astype(dtype, copy=True)


# ----------------------------------------------------------------- host data

@dataclass
class COO:
    """struct COO (include/mmio.hpp:15-19)."""
    M: int
    N: int
    rows: np.ndarray
    cols: np.ndarray
    vals: np.ndarray


@dataclass
class CSR:
    """struct CSR (include/csr.hpp:8-13), host arrays."""
    M: int
    N: int
    nnz: int
    row_ptr: np.ndarray
    col: np.ndarray
    val: np.ndarray

    def _struct(self):
        self.row_ptr = np.ascontiguousarray(self.row_ptr, np.int32)
        self.col = np.ascontiguousarray(self.col, np.int32)
        self.val = np.ascontiguousarray(self.val, np.float32)
        return _Csr(self.M, self.N, self.nnz, self.row_ptr.ctypes.data,
                    self.col.ctypes.data, self.val.ctypes.data)


@dataclass
class VCSRSpMM:
    """struct VCSRSpMM (include/vcsr.hpp:12-23), host arrays."""
    M: int
    N: int
    segw: int
    bundle: int
    group_ptr: np.ndarray
    group_depth: np.ndarray
    group_seg_base: np.ndarray
    group_rows: np.ndarray
    lcol: np.ndarray
    val: np.ndarray
    segment_group_start: np.ndarray

    @property
    def num_groups(self):
        return len(self.group_depth)

    @property
    def num_slots(self):
        return len(self.lcol)

    def as_dict(self):
        return dict(M=self.M, N=self.N, segw=self.segw, bundle=self.bundle,
                    num_groups=self.num_groups, num_slots=self.num_slots,
                    group_ptr=self.group_ptr, group_depth=self.group_depth,
                    group_seg_base=self.group_seg_base, group_rows=self.group_rows,
                    lcol=self.lcol, val=self.val,
                    segment_group_start=self.segment_group_start)


def _csr_from_struct(s):
    L = lib()
    out = CSR(s.M, s.N, s.nnz, _take(s.row_ptr, s.M + 1, np.int32),
              _take(s.col, s.nnz, np.int32), _take(s.val, s.nnz, np.float32))
    L.vcsr_csr_free(C.byref(s), HOST)
    return out


def _vcsr_from_host_struct(v):
    G, P, S, b = v.num_groups, v.num_slots, v.num_segments, v.bundle
    out = VCSRSpMM(v.M, v.N, v.segw, b, _take(v.group_ptr, G + 1, np.int32),
                   _take(v.group_depth, G, np.int32),
                   _take(v.group_seg_base, G, np.int32),
                   _take(v.group_rows, G * b, np.int32),
                   _take(v.lcol, P, np.int32), _take(v.val, P, np.float32),
                   _take(v.segment_group_start, S + 1, np.int32))
    lib().vcsr_vcsr_free(C.byref(v), HOST)
    return out


def read_matrix_market_coo(path, banner=False) -> COO:
    """read_matrix_market_coo (include/mmio.hpp:22-45); with banner=True the
    Matrix Market banner is followed (pattern / complex fields, symmetric,
    skew-symmetric and hermitian expansion: vcsr_read_mtx_ex)."""
    L = lib()
    s = _Coo()
    if banner:
        _check(L.vcsr_read_mtx_ex(os.fsencode(path), MTX_BANNER, C.byref(s)))
    else:
        _check(L.vcsr_read_mtx(os.fsencode(path), C.byref(s)))
    out = COO(s.M, s.N, _take(s.rows, s.nnz, np.int32),
              _take(s.cols, s.nnz, np.int32), _take(s.vals, s.nnz, np.float32))
    L.vcsr_coo_free(C.byref(s))
    return out


def coo_to_csr(coo: COO) -> CSR:
    """coo_to_csr (include/csr.hpp:16-37)."""
    L = lib()
    r = np.ascontiguousarray(coo.rows, np.int32)
    c = np.ascontiguousarray(coo.cols, np.int32)
    v = np.ascontiguousarray(coo.vals, np.float32)
    s = _Coo(coo.M, coo.N, len(v), r.ctypes.data_as(_i32p), c.ctypes.data_as(_i32p),
             v.ctypes.data_as(_f32p))
    out = _Csr()
    _check(L.vcsr_coo_to_csr(C.byref(s), C.byref(out)))
    return _csr_from_struct(out)


def gen_csr(config: str, seed: int = 0, size: int = 0) -> CSR:
    """Deterministic synthetic matrix (vcsr_gen_csr)."""
    out = _Csr()
    _check(lib().vcsr_gen_csr(config.encode(), seed, size, C.byref(out)))
    return _csr_from_struct(out)


def gen_dense_host(rows, cols, seed, lo=-1.0, hi=1.0) -> np.ndarray:
    a = np.empty((rows, cols), np.float32)
    _check(lib().vcsr_gen_dense(a.ctypes.data, rows, cols, cols, seed, lo, hi,
                                HOST, None))
    return a


def gen_dense_device(t, seed, lo=-1.0, hi=1.0, stream=None):
    """Fill a 2-D torch CUDA float32 tensor in place (same bits as the host)."""
    rows, cols = t.shape
    _check(lib().vcsr_gen_dense(_ptr(t), rows, cols, t.stride(0), seed, lo, hi,
                                DEVICE, _stream(stream)))
    return t


def partition_rows(row_ptr, parts, align=1, row_weight=0.0) -> np.ndarray:
    """Row cuts of balanced panels: each row weighs its nnz + row_weight."""
    rp = np.ascontiguousarray(row_ptr, np.int32)
    cuts = np.zeros(parts + 1, np.int32)
    _check(lib().vcsr_partition_rows_weighted(rp.ctypes.data_as(_i32p), len(rp) - 1, parts,
                                              align, float(row_weight),
                                              cuts.ctypes.data_as(_i32p)))
    return cuts


def csr_row_panel(csr: CSR, r0, r1) -> CSR:
    s = csr._struct()
    out = _Csr()
    _check(lib().vcsr_csr_row_panel(C.byref(s), r0, r1, C.byref(out)))
    return _csr_from_struct(out)


# --------------------------------------------------------------- device data

class DeviceCSR:
    """A CSR whose arrays are torch CUDA tensors."""

    def __init__(self, csr: CSR, device=None):
        import torch
        dev = device or torch.device("cuda", torch.cuda.current_device())
        self.M, self.N, self.nnz = csr.M, csr.N, csr.nnz
        self.row_ptr = torch.from_numpy(np.ascontiguousarray(csr.row_ptr, np.int32)).to(dev)
        self.col = torch.from_numpy(np.ascontiguousarray(csr.col, np.int32)).to(dev)
        self.val = torch.from_numpy(np.ascontiguousarray(csr.val, np.float32)).to(dev)

    def _struct(self):
        return _Csr(self.M, self.N, self.nnz, self.row_ptr.data_ptr(),
                    self.col.data_ptr(), self.val.data_ptr())


class DeviceVCSR:
    """A segment-major VCSR with device arrays owned by the library."""

    def __init__(self, s: _Vcsr):
        self._s = s

    @property
    def num_groups(self):
        return self._s.num_groups

    @property
    def num_slots(self):
        return self._s.num_slots

    def to_host(self) -> VCSRSpMM:
        h = _Vcsr()
        _check(lib().vcsr_vcsr_to_host(C.byref(self._s), C.byref(h)))
        return _vcsr_from_host_struct(h)

    def close(self):
        if getattr(self, "_s", None) is not None and _LIB is not None:
            _LIB.vcsr_vcsr_free(C.byref(self._s), DEVICE)
        self._s = None

    __del__ = close


def csr_to_vcsr_spmm(dcsr: DeviceCSR, segw=4, bundle=32, stream=None) -> DeviceVCSR:
    """csr_to_vcsr_spmm (include/vcsr.hpp:25-109), built on the GPU."""
    s = dcsr._struct()
    out = _Vcsr()
    _check(lib().vcsr_build_vcsr(C.byref(s), segw, bundle, C.byref(out),
                                 _stream(stream)))
    return DeviceVCSR(out)


def run_vcsr_spmm_gpu(V: DeviceVCSR, dB, O, tileK, dC, stream=None):
    """run_vcsr_spmm_gpu (src/kernels.cu:120): C += A*B for the matrix V
    holds, on the engine: a plan built on the GPU from V's slots
    (vcsr_plan_from_vcsr), then vcsr_spmm_accumulate."""
    plan = Plan.from_vcsr(V, tileK=tileK, max_O=max(O, 512), stream=stream)
    plan.spmm(dB, dC, O=O, ldb=O, ldc=O, stream=stream, accumulate=True)
    plan.check(stream)


def run_vcsr_spmm_segmented_gpu(V: DeviceVCSR, dB, O, tileK, dC, stream=None):
    """The segment-major kernel on V itself (vcsr_spmm_segmented): C += A*B,
    race-free form of src/kernels.cu:37-103."""
    _check(lib().vcsr_spmm_segmented(C.byref(V._s), _ptr(dB), O, tileK, _ptr(dC),
                                     _stream(stream)))


def run_csr_spmm_gpu(M, d_rowptr, d_col, d_val, dB, O, dC, stream=None):
    """run_csr_spmm_gpu (src/kernels.cu:107): C = A*B."""
    _check(lib().vcsr_csr_spmm(M, _ptr(d_rowptr), _ptr(d_col), _ptr(d_val),
                               _ptr(dB), O, _ptr(dC), _stream(stream)))


def csr_spmm_noalloc(M, d_rowptr, d_col, d_val, dB, O, dC, stream=None):
    """C = A*B like run_csr_spmm_gpu, without allocating device memory: the
    scratch for split long rows is a fixed array inside the library
    (vcsr_csr_spmm_noalloc).  Synchronises the stream."""
    _check(lib().vcsr_csr_spmm_noalloc(M, _ptr(d_rowptr), _ptr(d_col), _ptr(d_val),
                                       _ptr(dB), O, _ptr(dC), _stream(stream)))


class CuSparse:
    """cuSPARSE SpMM with handle/buffer made once (src/kernels.cu:170-235)."""
    ALGS = {0: "ALG_DEFAULT", 1: "CSR_ALG1", 2: "CSR_ALG2", 3: "CSR_ALG3"}

    def __init__(self, dcsr: DeviceCSR, dB, O, dC, alg=0, stream=None):
        h = C.c_void_p()
        _check(lib().vcsr_cusparse_create(dcsr.M, dcsr.N, dcsr.nnz,
                                          _ptr(dcsr.row_ptr), _ptr(dcsr.col),
                                          _ptr(dcsr.val), _ptr(dB), O, _ptr(dC),
                                          alg, _stream(stream), C.byref(h)))
        self._h = h
        self.alg = alg

    def run(self, stream=None):
        _check(lib().vcsr_cusparse_run(self._h, _stream(stream)))

    def close(self):
        if getattr(self, "_h", None) and _LIB is not None:
            _LIB.vcsr_cusparse_destroy(self._h)
        self._h = None

    __del__ = close


class Plan:
    """Build-once SpMM operator (vcsr_plan_*).  csr is a host CSR or a DeviceCSR."""

    def __init__(self, csr, segw=4, bundle=32, tileK=0, max_O=512, vec_rows=0,
                 chunk=0, reference_format=False, tf32_panels=False, panel_min_nnz=0,
                 target_O=0, host_build=False, tc_segments=False, seg_min_run=0,
                 stream=None):
        L = lib()
        p = _PlanParams()
        L.vcsr_plan_params_default(C.byref(p))
        p.segw, p.bundle, p.tileK, p.max_O = segw, bundle, tileK, max_O
        p.vec_rows, p.chunk = vec_rows, chunk
        p.flags = ((PLAN_REFERENCE_FORMAT if reference_format else 0)
                   | (PLAN_TF32_PANELS if tf32_panels else 0)
                   | (PLAN_HOST_BUILD if host_build else 0)
                   | (PLAN_TC_SEGMENTS if tc_segments else 0))
        p.panel_min_nnz = panel_min_nnz
        p.target_O = target_O
        p.seg_min_run = seg_min_run
        where = DEVICE if isinstance(csr, DeviceCSR) else HOST
        s = csr._struct()
        h = C.c_void_p()
        _check(L.vcsr_plan_create(C.byref(s), where, C.byref(p), C.byref(h),
                                  _stream(stream)))
        self._h = h
        self.M, self.N, self.nnz = csr.M, csr.N, csr.nnz
        self.last_launches = 0

    @classmethod
    def from_vcsr(cls, V, tileK=0, max_O=512, stream=None):
        """The engine's plan for the matrix a segment-major VCSR holds
        (vcsr_plan_from_vcsr): a DeviceVCSR, or a host VCSRSpMM."""
        L = lib()
        p = _PlanParams()
        L.vcsr_plan_params_default(C.byref(p))
        p.tileK, p.max_O = tileK, max_O
        keep = None
        if isinstance(V, DeviceVCSR):
            s, where = V._s, DEVICE
        else:
            keep = [np.ascontiguousarray(a, dtype) for a, dtype in (
                (V.group_ptr, np.int32), (V.group_depth, np.int32),
                (V.group_seg_base, np.int32), (V.group_rows, np.int32),
                (V.lcol, np.int32), (V.val, np.float32))]
            s = _Vcsr()
            s.M, s.N, s.segw, s.bundle = V.M, V.N, V.segw, V.bundle
            s.num_groups = len(keep[1])
            s.num_segments = -(-V.N // V.segw) if V.segw > 0 else 0
            s.num_slots = len(keep[4])
            (s.group_ptr, s.group_depth, s.group_seg_base, s.group_rows, s.lcol,
             s.val) = (a.ctypes.data for a in keep)
            where = HOST
        p.segw, p.bundle = s.segw, s.bundle
        h = C.c_void_p()
        _check(L.vcsr_plan_from_vcsr(C.byref(s), where, C.byref(p), C.byref(h),
                                     _stream(stream)))
        self = cls.__new__(cls)
        self._h = h
        i = self.info()
        self.M, self.N, self.nnz = i["M"], i["N"], i["nnz"]
        self.last_launches = 0
        return self

    def info(self):
        i = _PlanInfo()
        _check(lib().vcsr_plan_get_info(self._h, C.byref(i)))
        return {k: getattr(i, k) for k, _ in _PlanInfo._fields_}

    def export(self) -> VCSRSpMM:
        v = _Vcsr()
        _check(lib().vcsr_plan_export(self._h, C.byref(v)))
        return _vcsr_from_host_struct(v)

    def spmm(self, B, Cout, O=None, ldb=None, ldc=None, stream=None, accumulate=False):
        """C = A*B on device tensors (or raw pointers with O/ldb/ldc given);
        with accumulate=True, C += A*B (vcsr_spmm_accumulate, FP32 B).
        A bfloat16 or float16 B runs vcsr_spmm_bf16 / vcsr_spmm_f16 (FP32 C)."""
        if O is None:
            O = B.shape[1]
        if ldb is None:
            ldb = B.stride(0) if hasattr(B, "stride") else O
        if ldc is None:
            ldc = Cout.stride(0) if hasattr(Cout, "stride") else O
        n = C.c_int(0)
        dt = str(getattr(B, "dtype", ""))
        if accumulate:
            if dt in ("torch.bfloat16", "torch.float16"):
                raise VcsrError(5, "accumulate takes an FP32 B")
            _check(lib().vcsr_spmm_accumulate(self._h, _ptr(B), ldb, _ptr(Cout), ldc, O,
                                              _stream(stream), C.byref(n)))
        elif dt == "torch.bfloat16":  # 16-bit inputs, FP32 sums
            _check(lib().vcsr_spmm_bf16(self._h, _ptr(B), ldb, _ptr(Cout), ldc, O,
                                        _stream(stream), C.byref(n)))
        elif dt == "torch.float16":
            _check(lib().vcsr_spmm_f16(self._h, _ptr(B), ldb, _ptr(Cout), ldc, O,
                                       _stream(stream), C.byref(n)))
        else:
            _check(lib().vcsr_spmm(self._h, _ptr(B), ldb, _ptr(Cout), ldc, O,
                                   _stream(stream), C.byref(n)))
        self.last_launches = n.value
        return Cout

    def save(self, path):
        """Write the plan to `path` (vcsr_plan_save)."""
        _check(lib().vcsr_plan_save(self._h, os.fsencode(path)))

    @classmethod
    def load(cls, path, stream=None):
        """A plan read from a file written by save() (vcsr_plan_load)."""
        h = C.c_void_p()
        _check(lib().vcsr_plan_load(os.fsencode(path), C.byref(h), _stream(stream)))
        self = cls.__new__(cls)
        self._h = h
        i = self.info()
        self.M, self.N, self.nnz = i["M"], i["N"], i["nnz"]
        self.last_launches = 0
        return self

    def row_panels(self):
        """[(row0, row1, col_max)] of the plan's row panels (empty for small
        plans and plans with TF32 panels)."""
        n = C.c_int(0)
        _check(lib().vcsr_plan_row_panels(self._h, C.byref(n), None, None, None))
        if n.value == 0:
            return []
        r0, r1, cm = (np.zeros(n.value, np.int32) for _ in range(3))
        _check(lib().vcsr_plan_row_panels(self._h, C.byref(n), r0.ctypes.data, r1.ctypes.data,
                                          cm.ctypes.data))
        return [(int(a), int(b), int(c)) for a, b, c in zip(r0, r1, cm)]

    def spmm_row_panel(self, panel, B, Cout, O=None, ldb=None, ldc=None, stream=None):
        """Rows of one row panel of C = A*B (vcsr_spmm_row_panel)."""
        if O is None:
            O = B.shape[1]
        if ldb is None:
            ldb = B.stride(0) if hasattr(B, "stride") else O
        if ldc is None:
            ldc = Cout.stride(0) if hasattr(Cout, "stride") else O
        n = C.c_int(0)
        _check(lib().vcsr_spmm_row_panel(self._h, panel, _ptr(B), ldb, _ptr(Cout), ldc, O,
                                         _stream(stream), C.byref(n)))
        self.last_launches = n.value
        return Cout

    def check(self, stream=None):
        """Synchronise and raise VcsrError (status 7) if a bounded wait of the
        plan's kernels ran out since the last check."""
        _check(lib().vcsr_plan_check(self._h, _stream(stream)))

    def test_withhold_signal(self):
        """Test hook: the next TF32 panel launch withholds one barrier signal,
        so a bounded wait runs out and check() raises (status 7)."""
        _check(lib().vcsr_plan_test_withhold_signal(self._h))

    def spmm_host(self, hB, hC, stream=None):
        """C = A*B with host buffers (H2D, SpMM, D2H, synchronise)."""
        O = hB.shape[1] if hB is not None else hC.shape[1]
        _check(lib().vcsr_spmm_host(self._h, _ptr(hB), _ptr(hC), O, _stream(stream)))
        return hC

    def host_rows(self, stream=None):
        """(B rows up, C rows down) per spmm_host call with page-locked
        buffers, O a multiple of 16 and more than 8 MB of B and C."""
        b, c = np.zeros(1, np.int32), np.zeros(1, np.int32)
        _check(lib().vcsr_plan_host_rows(self._h, b.ctypes.data_as(_i32p),
                                         c.ctypes.data_as(_i32p), _stream(stream)))
        return int(b[0]), int(c[0])

    def close(self):
        if getattr(self, "_h", None) and _LIB is not None:
            _LIB.vcsr_plan_destroy(self._h)
        self._h = None

    __del__ = close


class MultiGPU:
    """Row panels of A on several GPUs of this process (vcsr_mgpu_*): one plan
    per GPU, B replicated by one NCCL broadcast, disjoint C panels."""

    def __init__(self, csr: CSR, ngpus, devices=None, segw=4, bundle=32, max_O=512,
                 vec_rows=0):
        L = lib()
        p = _PlanParams()
        L.vcsr_plan_params_default(C.byref(p))
        p.segw, p.bundle, p.max_O, p.vec_rows = segw, bundle, max_O, vec_rows
        s = csr._struct()
        devs = None
        if devices is not None:
            self._devs = np.ascontiguousarray(devices, np.int32)
            devs = self._devs.ctypes.data_as(_i32p)
        h = C.c_void_p()
        _check(L.vcsr_mgpu_create(C.byref(s), ngpus, devs, C.byref(p), C.byref(h)))
        self._h = h
        self.n = ngpus
        self.M, self.N = csr.M, csr.N

    def cuts(self):
        c = np.zeros(self.n + 1, np.int32)
        _check(lib().vcsr_mgpu_cuts(self._h, c.ctypes.data_as(_i32p)))
        return c

    def set_b(self, hB):
        hB = np.ascontiguousarray(hB, np.float32)
        ms = C.c_float()
        _check(lib().vcsr_mgpu_set_b(self._h, hB.ctypes.data, hB.shape[1], C.byref(ms)))
        self.O = hB.shape[1]
        return ms.value

    def spmm(self):
        ms = C.c_float()
        _check(lib().vcsr_mgpu_spmm(self._h, self.O, C.byref(ms)))
        return ms.value

    def gather_c(self):
        out = np.empty((self.M, self.O), np.float32)
        _check(lib().vcsr_mgpu_gather_c(self._h, out.ctypes.data))
        return out

    def close(self):
        if getattr(self, "_h", None) and _LIB is not None:
            _LIB.vcsr_mgpu_destroy(self._h)
        self._h = None

    __del__ = close
