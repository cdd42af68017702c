"""ctypes front end of the CPU oracle (oracle.c) and of the reference's own code
built into oracle/_ref/.

TEST INFRASTRUCTURE ONLY.  The product package never imports this module; only
tests/, __graft_entry__.smoke() and bench.py's CPU baseline legs do, and only
as the checker or the timed CPU algorithm.

Reference code each function stands for is cited in oracle.c
(include/mmio.hpp:22-45, include/csr.hpp:16-37, include/vcsr.hpp:25-109,
src/kernels.cu:15-33 and :82-101).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None
_REFK = None

_i32p = C.POINTER(C.c_int)
_f32p = C.POINTER(C.c_float)
_f64p = C.POINTER(C.c_double)


class OracleError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


class _VCSR(C.Structure):
    _fields_ = [("M", C.c_int), ("N", C.c_int), ("segw", C.c_int),
                ("bundle", C.c_int), ("num_groups", C.c_int),
                ("num_segments", C.c_int), ("num_slots", C.c_int64),
                ("group_ptr", _i32p), ("group_depth", _i32p),
                ("group_seg_base", _i32p), ("group_rows", _i32p),
                ("lcol", _i32p), ("val", _f32p),
                ("segment_group_start", _i32p)]


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise OracleError(-1, f"{path} missing: run `make -C oracle`")
        L = C.CDLL(path)
        L.oracle_last_error.restype = C.c_char_p
        L.oracle_read_mtx.argtypes = [C.c_char_p, _i32p, _i32p, _i32p,
                                      C.POINTER(_i32p), C.POINTER(_i32p),
                                      C.POINTER(_f32p)]
        L.oracle_coo_to_csr.argtypes = [C.c_int, C.c_int, C.c_int, _i32p, _i32p,
                                        _f32p, C.POINTER(_i32p),
                                        C.POINTER(_i32p), C.POINTER(_f32p)]
        L.oracle_csr_spmm_f32.argtypes = [C.c_int, _i32p, _i32p, _f32p, _f32p,
                                          C.c_int64, C.c_int, _f32p, C.c_int64,
                                          C.c_int]
        L.oracle_csr_spmm_f64.argtypes = [C.c_int, _i32p, _i32p, _f32p, _f32p,
                                          C.c_int64, C.c_int, _f64p, C.c_int64,
                                          C.c_int]
        L.oracle_csr_to_vcsr.argtypes = [C.c_int, C.c_int, _i32p, _i32p, _f32p,
                                         C.c_int, C.c_int, C.POINTER(_VCSR)]
        L.oracle_vcsr_spmm.argtypes = [C.POINTER(_VCSR), _f32p, C.c_int, _f32p]
        L.oracle_vcsr_free.argtypes = [C.POINTER(_VCSR)]
        L.oracle_free.argtypes = [C.c_void_p]
        L.oracle_gen_dense.argtypes = [_f32p, C.c_int64, C.c_int64, C.c_uint64, C.c_float,
                                       C.c_float]
        L.oracle_gen_rmat.argtypes = [C.c_int, C.c_uint64, _i32p, C.POINTER(_i32p),
                                      C.POINTER(_i32p), C.POINTER(_f32p), _i32p]
        L.oracle_max_threads.restype = C.c_int
        _LIB = L
    return _LIB


def max_threads() -> int:
    return lib().oracle_max_threads()


def _p(a, t):
    return a.ctypes.data_as(t)


def _take(ptr, n, dtype, free):
    if n == 0:
        out = np.zeros(0, dtype)
    else:
        out = np.ctypeslib.as_array(ptr, shape=(n,)).astype(dtype, copy=True)
    free(C.cast(ptr, C.c_void_p))
    return out


def gen_dense(rows, cols, seed, lo=-1.0, hi=1.0):
    """The engine's seeded dense fill (vcsr_gen_dense), restated on the CPU."""
    out = np.empty((rows, cols), np.float32)
    lib().oracle_gen_dense(_p(out, _f32p), rows, cols, seed, lo, hi)
    return out


def gen_rmat(scale, seed=0):
    """The engine's R-MAT matrix (gen_rmat), restated on the CPU ->
    (M, row_ptr, col, val)."""
    L = lib()
    M, Z = C.c_int(), C.c_int()
    r, c, v = _i32p(), _i32p(), _f32p()
    rc = L.oracle_gen_rmat(scale, seed, C.byref(M), C.byref(r), C.byref(c), C.byref(v),
                           C.byref(Z))
    if rc:
        raise OracleError(rc, L.oracle_last_error().decode())
    return (M.value, _take(r, M.value + 1, np.int32, L.oracle_free),
            _take(c, Z.value, np.int32, L.oracle_free), _take(v, Z.value, np.float32, L.oracle_free))


def read_mtx(path):
    """read_matrix_market_coo (include/mmio.hpp:22-45) -> (M, N, rows, cols, vals)."""
    L = lib()
    M, N, Z = C.c_int(), C.c_int(), C.c_int()
    r, c, v = _i32p(), _i32p(), _f32p()
    rc = L.oracle_read_mtx(path.encode(), C.byref(M), C.byref(N), C.byref(Z),
                           C.byref(r), C.byref(c), C.byref(v))
    if rc:
        raise OracleError(rc, L.oracle_last_error().decode())
    n = Z.value
    return (M.value, N.value, _take(r, n, np.int32, L.oracle_free),
            _take(c, n, np.int32, L.oracle_free),
            _take(v, n, np.float32, L.oracle_free))


def coo_to_csr(M, N, rows, cols, vals):
    """coo_to_csr (include/csr.hpp:16-37) -> (row_ptr, col, val)."""
    L = lib()
    rows = np.ascontiguousarray(rows, np.int32)
    cols = np.ascontiguousarray(cols, np.int32)
    vals = np.ascontiguousarray(vals, np.float32)
    rp, cc, vv = _i32p(), _i32p(), _f32p()
    rc = L.oracle_coo_to_csr(M, N, len(vals), _p(rows, _i32p), _p(cols, _i32p),
                             _p(vals, _f32p), C.byref(rp), C.byref(cc),
                             C.byref(vv))
    if rc:
        raise OracleError(rc, L.oracle_last_error().decode())
    nnz = len(vals)
    return (_take(rp, M + 1, np.int32, L.oracle_free),
            _take(cc, nnz, np.int32, L.oracle_free),
            _take(vv, nnz, np.float32, L.oracle_free))


def csr_spmm_f32(M, row_ptr, col, val, B, nthreads=0):
    """csr_spmm_kernel semantics (src/kernels.cu:15-33): FP32, CSR order, FMA."""
    B = np.ascontiguousarray(B, np.float32)
    O = B.shape[1]
    Cm = np.empty((M, O), np.float32)
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col = np.ascontiguousarray(col, np.int32)
    val = np.ascontiguousarray(val, np.float32)
    lib().oracle_csr_spmm_f32(M, _p(row_ptr, _i32p), _p(col, _i32p),
                              _p(val, _f32p), _p(B, _f32p), O, O, _p(Cm, _f32p),
                              O, nthreads)
    return Cm


def csr_spmm_f32_into(M, row_ptr, col, val, B, Cm, nthreads=0):
    """Same as csr_spmm_f32, writing a preallocated C (used for timing)."""
    O = B.shape[1]
    lib().oracle_csr_spmm_f32(M, _p(row_ptr, _i32p), _p(col, _i32p),
                              _p(val, _f32p), _p(B, _f32p), B.strides[0] // 4,
                              O, _p(Cm, _f32p), Cm.strides[0] // 4, nthreads)


def csr_spmm_f64(M, row_ptr, col, val, B, nthreads=0):
    B = np.ascontiguousarray(B, np.float32)
    O = B.shape[1]
    Cm = np.empty((M, O), np.float64)
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col = np.ascontiguousarray(col, np.int32)
    val = np.ascontiguousarray(val, np.float32)
    lib().oracle_csr_spmm_f64(M, _p(row_ptr, _i32p), _p(col, _i32p),
                              _p(val, _f32p), _p(B, _f32p), O, O, _p(Cm, _f64p),
                              O, nthreads)
    return Cm


_VCSR_KEYS = ("group_ptr", "group_depth", "group_seg_base", "group_rows",
              "lcol", "val", "segment_group_start")


def csr_to_vcsr(M, N, row_ptr, col, val, segw, bundle):
    """csr_to_vcsr_spmm (include/vcsr.hpp:25-109), ties (count desc, row asc)."""
    L = lib()
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col = np.ascontiguousarray(col, np.int32)
    val = np.ascontiguousarray(val, np.float32)
    v = _VCSR()
    rc = L.oracle_csr_to_vcsr(M, N, _p(row_ptr, _i32p), _p(col, _i32p),
                              _p(val, _f32p), segw, bundle, C.byref(v))
    if rc:
        raise OracleError(rc, L.oracle_last_error().decode())
    G, P, S = v.num_groups, v.num_slots, v.num_segments

    def arr(ptr, n, dt):
        if n == 0:
            return np.zeros(0, dt)
        return np.ctypeslib.as_array(ptr, shape=(n,)).astype(dt, copy=True)

    out = dict(M=M, N=N, segw=segw, bundle=bundle, num_groups=G, num_slots=P,
               num_segments=S,
               group_ptr=arr(v.group_ptr, G + 1, np.int32),
               group_depth=arr(v.group_depth, G, np.int32),
               group_seg_base=arr(v.group_seg_base, G, np.int32),
               group_rows=arr(v.group_rows, G * bundle, np.int32),
               lcol=arr(v.lcol, P, np.int32), val=arr(v.val, P, np.float32),
               segment_group_start=arr(v.segment_group_start, S + 1, np.int32))
    L.oracle_vcsr_free(C.byref(v))
    return out


def vcsr_spmm(v, B):
    """Sequential vcsr_spmm_kernel update (src/kernels.cu:82-101), C from 0."""
    L = lib()
    B = np.ascontiguousarray(B, np.float32)
    O = B.shape[1]
    keep = {k: np.ascontiguousarray(v[k]) for k in _VCSR_KEYS}
    s = _VCSR(v["M"], v["N"], v["segw"], v["bundle"], v["num_groups"],
              v.get("num_segments", 0), v["num_slots"],
              _p(keep["group_ptr"], _i32p), _p(keep["group_depth"], _i32p),
              _p(keep["group_seg_base"], _i32p), _p(keep["group_rows"], _i32p),
              _p(keep["lcol"], _i32p), _p(keep["val"], _f32p),
              _p(keep["segment_group_start"], _i32p))
    Cm = np.zeros((v["M"], O), np.float32)
    L.oracle_vcsr_spmm(C.byref(s), _p(B, _f32p), O, _p(Cm, _f32p))
    return Cm


def canonical_vcsr(v):
    """Re-pack a segment-major VCSR so that any tie order the reference's
    std::sort may pick maps to the same arrays.

    Within each segment the lanes are re-ordered by (count desc, row asc);
    lanes of rows with no entry in the segment (count 0) keep their position at
    the end but their row id becomes -2 (the reference may pick any such rows);
    lanes past the last row stay -1.  Group metadata is unchanged (it depends
    only on the sorted count sequence).  Returns a dict with the same keys.
    """
    G, bundle = int(v["num_groups"]), int(v["bundle"])
    gp = np.asarray(v["group_ptr"], np.int64)
    depth = np.asarray(v["group_depth"], np.int64)
    sb = np.asarray(v["group_seg_base"], np.int64)
    rows = np.asarray(v["group_rows"], np.int64).reshape(G, bundle) if G else \
        np.zeros((0, bundle), np.int64)
    lcol = np.asarray(v["lcol"], np.int64)
    val = np.asarray(v["val"], np.float32)
    out_rows = rows.copy()
    out_lcol = lcol.copy()
    out_val = val.copy()
    g = 0
    while g < G:
        h = g
        while h < G and sb[h] == sb[g]:
            h += 1
        lanes = []  # (key, row, entries)
        for gg in range(g, h):
            d = int(depth[gg])
            blk_l = lcol[gp[gg]:gp[gg] + d * bundle].reshape(d, bundle)
            blk_v = val[gp[gg]:gp[gg] + d * bundle].reshape(d, bundle)
            for ln in range(bundle):
                r = int(rows[gg, ln])
                ent = [(int(blk_l[k, ln]), blk_v[k, ln]) for k in range(d)
                       if blk_l[k, ln] != -1]
                cnt = len(ent)
                if r < 0:
                    key = (2, 0, 0)
                elif cnt == 0:
                    key = (1, 0, 0)
                    r = -2
                else:
                    key = (0, -cnt, r)
                lanes.append((key, r, ent))
        lanes.sort(key=lambda t: t[0])
        i = 0
        for gg in range(g, h):
            d = int(depth[gg])
            for ln in range(bundle):
                key, r, ent = lanes[i]
                i += 1
                out_rows[gg, ln] = r
                for k in range(d):
                    s = gp[gg] + k * bundle + ln
                    if k < len(ent):
                        out_lcol[s], out_val[s] = ent[k]
                    else:
                        out_lcol[s], out_val[s] = -1, np.float32(0)
        g = h
    out = dict(v)
    out["group_rows"] = out_rows.reshape(-1).astype(np.int32)
    out["lcol"] = out_lcol.astype(np.int32)
    out["val"] = out_val
    return out


# ------------------------------------------------- reference's own code (_ref)

def ref_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libvcsr_ref.so"))


def ref_lib():
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libvcsr_ref.so")
        if not os.path.exists(path):
            raise OracleError(-1, f"{path} missing: build with `make -C oracle`"
                                  " where the reference tree is present")
        L = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_free.argtypes = [C.c_void_p]
        L.ref_read_mtx.argtypes = [C.c_char_p, _i32p, _i32p, _i32p,
                                   C.POINTER(_i32p), C.POINTER(_i32p),
                                   C.POINTER(_f32p)]
        L.ref_coo_to_csr.argtypes = [C.c_int, C.c_int, C.c_int, _i32p, _i32p,
                                     _f32p, C.POINTER(_i32p), C.POINTER(_i32p),
                                     C.POINTER(_f32p)]
        L.ref_csr_to_vcsr.argtypes = [C.c_int, C.c_int, _i32p, _i32p, _f32p,
                                      C.c_int, C.c_int, _i32p,
                                      C.POINTER(C.c_longlong)] + \
            [C.POINTER(_i32p)] * 5 + [C.POINTER(_f32p)]
        _REF = L
    return _REF


def ref_read_mtx(path):
    L = ref_lib()
    M, N, Z = C.c_int(), C.c_int(), C.c_int()
    r, c, v = _i32p(), _i32p(), _f32p()
    rc = L.ref_read_mtx(path.encode(), C.byref(M), C.byref(N), C.byref(Z),
                        C.byref(r), C.byref(c), C.byref(v))
    if rc:
        raise OracleError(rc, L.ref_last_error().decode())
    n = Z.value
    return (M.value, N.value, _take(r, n, np.int32, L.ref_free),
            _take(c, n, np.int32, L.ref_free), _take(v, n, np.float32, L.ref_free))


def ref_coo_to_csr(M, N, rows, cols, vals):
    L = ref_lib()
    rows = np.ascontiguousarray(rows, np.int32)
    cols = np.ascontiguousarray(cols, np.int32)
    vals = np.ascontiguousarray(vals, np.float32)
    rp, cc, vv = _i32p(), _i32p(), _f32p()
    rc = L.ref_coo_to_csr(M, N, len(vals), _p(rows, _i32p), _p(cols, _i32p),
                          _p(vals, _f32p), C.byref(rp), C.byref(cc), C.byref(vv))
    if rc:
        raise OracleError(rc, L.ref_last_error().decode())
    n = len(vals)
    return (_take(rp, M + 1, np.int32, L.ref_free), _take(cc, n, np.int32, L.ref_free),
            _take(vv, n, np.float32, L.ref_free))


def ref_csr_to_vcsr(M, N, row_ptr, col, val, segw, bundle):
    L = ref_lib()
    row_ptr = np.ascontiguousarray(row_ptr, np.int32)
    col = np.ascontiguousarray(col, np.int32)
    val = np.ascontiguousarray(val, np.float32)
    G, P = C.c_int(), C.c_longlong()
    ptrs = [_i32p() for _ in range(5)]
    vptr = _f32p()
    rc = L.ref_csr_to_vcsr(M, N, _p(row_ptr, _i32p), _p(col, _i32p),
                           _p(val, _f32p), segw, bundle, C.byref(G), C.byref(P),
                           *[C.byref(p) for p in ptrs], C.byref(vptr))
    if rc:
        raise OracleError(rc, L.ref_last_error().decode())
    g, p = G.value, P.value
    return dict(M=M, N=N, segw=segw, bundle=bundle, num_groups=g, num_slots=p,
                group_ptr=_take(ptrs[0], g + 1, np.int32, L.ref_free),
                group_depth=_take(ptrs[1], g, np.int32, L.ref_free),
                group_seg_base=_take(ptrs[2], g, np.int32, L.ref_free),
                group_rows=_take(ptrs[3], g * bundle, np.int32, L.ref_free),
                lcol=_take(ptrs[4], p, np.int32, L.ref_free),
                val=_take(vptr, p, np.float32, L.ref_free))


def ref_kernels_available() -> bool:
    return os.path.exists(os.path.join(HERE, "_ref", "libvcsr_ref_kernels.so"))


def ref_kernels_lib():
    """The reference's src/kernels.cu launchers rebuilt for sm_100a."""
    global _REFK
    if _REFK is None:
        path = os.path.join(HERE, "_ref", "libvcsr_ref_kernels.so")
        if not os.path.exists(path):
            raise OracleError(-1, f"{path} missing")
        L = C.CDLL(path)
        L.ref_gpu_csr_spmm.argtypes = [C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_void_p, C.c_void_p, C.c_int,
                                       C.c_void_p, C.c_void_p,
                                       C.POINTER(C.c_float)]
        L.ref_gpu_vcsr_spmm.argtypes = [C.c_int] * 5 + [_i32p] * 4 + \
            [C.c_longlong, _i32p, _f32p, C.c_void_p, C.c_int, C.c_int,
             C.c_void_p, C.c_void_p, C.POINTER(C.c_float)]
        L.ref_gpu_cusparse_spmm.argtypes = [C.c_int, C.c_int, C.c_int] + \
            [C.c_void_p] * 4 + [C.c_int, C.c_void_p]
        L.ref_gpu_cusparse_spmm.restype = C.c_float
        _REFK = L
    return _REFK
