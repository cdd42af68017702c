"""Timing of the reference's own GPU kernels rebuilt for sm_100a
(_ref/libref_gpu.so, see ref_gpu_shim.cu), as benchmark peers of the engine.

time_all() runs each kernel on the input it takes and reports GFLOP/s =
2*nnz*O / (its own event time of the kernel alone), the L2 flushed before
every call, as the reference's harness reports them (src/main.cpp:111).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libref_gpu.so")
_L = None
_vp, _i32p, _f32p = C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_float)


def lib():
    global _L
    if _L is None:
        if not os.path.exists(LIB):
            raise FileNotFoundError(LIB)
        L = C.CDLL(LIB)
        L.ref_gpu_csr.argtypes = [C.c_int, _vp, _vp, _vp, _vp, C.c_int, _vp, _vp, _f32p]
        L.ref_gpu_aspt.argtypes = [C.c_int, _vp, _vp, _vp, _vp, C.c_int, _vp, _vp, _f32p]
        L.ref_vcsr_create.argtypes = [C.c_int] * 5 + [_i32p] * 4 + [C.c_longlong, _i32p, _f32p]
        L.ref_vcsr_create.restype = _vp
        L.ref_vcsr_run.argtypes = [_vp, C.c_int, _vp, C.c_int, C.c_int, _vp, _vp, _f32p]
        L.ref_vcsr_destroy.argtypes = [_vp, _vp]
        _L = L
    return _L


def _p(a, t):
    return np.ascontiguousarray(a).ctypes.data_as(t)


def time_all(torch, V, csr, dB32, O, flush, stream, flops, reps, tileK=64, segw=4, bundle=32):
    L = lib()
    st = C.c_void_p(stream.cuda_stream)
    out = {"note": "each kernel's own CUDA-event time, L2 flushed before every call; "
                   "VCSR kernels on the engine's GPU-built reference format"}
    # B padded to whole segments (the segment kernels read segw rows at a time)
    Np = -(-csr.N // segw) * segw
    Bp = torch.zeros(Np + segw, O, device=dB32.device)
    Bp[:csr.N] = dB32
    dC = torch.zeros(csr.M, O, device=dB32.device)
    d = V.DeviceCSR(csr)
    ms = C.c_float()

    def run(fn):
        ts = []
        for _ in range(reps):
            flush.zero_()
            torch.cuda.synchronize()
            rc = fn()
            torch.cuda.synchronize()
            if rc != 0:
                raise RuntimeError(f"launcher returned {rc}")
            ts.append(ms.value)
        return round(flops / (float(np.mean(ts)) * 1e-3) / 1e9, 2)

    out["csr_spmm_kernel"] = run(lambda: L.ref_gpu_csr(
        csr.M, d.row_ptr.data_ptr(), d.col.data_ptr(), d.val.data_ptr(), Bp.data_ptr(), O,
        dC.data_ptr(), st, C.byref(ms)))
    if O % 64 == 0:
        # ASpT loads 32 entries at a time in long rows: 32 entries of padding
        colp = torch.zeros(csr.nnz + 32, dtype=torch.int32, device=dB32.device)
        valp = torch.zeros(csr.nnz + 32, dtype=torch.float32, device=dB32.device)
        colp[:csr.nnz] = d.col
        valp[:csr.nnz] = d.val
        out["aspt_spmm_kernel"] = run(lambda: L.ref_gpu_aspt(
            csr.M, d.row_ptr.data_ptr(), colp.data_ptr(), valp.data_ptr(), Bp.data_ptr(), O,
            dC.data_ptr(), st, C.byref(ms)))
        del colp, valp
    else:
        out["aspt_spmm_kernel"] = "N/A (needs O % 64 == 0)"
    v = V.csr_to_vcsr_spmm(d, segw=segw, bundle=bundle).to_host()
    G = len(v.group_depth)
    h = L.ref_vcsr_create(csr.M, csr.N, segw, bundle, G, _p(v.group_ptr, _i32p),
                          _p(v.group_depth, _i32p), _p(v.group_seg_base, _i32p),
                          _p(v.group_rows, _i32p), len(v.lcol), _p(v.lcol, _i32p),
                          _p(v.val, _f32p))
    try:
        for which, name in ((0, "vcsr_spmm_kernel"), (1, "vcsr_opt_kernel"),
                            (2, "vcsr_seg_prefetch_kernel")):
            out[name] = run(lambda: L.ref_vcsr_run(h, which, Bp.data_ptr(), O, tileK,
                                                   dC.data_ptr(), st, C.byref(ms)))
    finally:
        L.ref_vcsr_destroy(h, st)
    out["tileK"] = tileK
    del Bp, dC, d
    return out
