"""Host-side parts of the engine library, runnable without a GPU:
the C ABI surface, Matrix Market input and COO -> CSR against the reference's
golden outputs, the synthetic generators and the row partitioner."""
import ctypes
import os
import re

import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import MTX_DIR, ROOT, golden_cases, golden_errors

HEADER = os.path.join(ROOT, "include", "vcsr_spmm.h")


def header_functions():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    names = re.findall(r"\b(vcsr_[a-z0-9_]+)\s*\(", txt)
    return sorted(set(n for n in names))


def test_library_loads_and_exports_every_header_symbol():
    L = V.lib()
    declared = header_functions()
    assert len(declared) >= 25
    for name in declared:
        assert hasattr(L, name), name          # exported by the .so
        assert name in V.exported_names(), name  # and bound in Python
    assert L.vcsr_abi_version() == 3


def test_status_strings_and_last_error():
    L = V.lib()
    for s in range(9):
        assert L.vcsr_status_string(s)
    with pytest.raises(V.VcsrError) as ei:
        V.gen_csr("nope")
    assert ei.value.status == 1 and "unknown config" in ei.value.msg


@pytest.mark.parametrize("fname", sorted(os.listdir(MTX_DIR)))
def test_read_mtx_matches_reference(golden, fname):
    key = fname[:-4]
    errs = golden_errors(golden)
    path = os.path.join(MTX_DIR, fname)
    if key in errs and errs[key]["stage"] == "read":
        with pytest.raises(V.VcsrError) as ei:
            V.read_matrix_market_coo(path)
        assert ei.value.status == 4
        assert errs[key]["msg"] in ei.value.msg
        return
    coo = V.read_matrix_market_coo(path)
    assert [coo.M, coo.N] == list(golden[f"{key}/coo_shape"])
    assert np.array_equal(coo.rows, golden[f"{key}/coo_rows"])
    assert np.array_equal(coo.cols, golden[f"{key}/coo_cols"])
    assert np.array_equal(coo.vals.view(np.int32), golden[f"{key}/coo_vals"].view(np.int32))


def test_missing_file_is_io_error():
    with pytest.raises(V.VcsrError) as ei:
        V.read_matrix_market_coo("/nonexistent/x.mtx")
    assert ei.value.status == 4


def test_coo_to_csr_matches_reference(golden):
    errs = golden_errors(golden)
    for case in golden_cases(golden):
        if f"{case}/coo_shape" not in golden.files:
            continue
        M, N = (int(x) for x in golden[f"{case}/coo_shape"])
        coo = V.COO(M, N, golden[f"{case}/coo_rows"], golden[f"{case}/coo_cols"],
                    golden[f"{case}/coo_vals"])
        if case in errs and errs[case]["stage"] == "coo_to_csr":
            with pytest.raises(V.VcsrError) as ei:
                V.coo_to_csr(coo)
            assert ei.value.status == 8
            assert "row idx out of range" in ei.value.msg
            continue
        csr = V.coo_to_csr(coo)
        assert np.array_equal(csr.row_ptr, golden[f"{case}/csr_row_ptr"]), case
        assert np.array_equal(csr.col, golden[f"{case}/csr_col"]), case
        assert np.array_equal(csr.val, golden[f"{case}/csr_val"]), case


def test_coo_to_csr_rejects_bad_column():
    coo = V.COO(2, 2, np.array([0, 1], np.int32), np.array([0, 2], np.int32),
                np.array([1, 2], np.float32))
    with pytest.raises(V.VcsrError) as ei:
        V.coo_to_csr(coo)
    assert ei.value.status == 8


def test_coo_to_csr_long_rows_stable():
    rng = np.random.default_rng(0)
    M, N, n = 5, 40, 400
    rows = rng.integers(0, M, n).astype(np.int32)
    cols = rng.integers(0, N, n).astype(np.int32)
    vals = rng.standard_normal(n).astype(np.float32)
    csr = V.coo_to_csr(V.COO(M, N, rows, cols, vals))
    rp, cc, vv = oracle.coo_to_csr(M, N, rows, cols, vals)
    assert np.array_equal(csr.row_ptr, rp)
    assert np.array_equal(csr.col, cc)
    assert np.array_equal(csr.val, vv)


def _check_csr(csr):
    rp = csr.row_ptr
    assert rp[0] == 0 and rp[-1] == csr.nnz and np.all(np.diff(rp) >= 0)
    assert csr.col.min() >= 0 and csr.col.max() < csr.N
    for r in range(0, csr.M, max(1, csr.M // 50)):
        c = csr.col[rp[r]:rp[r + 1]]
        assert np.all(np.diff(c) >= 0)


@pytest.mark.parametrize("cfg,size", [("uniform", 0), ("fem", 3000), ("powerlaw", 20000),
                                      ("rmat", 12), ("blockdense", 1024)])
def test_generators_deterministic(cfg, size):
    a = V.gen_csr(cfg, 0, size)
    b = V.gen_csr(cfg, 0, size)
    c = V.gen_csr(cfg, 1, size)
    _check_csr(a)
    assert np.array_equal(a.row_ptr, b.row_ptr) and np.array_equal(a.col, b.col)
    assert np.array_equal(a.val, b.val)
    assert not (a.nnz == c.nnz and np.array_equal(a.col, c.col) and np.array_equal(a.val, c.val))


def test_generator_shapes_and_statistics():
    u = V.gen_csr("uniform")
    assert (u.M, u.N, u.nnz) == (4096, 4096, 65536)
    assert np.all(np.diff(u.row_ptr) == 16)
    assert np.all(np.diff(u.col.reshape(4096, 16), axis=1) > 0)  # distinct
    assert u.val.min() >= -1 and u.val.max() < 1
    f = V.gen_csr("fem", 0, 6000)
    lens = np.diff(f.row_ptr)
    assert 55 < lens.mean() < 73
    rows = np.repeat(np.arange(f.M), lens)
    assert np.abs(f.col - rows).max() <= 500
    # symmetric pattern and values
    key = set(zip(rows.tolist(), f.col.tolist()))
    assert all((c, r) in key for r, c in list(key)[:2000])
    # diagonal = |off-diagonal row sum| + 1
    for r in range(0, f.M, 997):
        s, e = f.row_ptr[r], f.row_ptr[r + 1]
        cols, vals = f.col[s:e], f.val[s:e]
        off = vals[cols != r].astype(np.float64).sum()
        assert abs(vals[cols == r][0] - (abs(off) + 1)) < 1e-5
    b = V.gen_csr("blockdense", 0, 2048)
    assert b.nnz > 2048 * 8


def test_dense_generator_host_bits():
    a = V.gen_dense_host(5, 7, 3)
    b = V.gen_dense_host(5, 7, 3)
    assert np.array_equal(a, b) and a.min() >= -1 and a.max() < 1
    # values are multiples of 2^-23 in [-1, 1)
    assert np.all(np.round(a * 2 ** 23) == a * 2 ** 23)


def test_partition_rows_balanced():
    f = V.gen_csr("fem", 0, 9000)
    for parts in (1, 2, 3, 4, 8):
        cuts = V.partition_rows(f.row_ptr, parts, 32)
        assert cuts[0] == 0 and cuts[-1] == f.M and np.all(np.diff(cuts) >= 0)
        assert all(c % 32 == 0 for c in cuts[:-1])
        nnz = np.diff(f.row_ptr[cuts])
        assert nnz.max() - nnz.min() <= 2 * 32 * 80  # within an align window
    # weighted cuts: row r weighs nnz_r + w; w = 0 is the unweighted cut, and a
    # matrix whose first half has long rows gets more of its short rows per
    # panel as w grows
    rp = np.concatenate([[0], np.cumsum(np.r_[np.full(1000, 40), np.full(3000, 2)])]).astype(np.int32)
    assert np.array_equal(V.partition_rows(rp, 4, 8, 0.0), V.partition_rows(rp, 4, 8))
    prev = None
    for w in (0.0, 2.0, 10.0, 100.0):
        cuts = V.partition_rows(rp, 2, 8, w)
        cost = np.diff(rp[cuts]) + w * np.diff(cuts)
        assert abs(cost[0] - cost[1]) <= 8 * (40 + w) + 1
        if prev is not None:
            assert cuts[1] >= prev
        prev = cuts[1]
    with pytest.raises(V.VcsrError):
        V.partition_rows(rp, 2, 8, -1.0)
    p = V.csr_row_panel(f, 100, 200)
    assert p.M == 100 and p.N == f.N
    assert np.array_equal(p.col, f.col[f.row_ptr[100]:f.row_ptr[200]])
