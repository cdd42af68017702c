"""The host-buffer entry point's row transfers (vcsr_spmm_host with page-locked
buffers): only the B rows the product reads go up, only the C rows that hold
an entry come down, and the empty C rows are zeroed on the host.

Contract: pinned and pageable buffers (the row transfers and the full-copy
path) give the same C bit for bit, since both cut O into the same column
chunks; every empty row is exactly zero even when the host buffer held NaN
before the call; untouched B rows (NaN here) are never read; C is within
1e-5 (relative L2) of the oracle's FP64 CSR sum on sampled rows and of the
device-buffer product over all rows (a product over a column chunk may sum a
long row's column groups in another order than one over all of O).
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def device_product(plan, B):
    dB = torch.from_numpy(B).cuda()
    dC = torch.full((plan.M, B.shape[1]), float("nan"), device="cuda")
    plan.spmm(dB, dC)
    torch.cuda.synchronize()
    return dC.cpu().numpy()


def host_product(plan, B, pinned):
    M, O = plan.M, B.shape[1]
    if pinned:
        hB = torch.empty(B.shape, dtype=torch.float32, pin_memory=True)
        hB.copy_(torch.from_numpy(B))
        hC = torch.full((M, O), float("nan"), dtype=torch.float32).pin_memory()
        plan.spmm_host(hB.numpy(), hC.numpy())
        return hC.numpy().copy()
    hC = np.full((M, O), np.nan, np.float32)
    plan.spmm_host(np.ascontiguousarray(B), hC)
    return hC


def holes(csr, row_lo, row_hi, col_lo, col_hi):
    """The CSR with rows [row_lo, row_hi) emptied and columns [col_lo,
    col_hi) dropped."""
    rp, cc, vv = csr.row_ptr, csr.col, csr.val
    rows = np.repeat(np.arange(csr.M), np.diff(rp))
    keep = ~(((rows >= row_lo) & (rows < row_hi)) | ((cc >= col_lo) & (cc < col_hi)))
    nrp = np.zeros(csr.M + 1, np.int64)
    np.add.at(nrp, rows[keep] + 1, 1)
    nrp = np.cumsum(nrp).astype(np.int32)
    return V.CSR(csr.M, csr.N, int(keep.sum()), nrp, cc[keep].astype(np.int32),
                 vv[keep].astype(np.float32))


def touched_and_nonempty(csr):
    cols = np.zeros(csr.N, bool)
    cols[csr.col] = True
    return cols, np.diff(csr.row_ptr) > 0


def check(csr, O, seed, **plan_kw):
    plan = V.Plan(csr, max_O=max(O, 512), **plan_kw)
    rng = np.random.default_rng(seed)
    B = rng.uniform(-1, 1, size=(csr.N, O)).astype(np.float32)
    cols, nonempty = touched_and_nonempty(csr)
    B[~cols] = np.nan  # rows the product never reads
    b_rows, c_rows = plan.host_rows()
    ref_dev = device_product(plan, B)
    got = host_product(plan, B, pinned=True)
    assert not np.isnan(got).any()
    assert (got[~nonempty] == 0).all()
    assert rel_l2(got, ref_dev) <= 1e-5
    sample = np.unique(rng.integers(0, csr.M, size=min(csr.M, 400)))
    rp = csr.row_ptr
    sub_rp = np.concatenate([[0], np.cumsum(rp[sample + 1] - rp[sample])]).astype(np.int32)
    idx = np.concatenate([np.arange(rp[r], rp[r + 1]) for r in sample]).astype(np.int64)
    Bz = np.nan_to_num(B, nan=0.0)
    ref = oracle.csr_spmm_f64(len(sample), sub_rp, csr.col[idx], csr.val[idx], Bz)
    assert rel_l2(got[sample].astype(np.float64), ref) <= 1e-5
    pageable = host_product(plan, B, pinned=False)
    assert np.array_equal(pageable, got)
    return plan, b_rows, c_rows, int(cols.sum()), int(nonempty.sum())


@pytest.mark.parametrize("O", [256, 48, 512])
def test_rmat_rows_only(O):
    csr = V.gen_csr("rmat", 0, 15)
    plan, b_rows, c_rows, n_cols, n_rows = check(csr, O, 3)
    # graph matrix: the entry point moves the touched / non-empty rows only
    assert (b_rows, c_rows) == (n_cols, n_rows)
    assert b_rows < csr.N and c_rows < csr.M
    # a second call reuses the row lists
    again = check(csr, O, 4)[1:3]
    assert again == (b_rows, c_rows)


@pytest.mark.parametrize("vec_rows", [1, 8])
def test_banded_with_holes(vec_rows):
    """Vectors of 8 rows: a row is non-empty when any union entry of its
    vector has its bit in the row mask; a band of empty rows and a band of
    untouched columns."""
    csr = holes(V.gen_csr("fem", 0, 12000), 2000, 5000, 7000, 9500)
    plan, b_rows, c_rows, n_cols, n_rows = check(csr, 128, 5, vec_rows=vec_rows)
    assert plan.info()["vec_rows"] == vec_rows
    assert (b_rows, c_rows) == (n_cols, n_rows)


def test_dense_coverage_takes_full_copies():
    """Every column touched and no empty row: nothing to save, N and M rows."""
    csr = V.gen_csr("fem", 0, 12000)
    plan, b_rows, c_rows, n_cols, n_rows = check(csr, 128, 6)
    assert (b_rows, c_rows) == (csr.N, csr.M)


def test_tf32_panel_plans_take_full_copies():
    csr = V.gen_csr("blockdense", 0, 2048)
    plan = V.Plan(csr, tf32_panels=True)
    assert plan.host_rows() == (csr.N, csr.M)
