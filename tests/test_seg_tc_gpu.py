"""Tensor-core segments (VCSR_PLAN_TC_SEGMENTS): column runs of 16-row
blocks on tcgen05 with every value split into a TF32 high part and
remainder, against the oracle's CSR sum.

Contract: FP32 accuracy, relative L2 <= 1e-5 against the FP64 CSR sum (the
split product's error is about 2^-22 per product); exact on small-integer
data (every part and partial sum representable), which pins the operand
layouts; the NaN / +Inf / -Inf pattern of C equals the CSR sum's for
non-finite B (recomputed outputs); deterministic run to run; plans survive a
save and load.
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import random_csr, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def product(plan, B, M):
    dB = torch.from_numpy(np.ascontiguousarray(B)).cuda()
    dC = torch.full((M, B.shape[1]), float("nan"), device="cuda")
    plan.spmm(dB, dC)
    plan.check()
    return dC.cpu().numpy()


@pytest.mark.parametrize("cfg,size,O,kw", [
    ("fem", 6000, 128, {}),
    ("fem", 6000, 32, {}),
    ("fem", 6000, 512, {}),
    ("fem", 3001, 100, {}),               # O % 32 != 0: 2-D boxes; M % 16 != 0
    ("fem", 3001, 64, {"seg_min_run": 8}),  # short runs to the residual
    ("fem", 6000, 256, {"seg_min_run": 40}),
    ("blockdense", 2048, 512, {}),        # dense blocks on the tensor cores + residual
    ("blockdense", 2048, 128, {"seg_min_run": 1}),
    ("uniform", 0, 64, {"seg_min_run": 1}),
])
def test_segments_match_oracle(cfg, size, O, kw):
    csr = V.gen_csr(cfg, 0, size)
    plan = V.Plan(csr, tc_segments=True, max_O=512, **kw)
    info = plan.info()
    assert info["num_seg_row_blocks"] > 0 and info["num_seg_pieces"] > 0
    B = V.gen_dense_host(csr.N, O, 17)
    C = product(plan, B, csr.M)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL, rel_l2(C, ref)
    C2 = product(plan, B, csr.M)
    assert np.array_equal(C, C2)  # deterministic


def test_fem_has_no_residual():
    """FEM's three-column runs are padded rather than left to a residual, so
    the segment kernel writes C alone."""
    plan = V.Plan(V.gen_csr("fem", 0, 6000), tc_segments=True)
    info = plan.info()
    assert info["seg_only"] == 1 and info["panel_nnz"] == info["nnz"]
    assert plan.info()["num_seg_row_blocks"] == -(-6000 // 16)


@pytest.mark.parametrize("cfg,size,O", [("fem", 3000, 128), ("blockdense", 1024, 96),
                                        ("fem", 1001, 32)])
def test_small_integers_are_exact(cfg, size, O):
    """Integer A and B of small magnitude: every TF32 part is exact (the low
    parts are zero) and every sum fits FP32's 24 bits, so C equals the CSR sum
    bit for bit -- any misplaced operand would show."""
    csr = V.gen_csr(cfg, 0, size)
    rng = np.random.default_rng(3)
    val = rng.integers(-4, 5, csr.nnz).astype(np.float32)
    csr = V.CSR(csr.M, csr.N, csr.nnz, csr.row_ptr, csr.col, val)
    B = rng.integers(-8, 9, (csr.N, O)).astype(np.float32)
    plan = V.Plan(csr, tc_segments=True)
    C = product(plan, B, csr.M)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert np.array_equal(C + 0.0, ref + 0.0)


def test_nonfinite_b_matches_csr():
    csr = V.gen_csr("fem", 0, 4000)
    B = V.gen_dense_host(csr.N, 128, 9)
    rng = np.random.default_rng(1)
    for c in rng.choice(csr.N, 30, replace=False):
        ks = rng.choice(128, 16, replace=False)
        B[c, ks] = rng.choice(np.array([np.inf, -np.inf, np.nan], np.float32), 16)
    plan = V.Plan(csr, tc_segments=True)
    C = product(plan, B, csr.M)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert np.array_equal(np.isnan(C), np.isnan(ref))
    assert np.array_equal(np.isposinf(C), np.isposinf(ref))
    assert np.array_equal(np.isneginf(C), np.isneginf(ref))
    fin = np.isfinite(ref)
    assert rel_l2(C[fin], ref[fin]) <= TOL


def test_unsorted_duplicates_empty_rows():
    """Unsorted rows with duplicates (summed into one tile value in CSR order),
    a dense row and a run of 40 empty rows (written as zeros)."""
    full_rp, full_col, full_val = random_csr(5, 333, 501, 0.05, dup_rows=range(0, 333, 7),
                                             dense_rows=(10,), unsorted=True)
    lens = np.diff(full_rp)
    lens[100:140] = 0
    new_rp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    idx = np.concatenate([np.arange(full_rp[r], full_rp[r] + lens[r]) for r in range(333)])
    csr = V.CSR(333, 501, len(idx), new_rp, full_col[idx], full_val[idx])
    B = V.gen_dense_host(501, 64, 2)
    plan = V.Plan(csr, tc_segments=True, seg_min_run=1)
    C = product(plan, B, 333)
    ref = oracle.csr_spmm_f64(333, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL
    assert np.all(C[100:140] == 0)


def test_save_load_and_host_entry_point(tmp_path):
    csr = V.gen_csr("blockdense", 0, 1024)
    plan = V.Plan(csr, tc_segments=True)
    path = str(tmp_path / "s.plan")
    plan.save(path)
    loaded = V.Plan.load(path)
    assert loaded.info()["num_seg_pieces"] == plan.info()["num_seg_pieces"]
    B = V.gen_dense_host(csr.N, 128, 5)
    assert np.array_equal(product(plan, B, csr.M), product(loaded, B, csr.M))
    Ch = np.zeros((csr.M, 128), np.float32)
    loaded.spmm_host(B, Ch)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(Ch, ref) <= TOL


def test_no_run_long_enough():
    """A plan whose runs are all shorter than seg_min_run has no pieces: the
    FP32 kernel computes everything."""
    csr = V.gen_csr("uniform", 0, 256)
    plan = V.Plan(csr, tc_segments=True, seg_min_run=1000)
    assert plan.info()["num_seg_pieces"] == 0
    B = V.gen_dense_host(csr.N, 16, 4)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(product(plan, B, csr.M), ref) <= TOL


def test_refusals():
    csr = V.gen_csr("fem", 0, 600)
    plan = V.Plan(csr, tc_segments=True)
    C = torch.empty(csr.M, 30, device="cuda")
    with pytest.raises(V.VcsrError) as ei:  # O % 4 != 0
        plan.spmm(torch.zeros(csr.N, 30, device="cuda"), C)
    assert ei.value.status == 5
    with pytest.raises(V.VcsrError) as ei:
        V.Plan(csr, tc_segments=True, tf32_panels=True)
    assert ei.value.status == 1
    with pytest.raises(V.VcsrError) as ei:
        V.Plan(csr, tc_segments=True, host_build=True)
    assert ei.value.status == 5
