"""The tcgen05 TF32 dense-panel path (VCSR_PLAN_TF32_PANELS): dense 16x16
blocks of A on the tensor cores (TF32 inputs, FP32 accumulation in tensor
memory), the residual entries on the FP32 kernel.  Contract: relative L2
<= 2e-3 against the FP64 CSR sum (the TF32 tolerance), deterministic run to
run, and exact on small-integer data (every product and partial sum is then
representable, so TF32 rounding does not enter)."""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL_TF32 = 2e-3


def csr_from_dense(A):
    rows, cols = np.nonzero(A)
    rp = np.zeros(A.shape[0] + 1, np.int32)
    np.add.at(rp, rows + 1, 1)
    return V.CSR(A.shape[0], A.shape[1], len(rows), np.cumsum(rp).astype(np.int32),
                 cols.astype(np.int32), A[rows, cols].astype(np.float32))


def run(csr, B, **kw):
    plan = V.Plan(csr, tf32_panels=True, max_O=max(B.shape[1], 512), **kw)
    dB = torch.from_numpy(B).cuda()
    dC = torch.full((csr.M, B.shape[1]), float("nan"), device="cuda")
    plan.spmm(dB, dC)
    plan.check()
    return plan, dB, dC


def block_matrix(seed, M, N, blocks, resid):
    """Dense 16x16 blocks at random block positions (clipped at the edges)
    plus `resid` random entries per row, values U[-1, 1)."""
    rng = np.random.default_rng(seed)
    nbr, nbc = -(-M // 16), -(-N // 16)
    A = np.zeros((M, N), np.float32)
    for c in rng.choice(nbr * nbc, size=blocks, replace=False):
        bi, bj = divmod(int(c), nbc)
        blk = A[16 * bi:16 * bi + 16, 16 * bj:16 * bj + 16]
        blk[...] = rng.uniform(-1, 1, blk.shape)
    for r in range(M):
        q = rng.integers(0, N, resid)
        A[r, q] = np.where(A[r, q] == 0, rng.uniform(-1, 1, resid), A[r, q])
    return A


def test_tf32_panels_exact_small_integers():
    rng = np.random.default_rng(5)
    A = np.zeros((64, 80), np.float32)
    A[16:32, 32:48] = rng.integers(-3, 4, (16, 16))
    A[48:64, 0:16] = rng.integers(-3, 4, (16, 16))
    A[48:64, 64:80] = rng.integers(-3, 4, (16, 16))
    A[3, 7] = 2.0  # residual entries
    A[40, 70] = -1.0
    B = rng.integers(-4, 5, (80, 256)).astype(np.float32)
    plan, _, dC = run(csr_from_dense(A), B, panel_min_nnz=2)
    info = plan.info()
    assert info["num_panel_blocks"] == 3 and info["num_panel_row_blocks"] == 2
    assert np.array_equal(dC.cpu().numpy(), (A.astype(np.float64) @ B).astype(np.float32))


@pytest.mark.parametrize("O,ldb", [(96, 96), (160, 160), (64, 72), (256, 260), (100, 104)])
def test_tf32_panels_exact_b_views(O, ldb):
    # O a multiple of 32 reads B through the 3-D slab view (one copy per slab),
    # partial last 128-column slices (96, 160) and padded rows (ldb > O)
    # included; O = 100 through the 2-D view.  Small integers: exact.
    rng = np.random.default_rng(O + ldb)
    A = np.zeros((96, 112), np.float32)
    for bi, bj in [(0, 1), (1, 6), (2, 0), (2, 3), (5, 6), (4, 2)]:
        A[16 * bi:16 * bi + 16, 16 * bj:16 * bj + 16] = rng.integers(-3, 4, (16, 16))
    A[7, 100] = 3.0
    Bfull = rng.integers(-4, 5, (112, ldb)).astype(np.float32)
    csr = csr_from_dense(A)
    plan = V.Plan(csr, tf32_panels=True, max_O=512, panel_min_nnz=2)
    assert plan.info()["num_panel_blocks"] == 6
    dB = torch.from_numpy(Bfull).cuda()
    dC = torch.full((96, O), float("nan"), device="cuda")
    plan.spmm(dB, dC, O=O, ldb=ldb, ldc=O)
    plan.check()
    want = (A.astype(np.float64) @ Bfull[:, :O]).astype(np.float32)
    assert np.array_equal(dC.cpu().numpy(), want)


@pytest.mark.parametrize("O", [128, 64, 100, 256])
def test_tf32_panels_blockdense(O):
    csr = V.gen_csr("blockdense", 0, 4096)
    B = V.gen_dense_host(csr.N, O, 3)
    plan, dB, dC = run(csr, B)
    info = plan.info()
    assert info["num_panel_blocks"] > 100
    assert info["panel_nnz"] >= info["num_panel_blocks"] * 128
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    err = rel_l2(dC.cpu().numpy(), ref)
    assert err <= TOL_TF32, err
    C2 = torch.empty_like(dC)
    plan.spmm(dB, C2)
    plan.check()
    assert torch.equal(dC, C2)


def test_tf32_panels_ragged_edges():
    A = block_matrix(1, 1000, 777, 120, 3)  # M, N not multiples of 16
    csr = csr_from_dense(A)
    B = V.gen_dense_host(csr.N, 132, 4)
    plan, _, dC = run(csr, B, panel_min_nnz=64)
    assert plan.info()["num_panel_blocks"] > 50
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(dC.cpu().numpy(), ref) <= TOL_TF32


def test_tf32_panels_host_entry_point():
    csr = V.gen_csr("blockdense", 1, 1024)
    B = V.gen_dense_host(csr.N, 64, 5)
    plan = V.Plan(csr, tf32_panels=True)
    C = np.empty((csr.M, 64), np.float32)
    plan.spmm_host(B, C)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL_TF32


def test_tf32_panels_host_pipeline():
    # 8 MB of B and C: the host entry point runs column chunks of 64 (upload,
    # product on the plan's compute stream, download), each chunk a TF32 call
    # on a 64-column slice of the staged B
    csr = V.gen_csr("blockdense", 2, 4096)
    O = 256
    B = V.gen_dense_host(csr.N, O, 6)
    plan = V.Plan(csr, tf32_panels=True)
    assert plan.info()["num_panel_blocks"] > 100
    C = np.empty((csr.M, O), np.float32)
    plan.spmm_host(B, C)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL_TF32
    dC = torch.empty(csr.M, O, device="cuda")
    plan.spmm(torch.from_numpy(B).cuda(), dC)
    plan.check()
    assert rel_l2(C, dC.cpu().numpy().astype(np.float64)) <= 1e-5
    C2 = np.empty_like(C)
    plan.spmm_host(B, C2)
    assert np.array_equal(C, C2)


def test_tf32_panels_need_aligned_o():
    csr = V.gen_csr("blockdense", 0, 1024)
    plan = V.Plan(csr, tf32_panels=True)
    dB = torch.zeros(csr.N, 30, device="cuda")
    dC = torch.zeros(csr.M, 30, device="cuda")
    with pytest.raises(V.VcsrError) as ei:
        plan.spmm(dB, dC)
    assert ei.value.status == 5


def test_cli_vcsr_tc():
    """spmm_vcsr --algo vcsr_tc runs the TF32 panel path and prints the
    'Name: <ms> ms <gflops> GFLOP/s [..]' line; with O % 4 != 0 it reports N/A."""
    import os
    import subprocess
    from helpers import ROOT
    exe = os.path.join(ROOT, "vcsr-spmm_b200", "bin", "spmm_vcsr")
    out = subprocess.run([exe, "--gen", "blockdense", "--size", "2048", "--O", "64",
                          "--algo", "vcsr_tc", "--repeat", "2"],
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    last = out.stdout.strip().splitlines()[-1]
    assert last.startswith("VCSR_TC:") and "GFLOP/s" in last and "panels=" in last
    na = subprocess.run([exe, "--gen", "blockdense", "--size", "1024", "--O", "30",
                         "--algo", "vcsr_tc", "--repeat", "2"],
                        capture_output=True, text=True, timeout=120)
    assert na.returncode == 0 and "N/A" in na.stdout
