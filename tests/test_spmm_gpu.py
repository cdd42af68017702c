"""GPU parity of the row-stationary VCSR SpMM (vcsr_plan_* / vcsr_spmm)
against the CPU oracle's CSR semantics (src/kernels.cu:15-33 restated).

Contract: FP32 output within relative L2 1e-5 of the oracle.  Rows whose
vector is walked by one column group and not split over several work units
match the oracle's FP32 result bit for bit up to the sign of zero (same FMA
chain in CSR order; padding entries add 0*b).  Split vectors and column groups
are summed in a fixed order, so results are deterministic run to run.
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import random_csr, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def run_plan(csr, B, **kw):
    plan = V.Plan(csr, **kw)
    dB = dev(B)
    dC = torch.full((csr.M, B.shape[1]), float("nan"), device="cuda")
    plan.spmm(dB, dC)
    torch.cuda.synchronize()
    return plan, dC.cpu().numpy()


def csr_of(rp, cc, vv, M, N):
    return V.CSR(M, N, len(vv), rp, cc, vv)


def csr_order(plan, O, aligned=True):
    """True when every row sums its entries in CSR order: no split vectors,
    and long units are walked by one column group (ceil(O / VW) >= 32)."""
    info = plan.info()
    vw = 4 if (aligned and O % 4 == 0) else 1
    return info["num_split_units"] == 0 and (info["num_long_units"] == 0 or -(-O // vw) >= 32)


def bitwise_rows(C, ref, rows):
    a = C[rows] + 0.0  # +0.0 maps -0 to +0
    b = ref[rows] + 0.0
    return np.array_equal(a.view(np.int32), b.view(np.int32))


@pytest.mark.parametrize("O", [1, 3, 8, 32, 64, 128, 256, 512])
@pytest.mark.parametrize("R", [0, 1, 2, 4, 8, 16])
def test_uniform_config_all_shapes(O, R):
    csr = V.gen_csr("uniform", 0)
    B = V.gen_dense_host(csr.N, O, 7)
    plan, C = run_plan(csr, B, vec_rows=R)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL
    if csr_order(plan, O):
        assert bitwise_rows(C, ref, slice(None))


@pytest.mark.parametrize("cfg,size,O", [("fem", 6000, 128), ("fem", 3001, 32),
                                        ("powerlaw", 40000, 8), ("powerlaw", 40000, 64),
                                        ("rmat", 14, 256), ("blockdense", 2048, 512),
                                        ("blockdense", 1024, 100)])
def test_configs_scaled(cfg, size, O):
    csr = V.gen_csr(cfg, 0, size)
    lo = 0.0 if cfg == "rmat" else -1.0
    B = V.gen_dense_host(csr.N, O, 11, lo, 1.0)
    plan, C = run_plan(csr, B, max_O=512)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    ref64 = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL
    assert rel_l2(C, ref64) <= TOL


def test_split_rows_deterministic_and_correct():
    # dense rows forced into many parts
    rp, cc, vv = random_csr(3, 300, 5000, 0.002, dense_rows=(0, 17, 299))
    csr = csr_of(rp, cc, vv, 300, 5000)
    B = V.gen_dense_host(5000, 64, 2)
    plan, C1 = run_plan(csr, B, vec_rows=1, chunk=97)
    info = plan.info()
    assert info["num_split_vectors"] == 3 and info["num_split_units"] > 100
    dB, dC = dev(B), torch.zeros(300, 64, device="cuda")
    for _ in range(3):  # tickets reset between launches
        plan.spmm(dB, dC)
    torch.cuda.synchronize()
    C2 = dC.cpu().numpy()
    assert np.array_equal(C1.view(np.int32), C2.view(np.int32))
    ref = oracle.csr_spmm_f32(300, rp, cc, vv, B)
    assert rel_l2(C1, ref) <= TOL
    unsplit = [r for r in range(300) if r not in (0, 17, 299)]
    assert bitwise_rows(C1, ref, unsplit)


@pytest.mark.parametrize("R", [2, 4, 8, 16])
def test_split_vectors_with_many_rows(R):
    rp, cc, vv = random_csr(4, 100, 3000, 0.01, dense_rows=(5, 6, 50))
    csr = csr_of(rp, cc, vv, 100, 3000)
    B = V.gen_dense_host(3000, 40, 5)
    plan, C = run_plan(csr, B, vec_rows=R, chunk=64, max_O=40)
    assert plan.info()["num_split_units"] > 0
    assert rel_l2(C, oracle.csr_spmm_f32(100, rp, cc, vv, B)) <= TOL


def test_edge_cases_empty_rows_duplicates_unsorted():
    rp, cc, vv = random_csr(9, 77, 45, 0.05, dup_rows=(2, 3, 40))
    lens = np.diff(rp)
    assert (lens == 0).any()
    for unsorted in (False, True):
        rp2, cc2, vv2 = random_csr(9, 77, 45, 0.05, dup_rows=(2, 3, 40),
                                   unsorted=unsorted)
        csr = csr_of(rp2, cc2, vv2, 77, 45)
        B = V.gen_dense_host(45, 12, 1)
        ref = oracle.csr_spmm_f64(77, rp2, cc2, vv2, B)
        for R in (1, 4, 16):
            _, C = run_plan(csr, B, vec_rows=R)
            assert rel_l2(C, ref) <= TOL, (unsorted, R)
            assert np.all(C[lens == 0] == 0)


def test_empty_matrix_and_zero_O():
    csr = csr_of(np.zeros(6, np.int32), np.zeros(0, np.int32),
                 np.zeros(0, np.float32), 5, 4)
    B = V.gen_dense_host(4, 8, 1)
    _, C = run_plan(csr, B)
    assert np.all(C == 0)
    plan = V.Plan(csr)
    plan.spmm(dev(B), torch.zeros(5, 8, device="cuda"), O=0)
    m0 = csr_of(np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0, np.float32),
                0, 4)
    V.Plan(m0).spmm(dev(B), torch.zeros(0, 8, device="cuda"))


def test_leading_dimensions_and_unaligned_pointers():
    csr = V.gen_csr("fem", 0, 1500)
    B = V.gen_dense_host(csr.N, 70, 3)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    plan = V.Plan(csr)
    # padded leading dimensions (ldb = 72, ldc = 80)
    dBp = torch.zeros(csr.N, 72, device="cuda")
    dBp[:, :70] = dev(B)
    dCp = torch.full((csr.M, 80), 7.0, device="cuda")
    plan.spmm(dBp, dCp, O=70, ldb=72, ldc=80)
    torch.cuda.synchronize()
    Cp = dCp.cpu().numpy()
    assert rel_l2(Cp[:, :70], ref) <= TOL
    assert np.all(Cp[:, 70:] == 7.0)  # untouched beyond O
    # pointers off 16-byte alignment take the scalar path
    big = torch.zeros(csr.N * 70 + 1, device="cuda")
    big[1:] = dev(B).reshape(-1)
    outb = torch.zeros(csr.M * 70 + 1, device="cuda")
    plan.spmm(big.data_ptr() + 4, outb.data_ptr() + 4, O=70, ldb=70, ldc=70)
    torch.cuda.synchronize()
    assert rel_l2(outb[1:].cpu().numpy().reshape(csr.M, 70), ref) <= TOL


def test_errors_are_reported_not_fatal():
    csr = V.gen_csr("powerlaw", 0, 30000)
    plan = V.Plan(csr, max_O=16, vec_rows=1)
    assert plan.info()["num_split_units"] > 0
    B = torch.zeros(csr.N, 32, device="cuda")
    C = torch.zeros(csr.M, 32, device="cuda")
    with pytest.raises(V.VcsrError) as ei:
        plan.spmm(B, C)  # O=32 > max_O=16 with split rows
    assert ei.value.status == 1
    with pytest.raises(V.VcsrError):
        plan.spmm(B, C, O=32, ldb=16, ldc=32)
    bad = csr_of(np.array([0, 1], np.int32), np.array([5], np.int32),
                 np.array([1], np.float32), 1, 3)
    with pytest.raises(V.VcsrError) as ei:
        V.Plan(bad)
    assert ei.value.status == 8


def test_device_csr_input_and_host_entry_point():
    csr = V.gen_csr("fem", 0, 3000)
    B = V.gen_dense_host(csr.N, 32, 9)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    plan = V.Plan(V.DeviceCSR(csr))
    C = np.zeros((csr.M, 32), np.float32)
    plan.spmm_host(B, C)
    assert rel_l2(C, ref) <= TOL
    C2 = np.zeros_like(C)
    plan.spmm_host(B, C2)
    assert np.array_equal(C, C2)


@pytest.mark.parametrize("cfg,O,pinned", [("fem", 128, True), ("fem", 200, False),
                                          ("powerlaw", 128, True), ("uniform", 512, True)])
def test_host_entry_point_pipelined(cfg, O, pinned):
    """Above 8 MB of B and C the host entry point overlaps transfers and work
    (row panels for the banded FEM matrix, column chunks for the power-law and
    uniform ones); the result equals the device entry point's, run after run,
    pinned host memory or not."""
    csr = V.gen_csr(cfg, 0)
    B = V.gen_dense_host(csr.N, O, 5)
    plan = V.Plan(csr)
    dC = torch.empty(csr.M, O, device="cuda")
    plan.spmm(torch.from_numpy(B).cuda(), dC)
    ref = dC.cpu().numpy()
    if pinned:
        hB = torch.from_numpy(B).pin_memory()
        hC = torch.full((csr.M, O), float("nan")).pin_memory()
        Bn, Cn = hB.numpy(), hC.numpy()
    else:
        Bn, Cn = B, np.full((csr.M, O), np.nan, np.float32)
    for _ in range(2):
        Cn[...] = np.nan
        plan.spmm_host(Bn, Cn)
        assert rel_l2(Cn, ref) <= 1e-6
        if cfg == "fem":  # no split or long units: the same sums, bit for bit
            assert np.array_equal(Cn, ref)


def test_full_fem_o128_against_oracle():
    """The bench workload at full size, checked element-wise."""
    csr = V.gen_csr("fem", 0)
    dB = torch.empty(csr.N, 128, device="cuda")
    V.gen_dense_device(dB, 42)
    B = dB.cpu().numpy()
    assert np.array_equal(B, V.gen_dense_host(csr.N, 128, 42))  # device == host bits
    plan = V.Plan(csr)
    dC = torch.empty(csr.M, 128, device="cuda")
    plan.spmm(dB, dC)
    torch.cuda.synchronize()
    C = dC.cpu().numpy()
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL
    if csr_order(plan, 128):
        assert bitwise_rows(C, ref, slice(None))


def test_full_rmat_properties():
    """R-MAT scale 22, O = 256: sampled rows against the oracle, plus
    linearity A(B1 + B2) = A B1 + A B2 and the checksum C 1 = A (B 1)."""
    csr = V.gen_csr("rmat", 0, 22)
    plan = V.Plan(csr, max_O=256)
    O = 256
    dB1 = torch.empty(csr.N, O, device="cuda")
    dB2 = torch.empty(csr.N, O, device="cuda")
    V.gen_dense_device(dB1, 1)
    V.gen_dense_device(dB2, 2)
    C1 = torch.empty(csr.M, O, device="cuda")
    C2 = torch.empty_like(C1)
    C12 = torch.empty_like(C1)
    plan.spmm(dB1, C1)
    plan.spmm(dB2, C2)
    plan.spmm(dB1 + dB2, C12)
    torch.cuda.synchronize()
    lin = torch.linalg.norm((C12 - C1 - C2).double()) / torch.linalg.norm(C12.double())
    assert lin.item() < 1e-6
    # checksum through the CSR row-wise kernel with O = 1
    ones = dB1.double().sum(dim=1, keepdim=True).float().contiguous()
    dcsr = V.DeviceCSR(csr)
    y = torch.empty(csr.M, 1, device="cuda")
    V.run_csr_spmm_gpu(csr.M, dcsr.row_ptr, dcsr.col, dcsr.val, ones, 1, y)
    torch.cuda.synchronize()
    cs = C1.double().sum(dim=1)
    err = torch.linalg.norm(cs - y[:, 0].double()) / torch.linalg.norm(cs)
    assert err.item() < 1e-5
    # sampled rows (heaviest rows included) against the oracle
    lens = np.diff(csr.row_ptr)
    rows = np.unique(np.concatenate([np.argsort(lens)[-8:],
                                     np.random.default_rng(0).integers(0, csr.M, 400)]))
    B1 = dB1.cpu().numpy()
    Cs = C1.cpu().numpy()
    for r in rows:
        sub = V.csr_row_panel(csr, int(r), int(r) + 1)
        ref = oracle.csr_spmm_f64(1, sub.row_ptr, sub.col, sub.val, B1)
        assert rel_l2(Cs[r:r + 1], ref) <= TOL


def test_repeat_runs_bitwise_identical():
    csr = V.gen_csr("powerlaw", 0)
    dB = torch.empty(csr.N, 64, device="cuda")
    V.gen_dense_device(dB, 5)
    plan = V.Plan(csr)
    outs = []
    for _ in range(3):
        dC = torch.empty(csr.M, 64, device="cuda")
        plan.spmm(dB, dC)
        outs.append(dC)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    B = dB.cpu().numpy()
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(outs[0].cpu().numpy(), ref) <= TOL


def test_target_o_picks_vector_height():
    """target_O > 128 turns an automatic 8-row choice into 4 rows; results
    stay within the FP32 tolerance either way; an explicit vec_rows wins."""
    csr = V.gen_csr("fem", 0, 6000)
    assert V.Plan(csr).info()["vec_rows"] == 8
    assert V.Plan(csr, target_O=128).info()["vec_rows"] == 8
    p = V.Plan(csr, target_O=512)
    assert p.info()["vec_rows"] == 4
    assert V.Plan(csr, target_O=512, vec_rows=8).info()["vec_rows"] == 8
    B = V.gen_dense_host(csr.N, 256, 3)
    C = torch.empty(csr.M, 256, device="cuda")
    p.spmm(torch.from_numpy(B).cuda(), C)
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C.cpu().numpy(), ref) <= TOL


def test_row_panels_compose_the_product():
    """vcsr_spmm_row_panel over all of a plan's row panels writes exactly
    the product vcsr_spmm writes, bit for bit; other rows are left alone."""
    for cfg, size in (("fem", 0), ("powerlaw", 0)):
        csr = V.gen_csr(cfg, 1, size)
        plan = V.Plan(csr)
        panels = plan.row_panels()
        assert panels and panels[0][0] == 0 and panels[-1][1] == csr.M
        assert all(a[1] == b[0] for a, b in zip(panels[:-1], panels[1:]))
        B = torch.randn(csr.N, 64, device="cuda")
        C1 = torch.empty(csr.M, 64, device="cuda")
        plan.spmm(B, C1)
        C2 = torch.full((csr.M, 64), float("nan"), device="cuda")
        for j in range(len(panels)):
            plan.spmm_row_panel(j, B, C2)
        torch.cuda.synchronize()
        assert torch.equal(C1, C2)
        C3 = torch.full((csr.M, 64), 7.0, device="cuda")
        a, b, _ = panels[1]
        plan.spmm_row_panel(1, B, C3)
        torch.cuda.synchronize()
        assert torch.equal(C3[a:b], C1[a:b]) and bool((C3[:a] == 7).all()) and bool((C3[b:] == 7).all())
    with pytest.raises(V.VcsrError) as ei:
        plan.spmm_row_panel(len(panels), B, C1)
    assert ei.value.status == 8
    assert V.Plan(V.gen_csr("fem", 0, 3000)).row_panels() == []  # small plans have none
