"""Full-size parity for every configuration bench.py times, against the CPU
oracle's CSR sum (src/kernels.cu:15-33 restated in oracle/oracle.c).

Each case builds the plan exactly as bench.py does (max_O = max(O, 512),
target_O = O, TF32 panels for the tensor-core workload) on the full
synthetic matrix with the bench's seeded B.  Where the oracle's full product
is cheap it is compared element-wise (FP32: relative L2 <= 1e-5, and rows
summed in CSR order bit for bit); the 43.5M-entry block-dense matrix at
O = 512 is checked on sampled rows against the FP64 oracle plus the checksum
C 1 = A (B 1) over every row.  The TF32 panel path uses its tolerance, 2e-3.
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5
TF32_TOL = 2e-3


def bench_plan(csr, O, tf32=False):
    return V.Plan(csr, segw=4, bundle=32, max_O=max(O, 512), tf32_panels=tf32, target_O=O)


def bench_b(csr, O, cfg, seed=0):
    dB = torch.empty(csr.N, O, device="cuda")
    V.gen_dense_device(dB, seed + 1000, 0.0 if cfg == "rmat" else -1.0, 1.0)
    return dB


def run(plan, dB, M, O):
    dC = torch.full((M, O), float("nan"), device="cuda")
    plan.spmm(dB, dC)
    torch.cuda.synchronize()
    return dC


def csr_order(plan, O):
    info = plan.info()
    return info["num_split_units"] == 0 and (info["num_long_units"] == 0 or O // 4 >= 32)


@pytest.mark.parametrize("cfg,O", [("fem", 32), ("fem", 512), ("powerlaw", 8),
                                   ("powerlaw", 64), ("powerlaw", 128), ("uniform", 32)])
def test_full_size_elementwise(cfg, O):
    csr = V.gen_csr(cfg, 0)
    plan = bench_plan(csr, O)
    dB = bench_b(csr, O, cfg)
    C = run(plan, dB, csr.M, O).cpu().numpy()
    B = dB.cpu().numpy()
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= TOL
    ref64 = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref64) <= TOL
    if csr_order(plan, O):
        a, b = C + 0.0, ref + 0.0  # +0.0 maps -0 to +0
        assert np.array_equal(a.view(np.int32), b.view(np.int32))


def sampled_and_checksum(csr, C, dB, tol, nsample=600):
    """Sampled rows (the longest included) against the FP64 oracle, and
    C 1 = A (B 1) over every row through the CSR row-wise kernel."""
    lens = np.diff(csr.row_ptr)
    rows = np.unique(np.concatenate([np.argsort(lens)[-8:],
                                     np.random.default_rng(1).integers(0, csr.M, nsample)]))
    B = dB.cpu().numpy()
    Cs = C.cpu().numpy()
    got, want = [], []
    for r in rows:
        sub = V.csr_row_panel(csr, int(r), int(r) + 1)
        want.append(oracle.csr_spmm_f64(1, sub.row_ptr, sub.col, sub.val, B)[0])
        got.append(Cs[r])
    assert rel_l2(np.array(got), np.array(want)) <= tol
    bsum = dB.double().sum(dim=1, keepdim=True).float().contiguous()
    d = V.DeviceCSR(csr)
    y = torch.empty(csr.M, 1, device="cuda")
    V.run_csr_spmm_gpu(csr.M, d.row_ptr, d.col, d.val, bsum, 1, y)
    torch.cuda.synchronize()
    cs = C.double().sum(dim=1)
    err = torch.linalg.norm(cs - y[:, 0].double()) / torch.linalg.norm(cs)
    assert err.item() < max(tol, 1e-5)


@pytest.mark.parametrize("tf32", [False, True])
def test_full_blockdense_o512(tf32):
    csr = V.gen_csr("blockdense", 0)
    O = 512
    plan = bench_plan(csr, O, tf32)
    if tf32:
        assert plan.info()["num_panel_blocks"] > 100000
    dB = bench_b(csr, O, "blockdense")
    C = run(plan, dB, csr.M, O)
    if tf32:
        plan.check()
    assert bool(torch.isfinite(C).all())
    sampled_and_checksum(csr, C, dB, TF32_TOL if tf32 else TOL)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_full_fem_16bit_b(dtype):
    """16-bit B widened as it is loaded, FP32 sums: the oracle on the widened
    values, element-wise."""
    csr = V.gen_csr("fem", 0)
    O = 128
    dB = bench_b(csr, O, "fem").to(getattr(torch, dtype))
    plan = bench_plan(csr, O)
    C = run(plan, dB, csr.M, O).cpu().numpy()
    Bw = dB.float().cpu().numpy()
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, Bw)
    assert rel_l2(C, ref) <= TOL


def test_full_rmat_bf16_b_sampled():
    csr = V.gen_csr("rmat", 0, 22)
    O = 256
    dB = bench_b(csr, O, "rmat").to(torch.bfloat16)
    plan = bench_plan(csr, O)
    C = run(plan, dB, csr.M, O)
    sampled_and_checksum(csr, C, dB.float(), TOL, nsample=300)
