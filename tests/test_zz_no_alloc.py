"""The allocation-free CSR SpMM entry point (vcsr_csr_spmm_noalloc).

It serves callers that may not allocate device memory, for instance a solver
inside an application whose framework has already handed all free device
memory to its own pool.  Its scratch for split long rows is one fixed array
compiled into the library, so this file checks, through the C ABI, that two
calls in a row give the same C as the ordinary entry point (vcsr_csr_spmm)
and as the CPU oracle's CSR sum, within the engine's tolerance, on matrices
whose long rows are split (one and two 256-column tiles of O, 128-bit and
scalar lanes); that sizes past the fixed limits are refused with an error,
both the one checked on the host (O) and the two the device detects (too many
long rows, too many parts); and that a call after a refused one is correct
again.  It is collected last and needs no state from other tests.
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5
SPLIT = 4096        # VCSR_NOALLOC_SPLIT: rows longer than this are cut into parts
MAX_LONG = 1024     # VCSR_NOALLOC_MAX_LONG_ROWS
MAX_PARTS = 2048    # VCSR_NOALLOC_MAX_PARTS


def rel_l2(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(x - ref) / np.linalg.norm(ref))


def noalloc_twice_and_check(csr, O, seed=3):
    d = V.DeviceCSR(csr)
    dB = torch.empty(csr.N, O, device="cuda")
    V.gen_dense_device(dB, seed)
    ref = torch.empty(csr.M, O, device="cuda")
    V.run_csr_spmm_gpu(csr.M, d.row_ptr, d.col, d.val, dB, O, ref)
    torch.cuda.synchronize()
    ref_np = ref.cpu().numpy()
    want = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, dB.cpu().numpy())
    for _ in range(2):  # the shared scratch is reused by the second call
        C = torch.full((csr.M, O), float("nan"), device="cuda")
        V.csr_spmm_noalloc(csr.M, d.row_ptr, d.col, d.val, dB, O, C)
        torch.cuda.synchronize()
        c = C.cpu().numpy()
        assert np.isfinite(c).all()
        assert rel_l2(c, ref_np) <= TOL
        assert rel_l2(c, want) <= TOL


@pytest.mark.parametrize("cfg,size,O", [("powerlaw", 60000, 64), ("powerlaw", 60000, 512),
                                        ("powerlaw", 60000, 30), ("fem", 6000, 128),
                                        ("uniform", 0, 30)])
def test_noalloc_matches_existing_entry_point_and_oracle_twice(cfg, size, O):
    csr = V.gen_csr(cfg, 0, size)
    if cfg == "powerlaw":
        assert (np.diff(csr.row_ptr) > SPLIT).sum() >= 3  # the split path runs
    noalloc_twice_and_check(csr, O)


def test_noalloc_rejects_o_past_its_limit():
    csr = V.gen_csr("uniform", 0, 64)
    d = V.DeviceCSR(csr)
    dB = torch.zeros(csr.N, 520, device="cuda")
    C = torch.zeros(csr.M, 520, device="cuda")
    with pytest.raises(V.VcsrError) as ei:
        V.csr_spmm_noalloc(csr.M, d.row_ptr, d.col, d.val, dB, 520, C)
    assert ei.value.status == 8 and "allocation-free" in ei.value.msg


def full_rows(M, length, N):
    """M rows holding columns 0..length-1 each (values in [-1, 1])."""
    rp = (np.arange(M + 1, dtype=np.int64) * length).astype(np.int32)
    col = np.tile(np.arange(length, dtype=np.int32), M)
    val = np.random.default_rng(M).uniform(-1, 1, M * length).astype(np.float32)
    return V.CSR(M, N, M * length, rp, col, val)


@pytest.mark.parametrize("case", ["long_rows", "parts"])
def test_noalloc_device_detected_overflow_then_recovers(case):
    if case == "long_rows":  # 1,025 rows longer than 4,096 entries
        csr, needle = full_rows(MAX_LONG + 1, SPLIT + 1, SPLIT + 1), "rows longer than"
    else:  # 3 rows of 733 parts each: 2,199 parts > 2,048
        n = 733 * SPLIT
        csr, needle = full_rows(3, n, n), "parts"
    d = V.DeviceCSR(csr)
    O = 4
    dB = torch.empty(csr.N, O, device="cuda")
    V.gen_dense_device(dB, 1)
    C = torch.zeros(csr.M, O, device="cuda")
    with pytest.raises(V.VcsrError) as ei:
        V.csr_spmm_noalloc(csr.M, d.row_ptr, d.col, d.val, dB, O, C)
    assert ei.value.status == 8  # VCSR_ERR_RANGE
    assert needle in ei.value.msg and "allocation-free" in ei.value.msg
    # the refused call leaves nothing behind that the next call reads
    noalloc_twice_and_check(V.gen_csr("powerlaw", 0, 60000), 64, seed=4)
