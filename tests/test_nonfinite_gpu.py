"""Non-finite B values on padded vector panels, against the oracle's CSR sum.

A vector of R > 1 rows multiplies every row's value, padding zeros included,
by each union column's B row.  0 * Inf and 0 * NaN are NaN, so without care a
row would turn NaN where the reference's CSR sum (src/kernels.cu:27-31) never
reads that B row.  The kernels recompute such rows over their own entries.

Contract checked here: the NaN, +Inf and -Inf pattern of C equals the
oracle's (oracle_csr_spmm_f32) element for element, and the finite entries
are within relative L2 1e-5; rows summed in CSR order are bit-exact.  Each
case also checks that a plain padded sum would have been wrong somewhere, so
the recomputation really runs.
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
scipy_sparse = pytest.importorskip("scipy.sparse")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def poison(B, seed, ncols=40):
    """Inf, -Inf and NaN at random positions of `ncols` random B rows."""
    rng = np.random.default_rng(seed)
    B = B.copy()
    rows = rng.choice(B.shape[0], size=min(ncols, B.shape[0]), replace=False)
    for c in rows:
        ks = rng.choice(B.shape[1], size=max(1, B.shape[1] // 8), replace=False)
        B[c, ks] = rng.choice(np.array([np.inf, -np.inf, np.nan], np.float32), size=len(ks))
    return B


def padded_would_be_wrong(csr, B, R, ref):
    """Entries a padded sum gets wrong: some row of the vector reads a
    non-finite B value there, while the row's own CSR sum is not NaN."""
    A = scipy_sparse.csr_matrix((np.ones(csr.nnz), csr.col, csr.row_ptr), shape=(csr.M, csr.N))
    bad = (A @ (~np.isfinite(B)).astype(np.float64)) > 0  # row reads a non-finite value
    V_ = -(-csr.M // R)
    pad = np.zeros((V_ * R, B.shape[1]), bool)
    pad[: csr.M] = bad
    vec = pad.reshape(V_, R, -1).any(axis=1)
    naive = np.repeat(vec, R, axis=0)[: csr.M]
    return int((naive & ~np.isnan(ref)).sum())


def check(C, ref):
    assert np.array_equal(np.isnan(C), np.isnan(ref)), "NaN pattern differs"
    assert np.array_equal(np.isposinf(C), np.isposinf(ref)), "+Inf pattern differs"
    assert np.array_equal(np.isneginf(C), np.isneginf(ref)), "-Inf pattern differs"
    fin = np.isfinite(ref)
    assert rel_l2(C[fin], ref[fin]) <= TOL


def run(csr, B, **kw):
    plan = V.Plan(csr, **kw)
    dB = torch.from_numpy(np.ascontiguousarray(B)).cuda()
    dC = torch.full((csr.M, B.shape[1]), 7.0, device="cuda")
    plan.spmm(dB, dC)
    torch.cuda.synchronize()
    return plan, dC.cpu().numpy()


@pytest.mark.parametrize("cfg,size,O,kw", [
    ("fem", 6000, 128, {}),                       # default R = 8, short units
    ("fem", 6000, 32, {}),                        # 8-lane sub-warps
    ("fem", 6000, 512, {"target_O": 512}),        # R = 4, two columns per lane
    ("fem", 6000, 64, {"vec_rows": 2}),           # R = 2: batches of vectors
    ("fem", 3001, 64, {"vec_rows": 16}),
    ("fem", 3001, 30, {"vec_rows": 4}),           # scalar lanes (O % 4 != 0)
    ("blockdense", 2048, 512, {}),                # long units (>= 128 columns)
    ("blockdense", 2048, 128, {"chunk": 256}),    # split vectors, last-part sums
    ("blockdense", 1024, 100, {"vec_rows": 8, "chunk": 128}),
])
def test_nonfinite_b_matches_csr(cfg, size, O, kw):
    csr = V.gen_csr(cfg, 0, size)
    B = poison(V.gen_dense_host(csr.N, O, 21), 5)
    plan, C = run(csr, B, max_O=512, **kw)
    R = plan.info()["vec_rows"]
    assert R > 1
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert padded_would_be_wrong(csr, B, R, ref) > 0
    check(C, ref)
    info = plan.info()
    if info["num_split_units"] == 0 and info["num_long_units"] == 0:
        fin = np.isfinite(ref)
        a, b = C[fin] + 0.0, ref[fin] + 0.0  # +0.0 maps -0 to +0
        assert np.array_equal(a.view(np.int32), b.view(np.int32))


def test_explicit_zero_times_inf_is_nan_like_csr():
    """A stored 0.0 entry times Inf is NaN in the CSR sum too; a padding zero
    is not an entry and must not be."""
    csr = V.gen_csr("fem", 0, 3000)
    val = csr.val.copy()
    val[::97] = 0.0  # explicit zeros
    csr = V.CSR(csr.M, csr.N, csr.nnz, csr.row_ptr, csr.col, val)
    B = V.gen_dense_host(csr.N, 64, 4)
    hit = np.unique(csr.col[::97])[:25]
    B[hit, :8] = np.inf
    plan, C = run(csr, B)
    assert plan.info()["vec_rows"] > 1
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert np.isnan(ref).any()
    check(C, ref)


def test_nonfinite_bf16_b():
    """The 16-bit path: the same recomputation on B widened as it is loaded."""
    csr = V.gen_csr("fem", 0, 4000)
    B = poison(V.gen_dense_host(csr.N, 128, 9), 3)
    Bt = torch.from_numpy(B).cuda().to(torch.bfloat16)
    plan = V.Plan(csr)
    dC = torch.empty(csr.M, 128, device="cuda")
    plan.spmm(Bt, dC)
    torch.cuda.synchronize()
    Bw = Bt.float().cpu().numpy()
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, Bw)
    assert padded_would_be_wrong(csr, Bw, plan.info()["vec_rows"], ref) > 0
    check(dC.cpu().numpy(), ref)


def test_nonfinite_after_save_and_load(tmp_path):
    """The row masks travel with a saved plan."""
    csr = V.gen_csr("fem", 0, 3000)
    B = poison(V.gen_dense_host(csr.N, 128, 8), 2)
    plan = V.Plan(csr)
    path = str(tmp_path / "p.plan")
    plan.save(path)
    loaded = V.Plan.load(path)
    dB = torch.from_numpy(B).cuda()
    dC = torch.empty(csr.M, 128, device="cuda")
    loaded.spmm(dB, dC)
    torch.cuda.synchronize()
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    check(dC.cpu().numpy(), ref)
