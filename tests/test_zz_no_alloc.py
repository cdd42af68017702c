"""The allocation-free CSR SpMM entry point (vcsr_csr_spmm_noalloc).

It serves callers that may not allocate device memory, for instance a solver
inside an application whose framework has already handed all free device
memory to its own pool.  Its scratch for split long rows is one fixed array
compiled into the library, so this file checks, through the C ABI, that two
calls in a row give the same C as the ordinary entry point (vcsr_csr_spmm)
within the engine's tolerance, on a matrix whose long rows are split, and that
sizes past the fixed limits are refused with an error.  It is collected last
and needs no state from other tests.
"""
import numpy as np
import pytest

import vcsr_b200 as V

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


def rel_l2(x, ref):
    x = x.double()
    ref = ref.double()
    return (torch.linalg.norm(x - ref) / torch.linalg.norm(ref)).item()


@pytest.mark.parametrize("cfg,size,O", [("powerlaw", 60000, 64), ("fem", 6000, 128),
                                        ("uniform", 0, 30)])
def test_noalloc_matches_existing_entry_point_twice(cfg, size, O):
    csr = V.gen_csr(cfg, 0, size)
    lens = np.diff(csr.row_ptr)
    d = V.DeviceCSR(csr)
    dB = torch.empty(csr.N, O, device="cuda")
    V.gen_dense_device(dB, 3)
    ref = torch.empty(csr.M, O, device="cuda")
    V.run_csr_spmm_gpu(csr.M, d.row_ptr, d.col, d.val, dB, O, ref)
    torch.cuda.synchronize()
    if cfg == "powerlaw":
        assert (lens > 4096).sum() >= 3  # the split path runs
    for _ in range(2):  # the shared scratch is reused by the second call
        C = torch.full((csr.M, O), float("nan"), device="cuda")
        V.csr_spmm_noalloc(csr.M, d.row_ptr, d.col, d.val, dB, O, C)
        torch.cuda.synchronize()
        assert torch.isfinite(C).all()
        assert rel_l2(C, ref) <= TOL


def test_noalloc_rejects_sizes_past_its_limit():
    csr = V.gen_csr("uniform", 0, 64)
    d = V.DeviceCSR(csr)
    dB = torch.zeros(csr.N, 520, device="cuda")
    C = torch.zeros(csr.M, 520, device="cuda")
    with pytest.raises(V.VcsrError) as ei:
        V.csr_spmm_noalloc(csr.M, d.row_ptr, d.col, d.val, dB, 520, C)
    assert ei.value.status == 8 and "allocation-free" in ei.value.msg
