"""vcsr_spmm_bf16 / vcsr_spmm_f16: B in bfloat16 or float16, widened to FP32
as it is loaded, FP32 sums.  Widening is exact, so C must equal, bit for bit,
the FP32 path run on the widened B (same kernels, same summation order), and
match the FP64 CSR sum of the widened B within the FP32 tolerance."""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL = 1e-5


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("cfg,size,R", [("fem", 4000, 0), ("fem", 4000, 2), ("powerlaw", 30000, 0),
                                        ("uniform", 0, 0), ("rmat", 14, 0), ("fem", 3000, 16)])
@pytest.mark.parametrize("O", [1, 3, 32, 100, 128, 256])
def test_16bit_equals_fp32_on_widened_b(cfg, size, R, O, dtype):
    csr = V.gen_csr(cfg, 4, size)
    plan = V.Plan(csr, vec_rows=R, max_O=512)
    g = torch.Generator().manual_seed(O)
    Bh = (torch.rand(csr.N, O, generator=g) * 2 - 1).to(getattr(torch, dtype))
    Bb = Bh.cuda()
    Bf = Bb.float()
    C1 = torch.full((csr.M, O), float("nan"), device="cuda")
    C2 = torch.full((csr.M, O), float("nan"), device="cuda")
    plan.spmm(Bb, C1)
    plan.spmm(Bf, C2)
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)
    if csr.M <= 40000:
        ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, Bf.cpu().numpy())
        assert rel_l2(C1.cpu().numpy(), ref) <= TOL


def test_f16_special_values_widen_exactly():
    # subnormal and largest finite FP16 values go through the conversion
    # unchanged: a one-entry-per-row identity A copies B to C.  Each sum starts
    # at +0, so a -0 in B gives +0 in C, as on the FP32 path.
    n, O = 64, 8
    rp = np.arange(n + 1, dtype=np.int32)
    csr = V.CSR(n, n, n, rp, np.arange(n, dtype=np.int32), np.ones(n, dtype=np.float32))
    plan = V.Plan(csr)
    vals = torch.tensor([6.0e-8, -6.0e-8, 65504.0, -65504.0, 0.0, -0.0, 1.0e-5, 3.140625],
                        dtype=torch.float16)
    Bh = vals.repeat(n, 1)
    C1 = torch.full((n, O), float("nan"), device="cuda")
    plan.spmm(Bh.cuda(), C1)
    torch.cuda.synchronize()
    assert torch.equal(C1.cpu(), Bh.float())
    assert not torch.signbit(C1.cpu()[:, 5]).any()


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_16bit_padded_ld_and_errors(dtype):
    csr = V.gen_csr("fem", 1, 2000)
    plan = V.Plan(csr)
    O, ldb, ldc = 60, 72, 68
    Bfull = (torch.randn(csr.N, ldb, device="cuda")).to(getattr(torch, dtype))
    Cfull = torch.zeros(csr.M, ldc, device="cuda")
    C2 = torch.zeros(csr.M, ldc, device="cuda")
    plan.spmm(Bfull, Cfull, O=O, ldb=ldb, ldc=ldc)
    plan.spmm(Bfull.float().contiguous(), C2, O=O, ldb=ldb, ldc=ldc)
    torch.cuda.synchronize()
    assert torch.equal(Cfull[:, :O], C2[:, :O])
    tplan = V.Plan(V.gen_csr("blockdense", 0, 1024), tf32_panels=True)
    Bb = torch.zeros(1024, 64, device="cuda", dtype=getattr(torch, dtype))
    with pytest.raises(V.VcsrError) as ei:
        tplan.spmm(Bb, torch.zeros(1024, 64, device="cuda"))
    assert ei.value.status == 5
