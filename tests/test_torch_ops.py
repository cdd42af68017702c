"""torch.ops.vcsr.spmm: the PyTorch operator over a plan.  The fake
(shape-only) implementation is checked on the CPU with a stand-in object; the
product itself on the GPU against Plan.spmm."""
from types import SimpleNamespace

import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
from vcsr_b200 import torch_ops  # noqa: E402


def test_op_is_registered_and_fake_shapes():
    assert hasattr(torch.ops.vcsr, "spmm")
    from torch._subclasses.fake_tensor import FakeTensorMode
    pid = torch_ops.register(SimpleNamespace(M=7, N=5))
    try:
        with FakeTensorMode():
            B = torch.empty(5, 12)
            C = torch.ops.vcsr.spmm(pid, B)
            assert tuple(C.shape) == (7, 12) and C.dtype == torch.float32
    finally:
        torch_ops.unregister(pid)
    with pytest.raises(ValueError):
        torch_ops._plan(pid)


@pytest.mark.gpu
def test_op_matches_plan():
    csr = V.gen_csr("fem", 0, 3000)
    plan = V.Plan(csr)
    pid = torch_ops.register(plan)
    try:
        B = torch.randn(csr.N, 64, device="cuda")
        C = torch.ops.vcsr.spmm(pid, B)
        C2 = torch.empty_like(C)
        plan.spmm(B, C2)
        torch.cuda.synchronize()
        assert torch.equal(C, C2)
        ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B.cpu().numpy())
        assert rel_l2(C.cpu().numpy(), ref) <= 1e-5  # the oracle's CSR sum
        Cb = torch.ops.vcsr.spmm(pid, B.to(torch.bfloat16))
        plan.spmm(B.to(torch.bfloat16).float(), C2)
        torch.cuda.synchronize()
        assert torch.equal(Cb, C2)
        Cs = torch.ops.vcsr.spmm(pid, B.t().contiguous().t())  # column-major B is copied
        assert torch.equal(Cs, C)
        with pytest.raises(ValueError):
            torch.ops.vcsr.spmm(pid, torch.randn(csr.N + 1, 8, device="cuda"))
    finally:
        torch_ops.unregister(pid)
