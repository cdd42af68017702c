"""The tensor-core panel kernel's bounded waits, made to run out on purpose.

vcsr_plan_test_withhold_signal makes the next TF32 panel launch withhold one
barrier signal (block 0's first accumulator-ready signal); that block's
epilogue wait gives up after a short bounded poll, the block stops its other
roles, waits for the copies and MMAs it issued, frees its tensor memory and
records the site.  Nothing faults or hangs: vcsr_plan_check reports
VCSR_ERR_TIMEOUT naming the barrier and block, and the next call on the same
plan (and on a fresh one) is correct again.
"""
import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TF32_TOL = 2e-3


def product(plan, csr, O, seed):
    dB = torch.empty(csr.N, O, device="cuda")
    V.gen_dense_device(dB, seed)
    dC = torch.empty(csr.M, O, device="cuda")
    plan.spmm(dB, dC)
    return dB, dC


def test_withheld_signal_times_out_then_recovers():
    csr = V.gen_csr("blockdense", 0, 2048)
    plan = V.Plan(csr, tf32_panels=True)
    assert plan.info()["num_panel_blocks"] > 0
    O = 128
    product(plan, csr, O, 1)
    plan.check()  # a normal call: no failure recorded

    plan.test_withhold_signal()
    product(plan, csr, O, 2)
    with pytest.raises(V.VcsrError) as ei:
        plan.check()
    assert ei.value.status == 7  # VCSR_ERR_TIMEOUT
    assert "accumulator-full" in ei.value.msg and "block 0" in ei.value.msg

    # the record is cleared and the hook was one-shot: the same plan is right again
    dB, dC = product(plan, csr, O, 3)
    plan.check()
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, dB.cpu().numpy())
    assert rel_l2(dC.cpu().numpy(), ref) <= TF32_TOL
    # and so is a fresh plan in the same context
    fresh = V.Plan(csr, tf32_panels=True)
    dB, dC = product(fresh, csr, O, 4)
    fresh.check()
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, dB.cpu().numpy())
    assert rel_l2(dC.cpu().numpy(), ref) <= TF32_TOL


def test_withhold_needs_tf32_panels():
    plan = V.Plan(V.gen_csr("fem", 0, 600))
    with pytest.raises(V.VcsrError) as ei:
        plan.test_withhold_signal()
    assert ei.value.status == 5
