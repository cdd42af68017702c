"""The reference's launcher on the engine: run_vcsr_spmm_gpu
(src/kernels.cu:120-167) receives the segment-major VCSRSpMM; the engine
turns its slots back into entries on the GPU (vcsr_plan_from_vcsr), lays them
out as its own plan and adds the product into C (vcsr_spmm_accumulate).

Contract checked here:
* the plan built from a VCSR equals, byte for byte in its saved form, the
  plan built from the CSR the VCSR came from (device and host VCSR input);
* C += A*B: with accumulate the result is, bit for bit, C0 + (the plain
  product) for the FP32 kernels (one FP32 add per value), within tolerance
  for the tensor-core paths (the residual and the panels add in turn);
* the product matches the oracle's CSR sum; malformed VCSRs are refused;
* a C++ caller of the reference's interface (tests/cpp/drop_in.cpp), compiled
  against include/vcsr_spmm.hpp, gets the CSR ground truth from
  run_vcsr_spmm_gpu and from the segment-major kernel.
"""
import os
import subprocess

import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import ROOT, random_csr, rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def saved(plan, path):
    plan.save(path)
    with open(path, "rb") as f:
        return f.read()


@pytest.mark.parametrize("cfg,size", [("fem", 3001), ("powerlaw", 60000), ("rmat", 16),
                                      ("blockdense", 1024), ("uniform", 0)])
def test_plan_from_vcsr_equals_plan_from_csr(tmp_path, cfg, size):
    csr = V.gen_csr(cfg, 0, size)
    d = V.DeviceCSR(csr)
    v = V.csr_to_vcsr_spmm(d, 4, 32)
    ref = saved(V.Plan(csr), str(tmp_path / "csr.plan"))
    assert saved(V.Plan.from_vcsr(v), str(tmp_path / "dev.plan")) == ref
    assert saved(V.Plan.from_vcsr(v.to_host()), str(tmp_path / "host.plan")) == ref


def test_plan_from_vcsr_segw_bundle_and_empty_rows(tmp_path):
    rp, col, val = random_csr(3, 500, 701, 0.02, dense_rows=(7,))
    lens = np.diff(rp)
    lens[100:180] = 0
    idx = np.concatenate([np.arange(rp[r], rp[r] + lens[r]) for r in range(500)])
    rp2 = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    csr = V.CSR(500, 701, len(idx), rp2, col[idx], val[idx])
    for segw, bundle in ((1, 32), (3, 8), (16, 64)):  # segw and bundle are saved too
        ref = saved(V.Plan(csr, segw=segw, bundle=bundle), str(tmp_path / "csr.plan"))
        v = V.csr_to_vcsr_spmm(V.DeviceCSR(csr), segw, bundle)
        assert saved(V.Plan.from_vcsr(v), str(tmp_path / "v.plan")) == ref, (segw, bundle)


@pytest.mark.parametrize("cfg,size,O,kw,exact", [
    ("fem", 6000, 128, {}, True),                   # R = 8 vectors
    ("powerlaw", 60000, 64, {}, True),              # split long rows
    ("rmat", 16, 256, {"max_O": 256}, True),
    ("uniform", 0, 30, {}, True),                   # scalar path (O % 4 != 0)
    ("blockdense", 1024, 128, {"tf32_panels": True}, False),
    ("fem", 3001, 64, {"tc_segments": True}, False),
    ("blockdense", 1024, 128, {"tc_segments": True}, False),
])
def test_accumulate(cfg, size, O, kw, exact):
    csr = V.gen_csr(cfg, 0, size)
    plan = V.Plan(csr, **kw)
    B = torch.from_numpy(V.gen_dense_host(csr.N, O, 5)).cuda()
    C0 = torch.from_numpy(V.gen_dense_host(csr.M, O, 6)).cuda()
    prod = torch.empty_like(C0)
    plan.spmm(B, prod)
    acc = C0.clone()
    plan.spmm(B, acc, accumulate=True)
    plan.check()
    want = (C0 + prod).cpu().numpy()
    got = acc.cpu().numpy()
    if exact:
        assert np.array_equal(got, want)
    else:
        assert rel_l2(got, want) <= (2e-3 if kw.get("tf32_panels") else 1e-5)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B.cpu().numpy())
    tol = 2e-3 if kw.get("tf32_panels") else 1e-5
    assert rel_l2(got - C0.cpu().numpy(), ref) <= tol * 10


def test_accumulate_leaves_empty_rows_and_nan():
    """Rows of A without entries keep C's values, NaN included."""
    rp = np.array([0, 2, 2, 3], np.int32)
    csr = V.CSR(3, 4, 3, rp, np.array([0, 3, 1], np.int32), np.array([1, 2, 3], np.float32))
    plan = V.Plan(csr)
    B = torch.arange(16, dtype=torch.float32, device="cuda").reshape(4, 4)
    C0 = torch.tensor([[1.0] * 4, [float("nan"), 5.0, -7.0, 0.5], [2.0] * 4], device="cuda")
    acc = C0.clone()
    plan.spmm(B, acc, accumulate=True)
    torch.cuda.synchronize()
    got = acc.cpu().numpy()
    assert np.isnan(got[1, 0]) and np.array_equal(got[1, 1:], [5.0, -7.0, 0.5])
    assert np.array_equal(got[0], 1.0 + np.array([0, 1, 2, 3]) + 2 * np.array([12, 13, 14, 15]))
    assert np.array_equal(got[2], 2.0 + 3 * np.array([4, 5, 6, 7]))


@pytest.mark.parametrize("O", [1, 8, 33, 128])
def test_run_vcsr_spmm_gpu_on_the_engine(O):
    csr = V.gen_csr("fem", 0, 3001)
    B = V.gen_dense_host(csr.N, O, 4)
    v = V.csr_to_vcsr_spmm(V.DeviceCSR(csr), 4, 32)
    dB = torch.from_numpy(B).cuda()
    dC = torch.zeros(csr.M, O, device="cuda")
    V.run_vcsr_spmm_gpu(v, dB, O, 64, dC)
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(dC.cpu().numpy(), ref) <= 1e-5
    V.run_vcsr_spmm_gpu(v, dB, O, 64, dC)  # C += A*B
    assert rel_l2(dC.cpu().numpy(), 2 * ref) <= 1e-5


def test_malformed_vcsr_refused():
    csr = V.gen_csr("fem", 0, 600)
    h = V.csr_to_vcsr_spmm(V.DeviceCSR(csr), 4, 32).to_host()

    def bad(**change):
        import dataclasses
        return dataclasses.replace(h, **change)

    gp = h.group_ptr.copy()
    gp[1] += 1
    lc = h.lcol.copy()
    lc[np.argmax(lc >= 0)] = 4  # >= segw
    gr = h.group_rows.copy()
    gr[0] = csr.M
    for v, status, words in ((bad(group_ptr=gp), 1, "group_ptr"),
                             (bad(lcol=lc), 8, "lcol"),
                             (bad(group_rows=gr), 8, "group_rows")):
        with pytest.raises(V.VcsrError) as ei:
            V.Plan.from_vcsr(v)
        assert ei.value.status == status and words in ei.value.msg


def write_mtx(path, csr):
    rows = np.repeat(np.arange(csr.M), np.diff(csr.row_ptr))
    with open(path, "w") as f:
        f.write("%%MatrixMarket matrix coordinate real general\n")
        f.write(f"{csr.M} {csr.N} {csr.nnz}\n")
        for r, c, x in zip(rows, csr.col, csr.val):
            f.write(f"{r + 1} {c + 1} {float(x):.9g}\n")


def test_cpp_caller_of_the_reference_interface(tmp_path):
    exe = str(tmp_path / "drop_in")
    lib = os.path.join(ROOT, "vcsr-spmm_b200", "lib")
    b = subprocess.run(["g++", "-O2", "-std=c++17", "-I" + os.path.join(ROOT, "include"),
                        "-I/usr/local/cuda/include", os.path.join(ROOT, "tests", "cpp", "drop_in.cpp"),
                        "-o", exe, "-L" + lib, "-lvcsr_b200", "-L/usr/local/cuda/lib64", "-lcudart",
                        "-Wl,-rpath," + lib], capture_output=True, text=True, timeout=300)
    assert b.returncode == 0, b.stderr
    mtx = str(tmp_path / "a.mtx")
    write_mtx(mtx, V.gen_csr("powerlaw", 0, 20000))
    for O in (16, 64):
        r = subprocess.run([exe, mtx, str(O)], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr
        f = r.stdout.split()
        assert f[0] == "engine" and f[2] == "twice" and f[4] == "segmented"
        assert float(f[1]) <= 1e-5 and float(f[3]) <= 1e-5 and float(f[5]) <= 1e-5, r.stdout
