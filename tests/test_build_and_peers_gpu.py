"""GPU VCSR construction (vcsr_build_vcsr) bit for bit against the oracle's
canonical build and the reference's own golden builds; the peer paths
(segment-major SpMM, CSR row-wise SpMM, cuSPARSE) against the oracle; and the
oracle's CSR semantics pinned to the reference's csr_spmm_kernel rebuilt for
sm_100a (oracle/_ref)."""
import ctypes as C

import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import (golden_cases, golden_vcsr_builds, random_csr, rel_l2,
                     vcsr_equal_canonical, vcsr_equal_exact)

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def gpu_build(csr, segw, bundle):
    d = V.DeviceCSR(csr)
    v = V.csr_to_vcsr_spmm(d, segw, bundle)
    h = v.to_host()
    v.close()
    return h.as_dict()


def check_against_oracle(csr, segw, bundle):
    mine = gpu_build(csr, segw, bundle)
    ref = oracle.csr_to_vcsr(csr.M, csr.N, csr.row_ptr, csr.col, csr.val, segw, bundle)
    assert mine["num_groups"] == ref["num_groups"]
    assert mine["num_slots"] == ref["num_slots"]
    ok, k = vcsr_equal_exact(mine, ref)  # canonical tie order on both sides
    assert ok, k
    assert np.array_equal(mine["segment_group_start"], ref["segment_group_start"])
    return mine


def test_builder_matches_reference_golden(golden):
    n = 0
    for case in golden_cases(golden):
        if f"{case}/csr_row_ptr" not in golden.files:
            continue
        M, N = (int(x) for x in golden[f"{case}/coo_shape"])
        csr = V.CSR(M, N, len(golden[f"{case}/csr_val"]), golden[f"{case}/csr_row_ptr"],
                    golden[f"{case}/csr_col"], golden[f"{case}/csr_val"])
        for segw, bundle, ref in golden_vcsr_builds(golden, case):
            mine = check_against_oracle(csr, segw, bundle)
            ok, k = vcsr_equal_canonical(mine, ref)
            assert ok, (case, segw, bundle, k)
            n += 1
    assert n >= 26


@pytest.mark.parametrize("cfg,size,segw,bundle", [
    ("uniform", 0, 4, 32), ("uniform", 0, 16, 32), ("fem", 6000, 4, 32),
    ("fem", 3001, 3, 7), ("powerlaw", 50000, 4, 32), ("rmat", 14, 4, 32),
    ("blockdense", 1024, 16, 16), ("blockdense", 1024, 4, 64)])
def test_builder_configs(cfg, size, segw, bundle):
    csr = V.gen_csr(cfg, 0, size)
    check_against_oracle(csr, segw, bundle)


def test_builder_edge_cases():
    for seed, (M, N, dens, segw, bundle, extra) in enumerate([
            (33, 40, 0.1, 4, 8, {}), (100, 103, 0.05, 4, 32, {}),
            (50, 200, 0.02, 8, 16, {"dense_rows": (7,)}),
            (20, 30, 0.15, 4, 4, {"dup_rows": (1, 5, 9)}),
            (300, 5, 0.9, 1, 1, {}), (5, 5, 0.0, 4, 32, {}),
            (2000, 64, 0.3, 4, 3, {})]):
        rp, cc, vv = random_csr(50 + seed, M, N, dens, **extra)
        check_against_oracle(V.CSR(M, N, len(vv), rp, cc, vv), segw, bundle)


def test_builder_rejects_bad_input():
    rp = np.array([0, 2], np.int32)
    bad_sorted = V.CSR(1, 4, 2, rp, np.array([3, 1], np.int32), np.ones(2, np.float32))
    with pytest.raises(V.VcsrError) as ei:
        V.csr_to_vcsr_spmm(V.DeviceCSR(bad_sorted), 4, 32)
    assert ei.value.status == 1
    bad_col = V.CSR(1, 4, 2, rp, np.array([1, 9], np.int32), np.ones(2, np.float32))
    with pytest.raises(V.VcsrError) as ei:
        V.csr_to_vcsr_spmm(V.DeviceCSR(bad_col), 4, 32)
    assert ei.value.status == 8


def test_plan_export_is_reference_format():
    csr = V.gen_csr("fem", 0, 3000)
    plan = V.Plan(csr, segw=4, bundle=32, reference_format=True)
    h = plan.export().as_dict()
    ref = oracle.csr_to_vcsr(csr.M, csr.N, csr.row_ptr, csr.col, csr.val, 4, 32)
    assert vcsr_equal_exact(h, ref)[0]
    assert plan.info()["has_reference_format"] == 1


@pytest.mark.parametrize("O", [1, 8, 33, 128])
@pytest.mark.parametrize("launch", ["run_vcsr_spmm_gpu", "run_vcsr_spmm_segmented_gpu"])
def test_segmented_spmm_drop_in(O, launch):
    """run_vcsr_spmm_gpu semantics, C += A*B, for the launcher on the engine
    and for the segment-major kernel on the format itself."""
    csr = V.gen_csr("fem", 0, 3001)  # N % segw != 0: the last segment is ragged
    B = V.gen_dense_host(csr.N, O, 4)
    d = V.DeviceCSR(csr)
    v = V.csr_to_vcsr_spmm(d, 4, 32)
    dB = torch.from_numpy(B).cuda()
    dC = torch.zeros(csr.M, O, device="cuda")
    run = getattr(V, launch)
    run(v, dB, O, 64, dC)
    torch.cuda.synchronize()
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(dC.cpu().numpy(), ref) <= 1e-5
    h = v.to_host().as_dict()
    seq = oracle.vcsr_spmm(h, B)  # the reference kernel's update, sequential
    assert rel_l2(dC.cpu().numpy(), seq) <= 1e-5
    # accumulate semantics: a second call doubles C
    run(v, dB, O, 64, dC)
    torch.cuda.synchronize()
    assert rel_l2(dC.cpu().numpy(), 2 * ref) <= 1e-5


@pytest.mark.parametrize("O", [1, 7, 32, 128])
def test_csr_rowwise_bitwise(O):
    csr = V.gen_csr("powerlaw", 0, 20000)
    B = V.gen_dense_host(csr.N, O, 8)
    d = V.DeviceCSR(csr)
    dB = torch.from_numpy(B).cuda()
    dC = torch.full((csr.M, O), float("nan"), device="cuda")
    V.run_csr_spmm_gpu(csr.M, d.row_ptr, d.col, d.val, dB, O, dC)
    torch.cuda.synchronize()
    ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
    got = dC.cpu().numpy() + 0.0
    assert np.array_equal(got.view(np.int32), (ref + 0.0).view(np.int32))


@pytest.mark.parametrize("alg", [0, 1, 2, 3])
def test_cusparse_harness(alg):
    csr = V.gen_csr("fem", 0, 6000)
    B = V.gen_dense_host(csr.N, 64, 3)
    d = V.DeviceCSR(csr)
    dB = torch.from_numpy(B).cuda()
    dC = torch.zeros(csr.M, 64, device="cuda")
    try:
        h = V.CuSparse(d, dB, 64, dC, alg=alg)
    except V.VcsrError as e:
        pytest.skip(f"cuSPARSE alg {alg} unavailable: {e}")
    h.run()
    torch.cuda.synchronize()
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(dC.cpu().numpy(), ref) <= 1e-5
    h.close()


@pytest.mark.skipif(not oracle.ref_kernels_available(),
                    reason="oracle/_ref/libvcsr_ref_kernels.so not built")
def test_oracle_pinned_to_reference_csr_kernel():
    """The reference's own csr_spmm_kernel (src/kernels.cu:15-33), rebuilt for
    sm_100a, gives the oracle's FP32 result bit for bit."""
    L = oracle.ref_kernels_lib()
    for cfg, size, O in [("uniform", 0, 32), ("fem", 3000, 16), ("powerlaw", 20000, 8)]:
        csr = V.gen_csr(cfg, 0, size)
        B = V.gen_dense_host(csr.N, O, 21)
        d = V.DeviceCSR(csr)
        dB = torch.from_numpy(B).cuda()
        dC = torch.zeros(csr.M, O, device="cuda")
        ms = C.c_float()
        st = torch.cuda.current_stream().cuda_stream
        rc = L.ref_gpu_csr_spmm(csr.M, d.row_ptr.data_ptr(), d.col.data_ptr(),
                                d.val.data_ptr(), dB.data_ptr(), O, dC.data_ptr(),
                                st, C.byref(ms))
        torch.cuda.synchronize()
        assert rc == 0
        ref = oracle.csr_spmm_f32(csr.M, csr.row_ptr, csr.col, csr.val, B)
        got = dC.cpu().numpy() + 0.0
        assert np.array_equal(got.view(np.int32), (ref + 0.0).view(np.int32)), cfg


def test_multi_gpu_row_panels():
    """vcsr_mgpu_*: nnz-balanced row panels, B by NCCL broadcast, C panels
    gathered; runs on every visible GPU (one on a single-GPU box)."""
    n = min(torch.cuda.device_count(), 8)
    csr = V.gen_csr("powerlaw", 0, 60000)
    B = V.gen_dense_host(csr.N, 64, 13)
    mg = V.MultiGPU(csr, n, bundle=32)
    cuts = mg.cuts()
    assert cuts[0] == 0 and cuts[-1] == csr.M and len(cuts) == n + 1
    bms = mg.set_b(B)
    assert bms >= 0
    ms = mg.spmm()
    assert ms > 0
    C = mg.gather_c()
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B)
    assert rel_l2(C, ref) <= 1e-5
    mg.close()


def test_cli_drop_in(tmp_path):
    """spmm_vcsr with the reference's flags prints the table and the
    'Name: <ms> ms <gflops> GFLOP/s [..]' lines the reference scripts parse."""
    import os
    import subprocess
    from helpers import ROOT
    exe = os.path.join(ROOT, "vcsr-spmm_b200", "bin", "spmm_vcsr")
    mtx = os.path.join(ROOT, "tests", "golden", "mtx", "empty_rows.mtx")
    out = subprocess.run([exe, "--mtx", mtx, "--O", "8", "--segw", "4", "--bundle", "32",
                          "--tileK", "64", "--repeat", "3", "--algo", "all", "--check"],
                         capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.strip().splitlines()
    assert any(l.startswith("Matrix: 8 x 10, nnz=7") for l in lines)
    tail = lines[-1].split()
    assert "ms" in tail and "GFLOP/s" in tail
    rel = [float(l.split("=")[-1]) for l in lines if "rel_l2" in l]
    assert rel and max(rel) < 1e-5
    g = subprocess.run([exe, "--gen", "fem", "--size", "3000", "--O", "32", "--algo", "vcsr",
                        "--repeat", "2"], capture_output=True, text=True, timeout=120)
    assert g.returncode == 0 and "VCSR:" in g.stdout.splitlines()[-1]
    # aspt names the engine kernels it runs; vcsr_tcseg runs the segment path;
    # fast runs the engine's 16-row condensed windows
    for algo, tag, what in (("aspt", "ASPT:", "1 row/vector"),
                            ("vcsr_tcseg", "VCSR_TCSEG:", "split-TF32"),
                            ("fast", "FAST:", "vec_rows=16")):
        g = subprocess.run([exe, "--gen", "fem", "--size", "3000", "--O", "64", "--algo", algo,
                            "--repeat", "2", "--check"], capture_output=True, text=True,
                           timeout=120)
        assert g.returncode == 0, g.stderr
        assert tag in g.stdout.splitlines()[-1] and what in g.stdout
    bad = subprocess.run([exe, "--mtx", "/nonexistent.mtx", "--O", "8"], capture_output=True,
                         text=True, timeout=60)
    assert bad.returncode != 0 and "Failed to open MTX" in bad.stderr
