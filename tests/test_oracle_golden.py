"""The CPU oracle against outputs of the reference's own code.

tests/golden/ref_outputs.npz was written by tests/golden/make_golden.py from
the reference's include/mmio.hpp, include/csr.hpp and include/vcsr.hpp
(compiled from the reference tree into oracle/_ref/).  These tests pin the
oracle (oracle/oracle.c) to it: Matrix Market parsing, COO -> CSR and the
VCSR build bit for bit (VCSR after fixing the tie order the reference's
std::sort leaves open), and the error cases.
"""
import os

import numpy as np
import pytest

import oracle
from helpers import (MTX_DIR, golden_cases, golden_errors, golden_vcsr_builds,
                     vcsr_equal_canonical, vcsr_equal_exact)


def test_fixture_inventory(golden):
    cases = golden_cases(golden)
    assert len(cases) >= 14
    errs = golden_errors(golden)
    assert set(errs) == {"bad_header", "short_data", "row_out_of_range",
                         "garbled_value"}


@pytest.mark.parametrize("fname", sorted(f for f in os.listdir(MTX_DIR)))
def test_read_mtx_matches_reference(golden, fname):
    key = fname[:-4]
    errs = golden_errors(golden)
    path = os.path.join(MTX_DIR, fname)
    if key in errs and errs[key]["stage"] == "read":
        with pytest.raises(oracle.OracleError) as ei:
            oracle.read_mtx(path)
        assert ei.value.msg == errs[key]["msg"]
        return
    M, N, r, c, v = oracle.read_mtx(path)
    assert [M, N] == list(golden[f"{key}/coo_shape"])
    assert np.array_equal(r, golden[f"{key}/coo_rows"])
    assert np.array_equal(c, golden[f"{key}/coo_cols"])
    assert np.array_equal(v.view(np.int32), golden[f"{key}/coo_vals"].view(np.int32))


def test_coo_to_csr_matches_reference(golden):
    errs = golden_errors(golden)
    n = 0
    for case in golden_cases(golden):
        if f"{case}/coo_shape" not in golden.files:
            continue
        M, N = (int(x) for x in golden[f"{case}/coo_shape"])
        args = (M, N, golden[f"{case}/coo_rows"], golden[f"{case}/coo_cols"],
                golden[f"{case}/coo_vals"])
        if case in errs and errs[case]["stage"] == "coo_to_csr":
            with pytest.raises(oracle.OracleError) as ei:
                oracle.coo_to_csr(*args)
            assert ei.value.msg == errs[case]["msg"]
            continue
        rp, cc, vv = oracle.coo_to_csr(*args)
        assert np.array_equal(rp, golden[f"{case}/csr_row_ptr"]), case
        assert np.array_equal(cc, golden[f"{case}/csr_col"]), case
        assert np.array_equal(vv, golden[f"{case}/csr_val"]), case
        n += 1
    assert n >= 14


def test_vcsr_build_matches_reference(golden):
    n_exact = n = 0
    for case in golden_cases(golden):
        if f"{case}/csr_row_ptr" not in golden.files:
            continue
        M, N = (int(x) for x in golden[f"{case}/coo_shape"])
        rp, cc, vv = (golden[f"{case}/csr_row_ptr"], golden[f"{case}/csr_col"],
                      golden[f"{case}/csr_val"])
        for segw, bundle, ref in golden_vcsr_builds(golden, case):
            mine = oracle.csr_to_vcsr(M, N, rp, cc, vv, segw, bundle)
            assert mine["num_groups"] == ref["num_groups"], (case, segw, bundle)
            assert mine["num_slots"] == ref["num_slots"], (case, segw, bundle)
            # metadata depends only on the sorted counts: exact
            for k in ("group_ptr", "group_depth", "group_seg_base"):
                assert np.array_equal(mine[k], ref[k]), (case, segw, bundle, k)
            ok, k = vcsr_equal_canonical(mine, ref)
            assert ok, (case, segw, bundle, k)
            n += 1
            n_exact += vcsr_equal_exact(mine, ref)[0]
    assert n >= 26
    assert n_exact >= 10  # cases without count ties match without canonicalising


def test_canonical_form_is_tie_invariant():
    """Shuffling equal-count rows inside a segment does not change the form."""
    from helpers import random_csr
    rp, cc, vv = random_csr(11, 40, 24, 0.2)
    v = oracle.csr_to_vcsr(40, 24, rp, cc, vv, 4, 8)
    c0 = oracle.canonical_vcsr(v)
    # swap the lanes of two rows with equal counts in the first group
    G, b = v["num_groups"], v["bundle"]
    rows = v["group_rows"].reshape(G, b).copy()
    d = v["group_depth"][0]
    lcol = v["lcol"].copy()
    val = v["val"].copy()
    cnt = [(lcol[v["group_ptr"][0] + np.arange(d) * b + ln] != -1).sum() for ln in range(b)]
    pair = next(((i, j) for i in range(b) for j in range(i + 1, b)
                 if cnt[i] == cnt[j] and rows[0, i] >= 0 and rows[0, j] >= 0), None)
    assert pair is not None
    i, j = pair
    rows[0, [i, j]] = rows[0, [j, i]]
    for dd in range(d):
        s = v["group_ptr"][0] + dd * b
        lcol[[s + i, s + j]] = lcol[[s + j, s + i]]
        val[[s + i, s + j]] = val[[s + j, s + i]]
    w = dict(v, group_rows=rows.reshape(-1), lcol=lcol, val=val)
    c1 = oracle.canonical_vcsr(w)
    for k in ("group_rows", "lcol", "val"):
        assert np.array_equal(c0[k], c1[k])


def test_csr_spmm_semantics_small():
    """oracle_csr_spmm_f32 is row-sequential FMA in CSR order."""
    from helpers import random_csr
    rp, cc, vv = random_csr(3, 30, 20, 0.3)
    B = np.random.default_rng(0).uniform(-1, 1, (20, 7)).astype(np.float32)
    C = oracle.csr_spmm_f32(30, rp, cc, vv, B)
    ref = np.zeros((30, 7), np.float32)
    for r in range(30):
        acc = np.zeros(7, np.float32)
        for p in range(rp[r], rp[r + 1]):
            # fmaf(a, b, acc): one rounding of the exact a*b + acc
            acc = (np.float64(vv[p]) * B[cc[p]].astype(np.float64) + acc).astype(np.float32)
        ref[r] = acc
    assert np.array_equal(C, ref)
    C64 = oracle.csr_spmm_f64(30, rp, cc, vv, B)
    assert np.max(np.abs(C64 - C)) < 1e-5


def test_vcsr_spmm_semantics_matches_csr():
    from helpers import random_csr, rel_l2
    rp, cc, vv = random_csr(5, 50, 37, 0.15, dup_rows=(3, 4))
    B = np.random.default_rng(1).uniform(-1, 1, (37, 9)).astype(np.float32)
    v = oracle.csr_to_vcsr(50, 37, rp, cc, vv, 4, 8)
    assert rel_l2(oracle.vcsr_spmm(v, B), oracle.csr_spmm_f64(50, rp, cc, vv, B)) < 1e-6


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built")
def test_oracle_matches_reference_on_random_matrices():
    """Fresh random cases straight through the reference's own headers."""
    from helpers import random_csr
    for seed, (M, N, dens, segw, bundle) in enumerate(
            [(70, 90, 0.05, 4, 32), (33, 17, 0.3, 3, 5), (128, 300, 0.02, 16, 32),
             (9, 9, 0.6, 2, 1)]):
        rp, cc, vv = random_csr(100 + seed, M, N, dens)
        ref = oracle.ref_csr_to_vcsr(M, N, rp, cc, vv, segw, bundle)
        mine = oracle.csr_to_vcsr(M, N, rp, cc, vv, segw, bundle)
        ok, k = vcsr_equal_canonical(mine, ref)
        assert ok, (seed, k)


def test_reference_arm_generators_match_the_library():
    """The oracle's restatement of the seeded inputs (the reference arm builds
    them without loading the engine) gives the engine generator's R-MAT matrix
    and dense B bit for bit."""
    import vcsr_b200 as V
    for scale, seed in ((10, 0), (13, 3)):
        M, rp, col, val = oracle.gen_rmat(scale, seed)
        ref = V.gen_csr("rmat", seed, scale)
        assert M == ref.M
        assert np.array_equal(rp, ref.row_ptr) and np.array_equal(col, ref.col)
        assert np.array_equal(val.view(np.int32), ref.val.view(np.int32))
    for rows, cols, seed, lo in ((1000, 37, 1000, -1.0), (513, 256, 7, 0.0)):
        assert np.array_equal(oracle.gen_dense(rows, cols, seed, lo, 1.0).view(np.int32),
                              V.gen_dense_host(rows, cols, seed, lo, 1.0).view(np.int32))
