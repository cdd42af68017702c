"""vcsr_read_mtx_ex: the Matrix Market reader that follows the banner (the
reference's reader ignores it).  Checked against scipy.io.mmread, an
independent implementation of the format, and against vcsr_read_mtx where the
two must agree.  Host code only (no GPU)."""
import os

import numpy as np
import pytest
import scipy.io

import vcsr_b200 as V


def write(tmp_path, name, text):
    p = os.path.join(tmp_path, name)
    with open(p, "w") as f:
        f.write(text)
    return p


def dense_of(coo, complex_real=False):
    A = np.zeros((coo.M, coo.N), np.float64)
    np.add.at(A, (coo.rows, coo.cols), coo.vals.astype(np.float64))
    return A


def scipy_dense(path):
    m = scipy.io.mmread(path)
    A = m.toarray() if hasattr(m, "toarray") else np.asarray(m)
    return np.real(A).astype(np.float64)


def test_general_real_matches_reference_reader(tmp_path):
    p = write(tmp_path, "g.mtx", "%%MatrixMarket matrix coordinate real general\n"
              "% comment\n\n4 5 4\n1 1 1.5\n2 3 -2e-1\n\n4 5 3\n3 2 +7\n")
    a = V.read_matrix_market_coo(p, banner=True)
    b = V.read_matrix_market_coo(p)
    assert (a.M, a.N, len(a.vals)) == (4, 5, 4)
    for x, y in ((a.rows, b.rows), (a.cols, b.cols), (a.vals, b.vals)):
        assert np.array_equal(x, y)
    assert np.array_equal(a.vals, np.array([1.5, -0.2, 3.0, 7.0], np.float32))


def test_comment_lines_inside_data(tmp_path):
    """The banner reader also skips '%' lines between entries (some writers
    emit them; scipy's reader does not take them); the reference's reader
    reads them as tokens and fails."""
    p = write(tmp_path, "c.mtx", "%%MatrixMarket matrix coordinate real general\n"
              "2 2 2\n1 1 1\n% between entries\n2 2 2\n")
    a = V.read_matrix_market_coo(p, banner=True)
    assert len(a.vals) == 2 and np.allclose(dense_of(a), np.diag([1.0, 2.0]))
    with pytest.raises(V.VcsrError):
        V.read_matrix_market_coo(p)


def test_symmetric_expansion_and_order(tmp_path):
    p = write(tmp_path, "s.mtx", "%%MatrixMarket matrix coordinate real symmetric\n"
              "3 3 4\n1 1 2.0\n2 1 -1.0\n3 2 4.5\n3 3 1.0\n")
    a = V.read_matrix_market_coo(p, banner=True)
    assert len(a.vals) == 6  # two off-diagonal entries mirrored
    assert list(zip(a.rows, a.cols)) == [(0, 0), (1, 0), (0, 1), (2, 1), (1, 2), (2, 2)]
    assert np.allclose(dense_of(a), scipy_dense(p))


def test_pattern_skew_hermitian(tmp_path):
    p = write(tmp_path, "p.mtx", "%%MatrixMarket matrix coordinate pattern general\n"
              "3 4 3\n1 4\n2 2\n3 1\n")
    a = V.read_matrix_market_coo(p, banner=True)
    assert np.all(a.vals == 1.0) and np.allclose(dense_of(a), scipy_dense(p))
    p = write(tmp_path, "k.mtx", "%%MatrixMarket matrix coordinate integer skew-symmetric\n"
              "3 3 2\n2 1 5\n3 1 -2\n")
    a = V.read_matrix_market_coo(p, banner=True)
    assert len(a.vals) == 4 and np.allclose(dense_of(a), scipy_dense(p))
    p = write(tmp_path, "h.mtx", "%%MatrixMarket matrix coordinate complex hermitian\n"
              "2 2 2\n1 1 3.0 0.0\n2 1 1.5 -2.0\n")
    a = V.read_matrix_market_coo(p, banner=True)
    assert len(a.vals) == 3 and np.allclose(dense_of(a), scipy_dense(p))


def test_large_symmetric_parallel_parse(tmp_path):
    """Enough entries for several parsing threads; compared entry by entry."""
    rng = np.random.default_rng(3)
    n, z = 5000, 300_000
    r = rng.integers(0, n, z)
    c = rng.integers(0, n, z)
    lo, hi = np.minimum(r, c), np.maximum(r, c)  # lower triangle
    v = rng.uniform(-1, 1, z).round(6)
    lines = "".join(f"{h + 1} {l + 1} {x:.6f}\n" for h, l, x in zip(hi, lo, v))
    p = write(tmp_path, "big.mtx", "%%MatrixMarket matrix coordinate real symmetric\n"
              f"{n} {n} {z}\n" + lines)
    a = V.read_matrix_market_coo(p, banner=True)
    off = hi != lo
    assert len(a.vals) == z + int(off.sum())
    exp_r = np.empty(len(a.vals), np.int64)
    exp_c = np.empty(len(a.vals), np.int64)
    exp_v = np.empty(len(a.vals), np.float32)
    pos = np.arange(z) + np.concatenate([[0], np.cumsum(off)[:-1]])  # slot of entry i
    exp_r[pos], exp_c[pos], exp_v[pos] = hi, lo, v.astype(np.float32)
    mpos = pos[off] + 1
    exp_r[mpos], exp_c[mpos], exp_v[mpos] = lo[off], hi[off], v[off].astype(np.float32)
    assert np.array_equal(a.rows, exp_r) and np.array_equal(a.cols, exp_c)
    assert np.array_equal(a.vals, exp_v)
    m = scipy.io.mmread(p)
    m = m.tocoo() if hasattr(m, "tocoo") else m
    key = lambda rr, cc: np.lexsort((cc, rr))
    k1, k2 = key(a.rows, a.cols), key(m.row, m.col)
    assert np.array_equal(a.rows[k1], m.row[k2]) and np.array_equal(a.cols[k1], m.col[k2])
    assert np.allclose(np.sort(a.vals[k1]), np.sort(m.data[k2].astype(np.float32)))


@pytest.mark.parametrize("text,status", [
    ("%%MatrixMarket matrix array real general\n2 2\n1\n2\n3\n4\n", 5),
    ("%%MatrixMarket matrix coordinate real unknown\n1 1 1\n1 1 1\n", 5),
    ("%%MatrixMarket vector coordinate real general\n1 1 1\n1 1 1\n", 5),
    ("1 1 1\n1 1 1\n", 4),                                               # no banner
    ("%%MatrixMarket matrix coordinate real general\n2 2 2\n1 1 1\n", 4),  # short
    ("%%MatrixMarket matrix coordinate real general\n2 2 1\n3 1 1\n", 4),  # out of range
    ("%%MatrixMarket matrix coordinate real general\n2 2 1\n1 x 1\n", 4),  # garbled
    ("%%MatrixMarket matrix coordinate real symmetric\n2 3 1\n1 1 1\n", 4),  # not square
])
def test_errors(tmp_path, text, status):
    p = write(tmp_path, "bad.mtx", text)
    with pytest.raises(V.VcsrError) as ei:
        V.read_matrix_market_coo(p, banner=True)
    assert ei.value.status == status


@pytest.mark.gpu
def test_cli_mtx_banner(tmp_path):
    """spmm_vcsr --mtx-banner expands a symmetric file before the run."""
    import subprocess
    from helpers import ROOT
    p = write(tmp_path, "s.mtx", "%%MatrixMarket matrix coordinate real symmetric\n"
              "3 3 3\n1 1 2\n2 1 1\n3 3 1\n")
    exe = os.path.join(ROOT, "vcsr-spmm_b200", "bin", "spmm_vcsr")
    out = subprocess.run([exe, "--mtx", p, "--O", "8", "--mtx-banner", "--algo", "vcsr",
                          "--repeat", "2"], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert any(l.startswith("Matrix: 3 x 3, nnz=4") for l in out.stdout.splitlines())
