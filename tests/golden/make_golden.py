"""Record golden outputs of the reference's own host code.

Runs the reference's include/mmio.hpp (read_matrix_market_coo),
include/csr.hpp (coo_to_csr) and include/vcsr.hpp (csr_to_vcsr_spmm), built
from the reference tree into oracle/_ref/libvcsr_ref.so by oracle/Makefile, on
  * the Matrix Market files under tests/golden/mtx/ (edge cases: 0/1-based,
    tokens split across lines, empty rows, no entries, error cases), and
  * small seeded random CSR matrices (ragged shapes, N % segw != 0,
    M % bundle != 0, duplicates, a dense row, the empty matrix),
and writes them to tests/golden/ref_outputs.npz.  The VCSR arrays are stored
as the reference produced them; tests compare after oracle.canonical_vcsr,
because the reference's std::sort leaves the order of equal-count rows open.

Run (where the reference tree is present):
    make -C oracle && python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402

MTX_CASES = {
    # file: list of (segw, bundle) VCSR builds to record
    "tiny_1based.mtx": [(4, 32), (2, 2), (1, 1)],
    "tiny_0based.mtx": [(4, 32), (2, 3)],
    "blank_lines.mtx": [(4, 2), (3, 1)],
    "empty_rows.mtx": [(4, 32), (4, 2), (16, 4)],
    "no_entries.mtx": [(4, 32)],
    "bad_header.mtx": [],
    "short_data.mtx": [],
    "row_out_of_range.mtx": [],
    "garbled_value.mtx": [],
}


def random_csr(seed, M, N, density, dup_rows=(), dense_rows=(), all_seg0=False):
    rng = np.random.default_rng(seed)
    rows, cols = [], []
    for r in range(M):
        if r in dense_rows:
            cs = np.arange(N)
        else:
            k = rng.binomial(N, density)
            cs = np.sort(rng.choice(N, size=k, replace=False))
        if all_seg0 and (len(cs) == 0 or cs[0] != 0):
            cs = np.concatenate([[0], cs[cs != 0]])
        if r in dup_rows and len(cs):
            cs = np.sort(np.concatenate([cs, cs[: min(3, len(cs))]]))
        rows += [r] * len(cs)
        cols += list(cs)
    rows = np.asarray(rows, np.int32)
    cols = np.asarray(cols, np.int32)
    vals = rng.uniform(-1, 1, len(rows)).astype(np.float32)
    perm = rng.permutation(len(rows))  # COO order is arbitrary
    return rows[perm], cols[perm], vals[perm]


RANDOM_CASES = [
    # name, seed, M, N, density, extras, [(segw, bundle)]
    ("r1", 1, 37, 50, 0.10, {}, [(4, 8), (4, 32)]),
    ("r2", 2, 100, 103, 0.05, {}, [(4, 32), (8, 16)]),
    ("r3", 3, 64, 64, 0.20, {}, [(16, 32), (4, 4)]),
    ("r4_dups", 4, 20, 30, 0.15, {"dup_rows": (1, 5, 9)}, [(4, 4), (2, 8)]),
    ("r5_dense_row", 5, 50, 200, 0.02, {"dense_rows": (7,)}, [(8, 16), (4, 32)]),
    ("r6_all_seg0", 6, 33, 40, 0.10, {"all_seg0": True}, [(4, 8), (5, 32)]),
    ("r7_unit", 7, 16, 16, 0.25, {}, [(1, 1), (1, 4)]),
    ("r8_empty", 8, 5, 5, 0.0, {}, [(4, 32)]),
    ("r9_wide_seg", 9, 10, 3, 0.5, {}, [(4, 2)]),
]


def put_vcsr(store, prefix, v):
    for k in ("group_ptr", "group_depth", "group_seg_base", "group_rows",
              "lcol", "val"):
        store[f"{prefix}/{k}"] = np.asarray(v[k])
    store[f"{prefix}/meta"] = np.asarray(
        [v["M"], v["N"], v["segw"], v["bundle"], v["num_groups"], v["num_slots"]],
        np.int64)


def main():
    if not oracle.ref_available():
        sys.exit("oracle/_ref/libvcsr_ref.so missing: run `make -C oracle` "
                 "where the reference tree is present")
    store = {}
    errors = {}
    for fname, builds in MTX_CASES.items():
        path = os.path.join(HERE, "mtx", fname)
        key = fname[:-4]
        try:
            M, N, r, c, v = oracle.ref_read_mtx(path)
        except oracle.OracleError as e:
            errors[key] = {"stage": "read", "msg": e.msg}
            continue
        store[f"{key}/coo_shape"] = np.asarray([M, N], np.int64)
        store[f"{key}/coo_rows"], store[f"{key}/coo_cols"] = r, c
        store[f"{key}/coo_vals"] = v
        try:
            rp, cc, vv = oracle.ref_coo_to_csr(M, N, r, c, v)
        except oracle.OracleError as e:
            errors[key] = {"stage": "coo_to_csr", "msg": e.msg}
            continue
        store[f"{key}/csr_row_ptr"], store[f"{key}/csr_col"] = rp, cc
        store[f"{key}/csr_val"] = vv
        for segw, bundle in builds:
            vc = oracle.ref_csr_to_vcsr(M, N, rp, cc, vv, segw, bundle)
            put_vcsr(store, f"{key}/vcsr_s{segw}_b{bundle}", vc)
    for name, seed, M, N, dens, extra, builds in RANDOM_CASES:
        r, c, v = random_csr(seed, M, N, dens, **extra)
        store[f"{name}/coo_shape"] = np.asarray([M, N], np.int64)
        store[f"{name}/coo_rows"], store[f"{name}/coo_cols"] = r, c
        store[f"{name}/coo_vals"] = v
        rp, cc, vv = oracle.ref_coo_to_csr(M, N, r, c, v)
        store[f"{name}/csr_row_ptr"], store[f"{name}/csr_col"] = rp, cc
        store[f"{name}/csr_val"] = vv
        for segw, bundle in builds:
            vc = oracle.ref_csr_to_vcsr(M, N, rp, cc, vv, segw, bundle)
            put_vcsr(store, f"{name}/vcsr_s{segw}_b{bundle}", vc)
    store["__errors__"] = np.frombuffer(json.dumps(errors, sort_keys=True).encode(),
                                        np.uint8)
    out = os.path.join(HERE, "ref_outputs.npz")
    np.savez_compressed(out, **store)
    print(f"wrote {out}: {len(store)} arrays, errors: {errors}")


if __name__ == "__main__":
    main()
