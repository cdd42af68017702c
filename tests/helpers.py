"""Shared test helpers: golden-fixture access and comparisons."""
import json
import os

import numpy as np

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
MTX_DIR = os.path.join(ROOT, "tests", "golden", "mtx")
VKEYS = ("group_ptr", "group_depth", "group_seg_base", "group_rows", "lcol", "val")


def golden_cases(z):
    return sorted({k.split("/")[0] for k in z.files if "/" in k})


def golden_errors(z):
    return json.loads(bytes(z["__errors__"]).decode())


def golden_vcsr_builds(z, case):
    """[(segw, bundle, reference VCSR dict)] recorded for a case."""
    out = []
    for k in z.files:
        if k.startswith(case + "/vcsr") and k.endswith("/meta"):
            pre = k[:-5]
            meta = z[k]
            d = {kk: z[f"{pre}/{kk}"] for kk in VKEYS}
            d.update(M=int(meta[0]), N=int(meta[1]), segw=int(meta[2]),
                     bundle=int(meta[3]), num_groups=int(meta[4]),
                     num_slots=int(meta[5]))
            out.append((d["segw"], d["bundle"], d))
    return sorted(out, key=lambda t: (t[0], t[1]))


def vcsr_equal_canonical(a, b):
    """Bit-exact equality after fixing the tie order (oracle.canonical_vcsr)."""
    ca, cb = oracle.canonical_vcsr(a), oracle.canonical_vcsr(b)
    for k in VKEYS:
        x, y = np.asarray(ca[k]), np.asarray(cb[k])
        if x.shape != y.shape or not np.array_equal(x.view(np.int32) if x.dtype == np.float32 else x,
                                                    y.view(np.int32) if y.dtype == np.float32 else y):
            return False, k
    return True, None


def vcsr_equal_exact(a, b):
    for k in VKEYS:
        x, y = np.asarray(a[k]), np.asarray(b[k])
        if x.shape != y.shape or not np.array_equal(x, y):
            return False, k
    return True, None


def rel_l2(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.linalg.norm(ref)
    num = np.linalg.norm(x - ref)
    return float(num / den) if den > 0 else float(num)


def random_csr(seed, M, N, density, dup_rows=(), dense_rows=(), unsorted=False):
    rng = np.random.default_rng(seed)
    rows, cols = [], []
    for r in range(M):
        if r in dense_rows:
            cs = np.arange(N)
        else:
            k = rng.binomial(N, density)
            cs = np.sort(rng.choice(N, size=k, replace=False))
        if r in dup_rows and len(cs):
            cs = np.sort(np.concatenate([cs, cs[: min(3, len(cs))]]))
        rows += [r] * len(cs)
        cols += list(cs)
    rows = np.asarray(rows, np.int32)
    cols = np.asarray(cols, np.int32)
    vals = rng.uniform(-1, 1, len(rows)).astype(np.float32)
    rp = np.zeros(M + 1, np.int32)
    np.add.at(rp, rows + 1, 1)
    rp = np.cumsum(rp).astype(np.int32)
    order = np.lexsort((cols, rows))
    col, val = cols[order], vals[order]
    if unsorted:
        for r in range(M):
            s, e = rp[r], rp[r + 1]
            p = rng.permutation(e - s)
            col[s:e], val[s:e] = col[s:e][p], val[s:e][p]
    return rp, col, val
