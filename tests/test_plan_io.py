"""vcsr_plan_save / vcsr_plan_load: a plan written to disk and read back
gives the same products, bit for bit; damaged, truncated, foreign and
other-version files are refused before anything reaches the device (those
cases run without a GPU)."""
import os
import struct

import numpy as np
import pytest

import oracle
import vcsr_b200 as V
from helpers import rel_l2


def fnv1a(b: bytes) -> int:
    h = 1469598103934665603
    for x in b:
        h = ((h ^ x) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def load_status(path):
    with pytest.raises(V.VcsrError) as ei:
        V.Plan.load(path)
    return ei.value.status


def test_refuses_missing_and_foreign_files(tmp_path):
    assert load_status(os.path.join(tmp_path, "none.plan")) == 4
    p = os.path.join(tmp_path, "junk.plan")
    with open(p, "wb") as f:
        f.write(os.urandom(4096))
    assert load_status(p) == 4
    with open(p, "wb") as f:  # right magic, wrong checksum
        f.write(b"VCSRPLAN" + os.urandom(200))
    assert load_status(p) == 4


def test_refuses_other_version_and_bad_header(tmp_path):
    p = os.path.join(tmp_path, "v.plan")
    body = b"VCSRPLAN" + struct.pack("<qq", 99, 1) + bytes(8 * 41)
    with open(p, "wb") as f:
        f.write(body + struct.pack("<Q", fnv1a(body)))
    assert load_status(p) == 5
    abi = V.lib().vcsr_abi_version()
    body = b"VCSRPLAN" + struct.pack("<qq", 4, abi) + struct.pack("<q", -5) + bytes(8 * 40)
    with open(p, "wb") as f:
        f.write(body + struct.pack("<Q", fnv1a(body)))
    assert load_status(p) == 4  # negative M


def _cuda():
    import torch as t
    return t


@pytest.mark.gpu
@pytest.mark.parametrize("cfg,size,O,kw", [
    ("fem", 20000, 128, {}),
    ("powerlaw", 60000, 64, {}),                 # split vectors and long units
    ("blockdense", 2048, 64, {"tf32_panels": True}),
    ("uniform", 0, 32, {"reference_format": True}),
])
def test_round_trip(tmp_path, cfg, size, O, kw):
    t = _cuda()
    csr = V.gen_csr(cfg, 2, size)
    a = V.Plan(csr, **kw)
    path = os.path.join(tmp_path, "a.plan")
    a.save(path)
    b = V.Plan.load(path)
    ia, ib = a.info(), b.info()
    for k in ia:
        if k not in ("build_ms",):
            assert ia[k] == ib[k], k
    B = t.from_numpy(V.gen_dense_host(csr.N, O, 3)).cuda()
    Ca = t.empty(csr.M, O, device="cuda")
    Cb = t.full((csr.M, O), float("nan"), device="cuda")
    a.spmm(B, Ca)
    b.spmm(B, Cb)
    b.check()
    t.cuda.synchronize()
    assert t.equal(Ca, Cb)
    # and the loaded plan's product is the oracle's CSR sum
    ref = oracle.csr_spmm_f64(csr.M, csr.row_ptr, csr.col, csr.val, B.cpu().numpy())
    assert rel_l2(Cb.cpu().numpy(), ref) <= (2e-3 if kw.get("tf32_panels") else 1e-5)
    if kw.get("reference_format"):
        ea, eb = a.export(), b.export()
        for f in ("group_ptr", "group_depth", "group_seg_base", "group_rows", "lcol", "val"):
            assert np.array_equal(getattr(ea, f), getattr(eb, f)), f
    # damaged and truncated copies of a real file
    raw = open(path, "rb").read()
    bad = bytearray(raw)
    bad[len(bad) // 2] ^= 0x40
    p2 = os.path.join(tmp_path, "bad.plan")
    open(p2, "wb").write(bytes(bad))
    assert load_status(p2) == 4
    open(p2, "wb").write(raw[: len(raw) - 100])
    assert load_status(p2) == 4
