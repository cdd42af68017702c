"""Failure paths made on the host, on CPU (no GPU is faulted or hung).

* An allocator limit: a child process lowers its address-space limit, then
  asks the library for more host memory than the limit leaves.  Every entry
  point must return VCSR_ERR_ALLOC (3) with a message: no crash, no C++
  exception across the C ABI, no partial output.
* A rank that never joins: the others' rendezvous ends with an error after a
  bounded timeout (vcsr_b200.dist.init_ranks), instead of waiting for ever.
* A rank that leaves between steps: the next collective of the ranks still
  running ends with an error (VcsrError, status 6), bounded by the timeout.
"""
import multiprocessing as mp
import os
import socket
import time

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _paths():
    import sys
    for p in (os.path.join(ROOT, "vcsr-spmm_b200"), os.path.join(ROOT, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _alloc_child(mtx_path, q):
    import ctypes as C
    import resource
    _paths()
    import vcsr_b200 as V
    L = V.lib()
    # current address space + 768 MB: the library's own allocations of a few GB fail
    with open("/proc/self/statm") as f:
        vm = int(f.read().split()[0]) * os.sysconf("SC_PAGE_SIZE")
    lim = vm + (768 << 20)
    resource.setrlimit(resource.RLIMIT_AS, (lim, lim))
    out = []
    csr = V._Csr()
    st = L.vcsr_gen_csr(b"rmat", 0, 25, C.byref(csr))  # 2^25 rows, 537M edges
    out.append(("gen_csr", st, L.vcsr_last_error().decode(), csr.M, bool(csr.row_ptr)))
    coo = V._Coo()
    st = L.vcsr_read_mtx(mtx_path.encode(), C.byref(coo))  # header claims 400M entries
    out.append(("read_mtx", st, L.vcsr_last_error().decode(), coo.nnz, bool(coo.rows)))
    # a small call still works afterwards
    st = L.vcsr_gen_csr(b"uniform", 0, 64, C.byref(csr))
    out.append(("after", st, "", csr.M, bool(csr.row_ptr)))
    L.vcsr_csr_free(C.byref(csr), 0)
    q.put(out)


def test_host_allocation_failure_is_a_status(tmp_path):
    mtx = tmp_path / "huge.mtx"
    mtx.write_text("%%MatrixMarket matrix coordinate real general\n"
                   "100000000 100000000 400000000\n1 1 1.0\n")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_alloc_child, args=(str(mtx), q))
    p.start()
    out = q.get(timeout=240)
    p.join(timeout=60)
    assert p.exitcode == 0
    (n1, s1, m1, M1, has1), (n2, s2, m2, z2, has2), (n3, s3, _, M3, has3) = out
    assert s1 == 3 and "host memory" in m1 and M1 == 0 and not has1, out[0]
    assert s2 == 3 and "host memory" in m2 and not has2, out[1]
    assert s3 == 0 and M3 == 64 and has3


def _never_join_rank0(port, q):
    _paths()
    import torch.distributed as dist
    from vcsr_b200 import VcsrError
    from vcsr_b200 import dist as D
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="0",
                      WORLD_SIZE="2")
    t0 = time.time()
    try:
        D.init_ranks(dist, "gloo", timeout_s=3)
        q.put(("joined", None, time.time() - t0))
    except VcsrError as e:
        q.put(("error", e.status, time.time() - t0))


def test_rank_that_never_joins_ends_in_a_bounded_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_never_join_rank0, args=(_free_port(), q))  # rank 1 never starts
    p.start()
    what, status, dt = q.get(timeout=120)
    p.join(timeout=30)
    assert what == "error" and status == 7
    assert dt < 30


def _leaving_rank(rank, port, q):
    _paths()
    import torch.distributed as dist
    from vcsr_b200 import VcsrError
    from vcsr_b200 import dist as D
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE="2")
    D.init_ranks(dist, "gloo", timeout_s=5)
    first = D.max_over_ranks(dist, 1.0 + rank)  # step 1: both ranks
    if rank == 1:
        q.put((rank, "left", first, 0.0))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # leaves between steps, with nothing in flight
    time.sleep(0.5)
    t0 = time.time()
    try:
        D.max_over_ranks(dist, 1.0)  # step 2: the peer is gone
        q.put((rank, "finished", first, time.time() - t0))
    except VcsrError as e:
        q.put((rank, f"error {e.status}", first, time.time() - t0))


def test_rank_that_leaves_between_steps_ends_the_next_collective():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leaving_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = {}
    for _ in range(2):
        r, what, first, dt = q.get(timeout=120)
        got[r] = (what, first, dt)
    for p in ps:
        p.join(timeout=60)
    assert got[1][0] == "left"
    assert got[0][1] == 2.0  # step 1 saw both ranks
    assert got[0][0] == "error 6" and got[0][2] < 30
