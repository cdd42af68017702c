"""The multi-GPU row-panel host logic (vcsr_b200.dist) with world size 2 on
the gloo backend, on CPU.  The CPU oracle stands in for each rank's GPU SpMM:
the test checks panel cuts, the broadcast of B, the gathered C against the
single-process result, the global nnz and the max-over-ranks timing."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, scaling, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path.insert(0, os.path.join(root, "vcsr-spmm_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import oracle
    import vcsr_b200 as V
    from vcsr_b200 import dist as D
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, size = ("rmat", 11) if scaling == "strong" else ("fem", 900)
        panel, row0, total = D.rank_panel(cfg, size, 0, rank, world, scaling)
        nnz = D.global_nnz(panel, scaling, world, total, dist)
        O = 16
        B = torch.zeros(panel.N, O)
        if rank == 0:
            B = torch.from_numpy(V.gen_dense_host(panel.N, O, 5))
        D.broadcast_b(dist, B, 0)
        C = oracle.csr_spmm_f32(panel.M, panel.row_ptr, panel.col, panel.val, B.numpy())
        t = D.max_over_ranks(dist, 1.0 + rank)
        sizes = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(sizes, torch.tensor([panel.M], dtype=torch.int64))
        mx = max(int(s.item()) for s in sizes)  # gloo gathers equal shapes: pad
        Ct = torch.zeros(mx, O)
        Ct[:panel.M] = torch.from_numpy(C)
        gathered = [torch.zeros(mx, O) for _ in sizes]
        dist.all_gather(gathered, Ct)
        if rank == 0:
            Cfull = torch.cat([g[:int(s.item())] for g, s in zip(gathered, sizes)])
            out.put((Cfull.numpy(), B.numpy(), nnz, t, row0))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.parametrize("scaling", ["strong", "weak"])
def test_two_rank_row_panels(scaling):
    import oracle
    import vcsr_b200 as V
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, scaling, q)) for r in range(2)]
    for p in procs:
        p.start()
    C, B, nnz, t, row0 = q.get(timeout=240)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert t == 2.0  # the slowest rank
    if scaling == "strong":
        full = V.gen_csr("rmat", 0, 11)
        ref = oracle.csr_spmm_f32(full.M, full.row_ptr, full.col, full.val, B)
        assert nnz == full.nnz
        assert np.array_equal(C, ref)  # same rows, same CSR order: bit for bit
        cuts = V.partition_rows(full.row_ptr, 2, 16)
        assert cuts[1] % 16 == 0
        left = full.row_ptr[cuts[1]]
        assert abs(left - (full.nnz - left)) <= 16 * np.diff(full.row_ptr).max()
    else:
        parts = [V.gen_csr("fem", r, 900) for r in range(2)]
        ref = np.concatenate([oracle.csr_spmm_f32(p.M, p.row_ptr, p.col, p.val, B)
                              for p in parts])
        assert nnz == sum(p.nnz for p in parts)
        assert np.array_equal(C, ref)


class _FakePlan:
    """Stands in for a GPU plan: row panels of about equal rows and their
    highest column; products by the CPU oracle.  Records which panels ran."""

    def __init__(self, csr, n_panels):
        import oracle
        self.oracle, self.csr, self.N, self.ran = oracle, csr, csr.N, []
        cuts = np.linspace(0, csr.M, n_panels + 1).astype(int) if n_panels else []
        self.panels = []
        for a, b in zip(cuts[:-1], cuts[1:]):
            cols = csr.col[csr.row_ptr[a]:csr.row_ptr[b]]
            self.panels.append((int(a), int(b), int(cols.max()) if len(cols) else -1))

    def row_panels(self):
        return self.panels

    def _rows(self, a, b, B, C):
        c = self.csr
        rp = (c.row_ptr[a:b + 1] - c.row_ptr[a]).astype(np.int32)
        C[a:b] = torch.from_numpy(self.oracle.csr_spmm_f32(
            b - a, rp, c.col[c.row_ptr[a]:c.row_ptr[b]], c.val[c.row_ptr[a]:c.row_ptr[b]],
            B.numpy()))

    def spmm_row_panel(self, j, B, C, stream=None):
        self.ran.append(j)
        a, b, _ = self.panels[j]
        self._rows(a, b, B, C)

    def spmm(self, B, C, stream=None):
        self.ran.append("all")
        self._rows(0, self.csr.M, B, C)


def _worker_overlap(rank, world, port, out):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    sys.path.insert(0, os.path.join(root, "vcsr-spmm_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    import vcsr_b200 as V
    from vcsr_b200 import dist as D
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # rank 0: a banded matrix with row panels; rank 1: a plan without panels
        csr = V.gen_csr("fem", rank, 24000)  # band ~460 rows < a 3000-row chunk
        plan = _FakePlan(csr, 8 if rank == 0 else 0)
        O = 8
        B = torch.zeros(csr.N, O)
        if rank == 0:
            B[:] = torch.from_numpy(V.gen_dense_host(csr.N, O, 7))
        C = torch.full((csr.M, O), float("nan"))
        early = D.broadcast_and_multiply(dist, plan, B, C, src=0, chunks=8)
        # a matrix whose early rows read late columns is not banded: one product
        # after all of B (the broadcasts are the same on both ranks)
        perm = _FakePlan(csr, 8)
        perm.panels = [(a, b, csr.N - 1) for a, b, _ in perm.panels]
        C2 = torch.full((csr.M, O), float("nan"))
        e2 = D.broadcast_and_multiply(dist, perm, B, C2, src=0, chunks=8)
        ref = torch.zeros_like(C)
        _FakePlan(csr, 0).spmm(B, ref)
        out[rank] = (early, plan.ran, bool(torch.equal(C, ref)) and e2 == 0 and perm.ran == ["all"],
                     bool(torch.equal(B, torch.from_numpy(V.gen_dense_host(csr.N, O, 7)))))
    finally:
        dist.destroy_process_group()


def test_two_rank_broadcast_overlapped_with_panels():
    """Chunked broadcast of B with each row panel multiplied as soon as its
    rows of B are in: every rank takes the same broadcasts, a banded plan runs
    panels before the last chunk, a plan without panels waits for all of B, and
    C is the full product on both."""
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker_overlap, args=(2, _free_port(), out), nprocs=2, join=True)
    e0, ran0, ok0, b0 = out[0]
    e1, ran1, ok1, b1 = out[1]
    assert ok0 and ok1 and b0 and b1
    assert ran0 == list(range(8)) and 0 < e0 <= 7  # banded: early panels
    assert ran1 == ["all"] and e1 == 0
