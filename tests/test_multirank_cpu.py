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
