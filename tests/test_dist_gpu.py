"""Two ranks over NCCL (needs two GPUs; skipped otherwise).

broadcast_and_multiply given a stream that is NOT the current one: every
product must still come after the chunk of B it reads.  Rank 1's B starts
as NaN, so a product that ran before its rows of B arrived would leave NaN
in C; C must equal, bit for bit, the same plan's product on the full B.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import sys
    import datetime
    import torch.distributed as dist
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.join(os.path.dirname(here), "vcsr-spmm_b200"))
    import vcsr_b200 as V
    from vcsr_b200 import dist as D
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        csr = V.gen_csr("fem", rank, 40000)  # banded: the plan has row panels
        plan = V.Plan(csr)
        O = 64
        full = torch.empty(csr.N, O, device=dev)
        V.gen_dense_device(full, 5)  # the same B on both ranks
        want = torch.empty(csr.M, O, device=dev)
        plan.spmm(full, want)
        torch.cuda.synchronize()
        dB = full.clone() if rank == 0 else torch.full_like(full, float("nan"))
        side = torch.cuda.Stream(device=dev)  # not the current stream
        results = []
        for _ in range(3):
            if rank != 0:
                dB.fill_(float("nan"))
            dC = torch.full((csr.M, O), float("nan"), device=dev)
            torch.cuda.synchronize()
            early = D.broadcast_and_multiply(dist, plan, dB, dC, src=0, chunks=4, stream=side)
            side.synchronize()
            torch.cuda.synchronize()
            results.append((early, bool(torch.equal(dC, want))))
        out[rank] = (len(plan.row_panels()), results)
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_broadcast_and_multiply_on_a_side_stream():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    for r in range(2):
        n_panels, results = out[r]
        assert n_panels > 0
        for early, same in results:
            assert same
