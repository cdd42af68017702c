"""Host logic of multi-GPU row panels (one process per GPU under torchrun).

The reference has no multi-GPU path.  The engine's: A is cut into row panels,
every rank builds a plan for its own panel, B is replicated once from rank 0
by a broadcast (NCCL over NVLink on GPUs; gloo in the CPU tests), C panels are
disjoint so nothing is reduced, and a timing is the max over ranks.

Two ways to own rows:
  * "strong": one global matrix, cut into panels of balanced cost (nnz plus
    a per-row weight, vcsr_partition_rows_weighted; cuts aligned to `align`
    rows);
  * "weak": every rank owns a full panel of its own (seed + rank), so the
    global matrix has world * M rows and per-rank work is fixed.
"""
from __future__ import annotations

from . import CSR, VcsrError, csr_row_panel, gen_csr, partition_rows

STATUS_NCCL, STATUS_TIMEOUT = 6, 7


def init_ranks(dist, backend: str = "nccl", timeout_s: float = 60.0, device=None):
    """init_process_group with a bounded rendezvous and collective timeout.

    A rank that never joins makes the others fail after about `timeout_s`
    with VcsrError(status 7) instead of waiting for ever; the same timeout
    bounds every later collective of the group."""
    import datetime
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None:
        kw["device_id"] = device
    try:
        dist.init_process_group(backend, **kw)
    except Exception as e:  # the store's rendezvous timed out or was refused
        raise VcsrError(STATUS_TIMEOUT, f"rank rendezvous ({backend}) did not complete "
                                        f"within {timeout_s:g} s: {e}") from e


def _collective(what, fn):
    """Run one collective; a peer that failed or left between steps turns
    into VcsrError(status 6) on the ranks still running."""
    try:
        return fn()
    except VcsrError:
        raise
    except Exception as e:
        raise VcsrError(STATUS_NCCL, f"{what}: a peer rank failed, left or timed out: {e}") from e


# Strong scaling cuts A into panels of equal nnz + ROW_WEIGHT * rows.  Each
# row also costs its C row write (as many bytes as one entry's B row) and
# its own set-up: measured on two B200s on R-MAT 2^22 at O = 256, panels of
# equal nnz took 3.15 ms (0.59M rows) and 3.72 ms (3.6M rows), i.e. about
# 0.093 ms per million entries and 0.19 ms per million rows: a row weighs
# about two entries.
ROW_WEIGHT = 2.0


def rank_panel(config: str, size: int, seed: int, rank: int, world: int,
               scaling: str, align: int = 16, row_weight: float = ROW_WEIGHT):
    """(panel CSR, first global row, global nnz) of this rank."""
    if scaling == "weak":
        csr = gen_csr(config, seed + rank, size)
        return csr, rank * csr.M, None
    full = gen_csr(config, seed, size)
    if world == 1:
        return full, 0, full.nnz
    cuts = partition_rows(full.row_ptr, world, align, row_weight)
    panel = csr_row_panel(full, int(cuts[rank]), int(cuts[rank + 1]))
    return panel, int(cuts[rank]), full.nnz


def global_nnz(panel: CSR, scaling: str, world: int, strong_total=None, dist=None,
               device=None):
    """Total nnz over all ranks (weak: summed with an all-reduce)."""
    if scaling == "strong" and strong_total is not None:
        return int(strong_total)
    if world == 1 or dist is None:
        return panel.nnz * world if dist is None else panel.nnz
    import torch
    t = torch.tensor([panel.nnz], dtype=torch.int64, device=device)
    _collective("global nnz", lambda: dist.all_reduce(t, op=dist.ReduceOp.SUM))
    return int(t.item())


def broadcast_b(dist, tensor, src: int = 0):
    """Replicate B from `src` to every rank (one collective)."""
    _collective("broadcast of B", lambda: dist.broadcast(tensor, src=src))
    return tensor


def broadcast_and_multiply(dist, plan, dB, dC, src: int = 0, chunks: int = 4, stream=None):
    """Replicate B from `src` and compute C = A*B with the two overlapped.

    B goes out as `chunks` row chunks (asynchronous broadcasts, the same on
    every rank, so every rank takes the same collective steps); this rank
    multiplies each of its plan's row panels as soon as the chunk holding the
    panel's highest column has arrived.  The broadcasts, the waits and the
    products are all issued with `stream` (a torch.cuda.Stream or a raw
    cudaStream_t; default the current stream) made the current stream: waiting
    on a collective makes the CURRENT stream wait, so the products, enqueued
    on that same stream, never read rows of B before they have arrived; the
    host does not wait.  For banded matrices the products of
    the early panels run while later chunks are still on the wire.  A plan
    without row panels, or whose panels are not banded (some panel reads rows of
    B beyond the next chunk), waits for all of B and multiplies in one call.
    Returns the number of panels multiplied before the last chunk arrived.
    Measured on two B200s each chunk costs a collective's latency (~20 us), so
    this pays only when the product is long next to the broadcast."""
    import contextlib
    ctx = contextlib.nullcontext()
    if stream is not None and getattr(dB, "is_cuda", False):
        import torch
        if isinstance(stream, int):
            stream = torch.cuda.ExternalStream(stream)
        ctx = torch.cuda.stream(stream)
    with ctx:
        return _broadcast_and_multiply(dist, plan, dB, dC, src, chunks, stream)


def _broadcast_and_multiply(dist, plan, dB, dC, src, chunks, stream):
    N = dB.shape[0]
    per = -(-N // chunks) if N else 0
    works = []
    for i in range(chunks):
        r0, r1 = min(N, i * per), min(N, (i + 1) * per)
        works.append(dist.broadcast(dB[r0:r1], src=src, async_op=True) if r1 > r0 else None)
    done = -1

    def wait_through(k):
        nonlocal done
        while done < k:
            done += 1
            if works[done] is not None:
                works[done].wait()

    panels = plan.row_panels()
    need = [0 if cm < 0 or per == 0 else min(chunks - 1, cm // per) for _, _, cm in panels]
    if not panels or any(need[j] > j + 1 for j in range(len(need))):
        wait_through(chunks - 1)
        plan.spmm(dB, dC, stream=stream)
        return 0
    early = 0
    for j in range(len(panels)):
        wait_through(need[j])
        if done < chunks - 1:
            early += 1
        plan.spmm_row_panel(j, dB, dC, stream=stream)
    wait_through(chunks - 1)
    return early


def sum_over_ranks(dist, value: int, device=None) -> int:
    """An integer summed over every rank (e.g. the global row count)."""
    import torch
    t = torch.tensor([int(value)], dtype=torch.int64, device=device)
    _collective("sum over ranks", lambda: dist.all_reduce(t, op=dist.ReduceOp.SUM))
    return int(t.item())


def max_over_ranks(dist, value: float, device=None) -> float:
    """The slowest rank's time."""
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    _collective("max over ranks", lambda: dist.all_reduce(t, op=dist.ReduceOp.MAX))
    return float(t.item())
