"""Host logic of multi-GPU row panels (one process per GPU under torchrun).

The reference has no multi-GPU path.  The engine's: A is cut into row panels,
every rank builds a plan for its own panel, B is replicated once from rank 0
by a broadcast (NCCL over NVLink on GPUs; gloo in the CPU tests), C panels are
disjoint so nothing is reduced, and a timing is the max over ranks.

Two ways to own rows:
  * "strong": one global matrix, cut into nnz-balanced panels
    (vcsr_partition_rows, cuts aligned to `align` rows);
  * "weak": every rank owns a full panel of its own (seed + rank), so the
    global matrix has world * M rows and per-rank work is fixed.
"""
from __future__ import annotations

from . import CSR, csr_row_panel, gen_csr, partition_rows


def rank_panel(config: str, size: int, seed: int, rank: int, world: int,
               scaling: str, align: int = 16):
    """(panel CSR, first global row, global nnz) of this rank."""
    if scaling == "weak":
        csr = gen_csr(config, seed + rank, size)
        return csr, rank * csr.M, None
    full = gen_csr(config, seed, size)
    if world == 1:
        return full, 0, full.nnz
    cuts = partition_rows(full.row_ptr, world, align)
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
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())


def broadcast_b(dist, tensor, src: int = 0):
    """Replicate B from `src` to every rank (one collective)."""
    dist.broadcast(tensor, src=src)
    return tensor


def max_over_ranks(dist, value: float, device=None) -> float:
    """The slowest rank's time."""
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
