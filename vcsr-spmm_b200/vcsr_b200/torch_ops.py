"""A PyTorch operator over the C ABI: torch.ops.vcsr.spmm(plan_id, B) -> C.

The reference has no Python or PyTorch binding; this one lets PyTorch code
(and graph capture by tracers, through the fake implementation below) call a
plan's C = A * B like any other operator.  Forward only: no gradient is
registered.  The product always runs on the engine's CUDA kernels; there is no
fallback when the library or a GPU is missing.

    from vcsr_b200 import Plan, torch_ops
    plan = Plan(csr)
    pid = torch_ops.register(plan)
    C = torch.ops.vcsr.spmm(pid, B)      # B: (N, O) float32 or bfloat16, CUDA
"""
from __future__ import annotations

import itertools
import threading

import torch

from . import Plan

_plans: dict[int, Plan] = {}
_ids = itertools.count(1)
_lock = threading.Lock()


def register(plan: Plan) -> int:
    """An id under which torch.ops.vcsr.spmm finds `plan` (kept alive until
    unregister)."""
    with _lock:
        pid = next(_ids)
        _plans[pid] = plan
    return pid


def unregister(pid: int) -> None:
    with _lock:
        _plans.pop(pid, None)


def _plan(pid: int) -> Plan:
    try:
        return _plans[pid]
    except KeyError:
        raise ValueError(f"no plan registered under id {pid}") from None


@torch.library.custom_op("vcsr::spmm", mutates_args=())
def spmm(plan_id: int, B: torch.Tensor) -> torch.Tensor:
    """C = A * B for the registered plan; B is (N, O), float32 or bfloat16,
    on a CUDA device; C is (M, O) float32 on the same device."""
    plan = _plan(plan_id)
    if B.dim() != 2 or B.shape[0] != plan.N:
        raise ValueError(f"B must be ({plan.N}, O), got {tuple(B.shape)}")
    if B.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"B must be float32 or bfloat16, got {B.dtype}")
    if B.stride(1) != 1:
        B = B.contiguous()
    C = torch.empty(plan.M, B.shape[1], device=B.device, dtype=torch.float32)
    plan.spmm(B, C, stream=torch.cuda.current_stream(B.device))
    return C


@spmm.register_fake
def _spmm_fake(plan_id: int, B: torch.Tensor) -> torch.Tensor:
    plan = _plan(plan_id)
    return B.new_empty((plan.M, B.shape[1]), dtype=torch.float32)
