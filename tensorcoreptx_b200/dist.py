"""Row-sharded multi-GPU GEMM: one process per GPU over torch.distributed.

The reference has no multi-GPU code; this is the sharded configuration its
benchmark calls for: A is partitioned by rows across the ranks, B is
replicated, and each rank computes its rows of C with the local tensor-core
GEMM.  No collective is on the data path; ``gather=True`` adds an all-gather
of C (NCCL over NVLink on GPUs) so every rank ends with the full C.

Failure behaviour: collectives use the process group's timeout, so a rank
that dies or never joins turns into an error on the others instead of a hang.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist


def shard_rows(M: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Rows [r0, r1) of an M-row matrix owned by `rank` of `world`.

    Shards are as equal as `align` allows (every boundary but the last is a
    multiple of `align`); earlier ranks get the larger shards.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank / world size")
    units = -(-M // align)
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return min(M, u0 * align), min(M, u1 * align)


def max_over_ranks(x: float, device: Optional[torch.device] = None, group=None) -> float:
    """Maximum of a host scalar over all ranks (identity when not distributed)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size(group) == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64,
                     device=device if device is not None else torch.device("cpu"))
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sharded_gemm_int8(A_local: torch.Tensor, BT: torch.Tensor, gather: bool = False,
                      out: Optional[torch.Tensor] = None, group=None,
                      local_gemm: Optional[Callable] = None) -> torch.Tensor:
    """C rows of this rank = A_local x BT^T (int8 -> int32); with gather=True
    return the full C (rows of rank r at the position shard_rows gives them,
    equal shards required) after an all-gather over `group`.

    `local_gemm` defaults to the tensor-core GEMM (gemm_int8).
    """
    if local_gemm is None:
        from .gemm import gemm_int8 as local_gemm
    C_local = local_gemm(A_local, BT)
    if not gather:
        return C_local
    world = dist.get_world_size(group)
    rows = C_local.shape[0]
    if out is None:
        out = torch.empty((rows * world, C_local.shape[1]), dtype=C_local.dtype, device=C_local.device)
    if out.shape[0] != rows * world:
        raise RuntimeError("gather needs equal shards: out must have world x local rows")
    dist.all_gather_into_tensor(out, C_local.contiguous(), group=group)
    return out
