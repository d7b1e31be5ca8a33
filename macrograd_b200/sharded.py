"""Row-sharded GEMM across ranks (one process per GPU).

C = A @ B where the rows of A (and so of C) are split over the ranks and B is
replicated. Rows of C depend only on the same rows of A, so each rank's GEMM is
independent -- no collective inside the GEMM. When the caller needs the whole C
on every device, the row blocks are all-gathered (NCCL over NVLink on GPUs,
gloo on CPU in the tests). The reference has no multi-device path; this is the
batch/row-sharded layer its matmul path gains here.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist


def row_block(rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous row range [r0, r1) of `rank`; the first rows % world ranks
    take one extra row, so any row count splits."""
    base, extra = divmod(rows, world)
    r0 = rank * base + min(rank, extra)
    r1 = r0 + base + (1 if rank < extra else 0)
    return r0, r1


def gather_rows(full: torch.Tensor, local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather the ranks' row blocks of C into `full` (every rank)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    rows = full.shape[0]
    sizes = [row_block(rows, world, r) for r in range(world)]
    even = all((b - a) == (sizes[0][1] - sizes[0][0]) for a, b in sizes)
    if even and full.is_cuda:
        dist.all_gather_into_tensor(full, local.contiguous(), group=group)
    else:
        parts = [full[a:b] for a, b in sizes]
        if even:
            dist.all_gather(parts, local.contiguous(), group=group)
        else:
            # uneven blocks: gather padded blocks, then keep each rank's rows
            pad = max(b - a for a, b in sizes)
            buf = local.new_zeros((pad,) + tuple(local.shape[1:]))
            buf[: local.shape[0]] = local
            bufs = [torch.empty_like(buf) for _ in range(world)]
            dist.all_gather(bufs, buf, group=group)
            for (a, b), got in zip(sizes, bufs):
                full[a:b] = got[: b - a]
    assert sizes[rank][1] - sizes[rank][0] == local.shape[0]
    return full


def sharded_matmul(A_local: torch.Tensor, B: torch.Tensor, full_out: Optional[torch.Tensor] = None,
                   group=None, local_out: Optional[torch.Tensor] = None,
                   matmul: Optional[Callable[..., torch.Tensor]] = None) -> torch.Tensor:
    """This rank's rows of C = A @ B, then (if `full_out` is given) C gathered
    into `full_out` on every rank. `matmul` defaults to the sm_100a library
    (functional.matmul); tests pass the oracle on CPU."""
    if matmul is None:
        from .functional import matmul as gpu_matmul

        def matmul(a, b, out=None):
            return gpu_matmul(a, b, out=out)

    C_local = matmul(A_local, B, out=local_out)
    if full_out is not None:
        gather_rows(full_out, C_local, group)
        return full_out
    return C_local
