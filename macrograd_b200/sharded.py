"""Row-sharded GEMM across ranks (one process per GPU).

C = A @ B where the rows of A (and so of C) are split over the ranks and B is
replicated -- or, for a batched product, its batches. Rows of C depend only on
the same rows of A (batches only on their own operands), so each rank's GEMM
is independent -- no collective inside the GEMM. When the caller needs the whole C
on every device, the row blocks are all-gathered (NCCL over NVLink on GPUs,
gloo on CPU in the tests), or -- the B200 path -- sent by each rank's GEMM into
every rank's C over NVLink peer mappings while it computes (PeerRows +
scatter_matmul: the kernel's export warps copy each finished tile, or with
MG_GEMM_EXPORT=2 the copy engines send each finished column band), so the
exchange overlaps the math. The reference has no multi-device path; this is
the row-sharded layer its matmul path gains here.
"""
from __future__ import annotations

import ctypes
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
    """All-gather the ranks' blocks of C along its first dim into `full` (every
    rank): row blocks of a 2-D C, or batch blocks of a batched one, split as
    row_block splits that dim."""
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


class PeerRows:
    """Every rank's full-C buffer, mapped into this process (CUDA IPC over
    NVLink), in rank order -- the destinations of the fused all-gather.
    Collective: every rank constructs it with its own `full` buffer."""

    def __init__(self, full: torch.Tensor, group=None):
        from . import _lib

        self._lib = _lib.load()
        self.group = group
        self.full = full
        rank = dist.get_rank(group)
        world = dist.get_world_size(group)
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_uint64(0)
        _lib.check(self._lib.mg_ipc_export(ctypes.c_void_p(full.data_ptr()), handle, ctypes.byref(offset)))
        mine = (bytes(handle.raw), int(offset.value))
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        self.ptrs = []
        self._imported = []
        for r, (h, off) in enumerate(everyone):
            if r == rank:
                self.ptrs.append(full.data_ptr())
                continue
            p = ctypes.c_void_p()
            _lib.check(self._lib.mg_ipc_import(h, off, ctypes.byref(p)))
            self.ptrs.append(p.value)
            self._imported.append(p.value)
        self.array = (ctypes.c_void_p * len(self.ptrs))(*self.ptrs)

    def close(self):
        """Unmap the peers' buffers (after every rank has stopped writing)."""
        for p in self._imported:
            self._lib.mg_ipc_close(ctypes.c_void_p(p))
        self._imported = []


def scatter_matmul(A_local: torch.Tensor, B: torch.Tensor, peers: PeerRows, row0: int,
                   stream: Optional[torch.cuda.Stream] = None) -> None:
    """This rank's rows of C = A @ B, sent into every rank's full C (at rows
    row0 ...) while the GEMM runs (mg_gemm_scatter_rows). A_local [M, K] and
    B [K, N] are contiguous fp32 on this rank's GPU; peers.full is the [rows,
    N] full C. The caller orders it across ranks before C is read."""
    from . import _lib

    full = peers.full
    for name, t in (("A_local", A_local), ("B", B), ("the full C", full)):
        if t.dim() != 2 or t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"scatter_matmul: {name} must be a contiguous 2-D float32 CUDA tensor "
                             f"(got {tuple(t.shape)}, {t.dtype}, {t.device}, contiguous={t.is_contiguous()})")
    if A_local.device != B.device or A_local.device != full.device:
        raise ValueError("scatter_matmul: A_local, B and the full C must be on one device")
    M, K = A_local.shape
    N = B.shape[1]
    if B.shape[0] != K or full.shape[1] != N:
        raise ValueError(f"scatter_matmul: shapes do not chain: A_local {tuple(A_local.shape)}, "
                         f"B {tuple(B.shape)}, full C {tuple(full.shape)}")
    if row0 < 0 or row0 + M > full.shape[0]:
        raise ValueError(f"scatter_matmul: rows [{row0}, {row0 + M}) are outside the {full.shape[0]} rows of C")
    lib = _lib.load()
    d = _lib.GemmDesc()
    lib.mg_gemm_desc_init(ctypes.byref(d), M, N, K, 0, 0)
    d.ldc = full.stride(0)
    if stream is not None and torch.device(stream.device) != A_local.device:
        raise ValueError(f"scatter_matmul: the stream is on {stream.device}, the operands on {A_local.device}")
    s = stream if stream is not None else torch.cuda.current_stream(A_local.device)
    # the library resolves its per-device state (and the K split's resident
    # CTAs) from the current device: make it the operands' one
    with torch.cuda.device(A_local.device):
        _lib.check(lib.mg_gemm_scatter_rows(ctypes.byref(d), ctypes.c_void_p(A_local.data_ptr()),
                                            ctypes.c_void_p(B.data_ptr()), None, peers.array, len(peers.ptrs),
                                            int(row0), int(full.shape[0]), ctypes.c_void_p(s.cuda_stream)))


def sharded_matmul(A_local: torch.Tensor, B: torch.Tensor, full_out: Optional[torch.Tensor] = None,
                   group=None, local_out: Optional[torch.Tensor] = None,
                   matmul: Optional[Callable[..., torch.Tensor]] = None) -> torch.Tensor:
    """This rank's rows of C = A @ B, then (if `full_out` is given) C gathered
    into `full_out` on every rank. For a batched product the same call shards
    the batches instead: A_local holds this rank's batches (row_block over the
    leading dim), B those batches too or one matrix broadcast to all, and the
    slices are gathered along the leading dim. `matmul` defaults to the
    sm_100a library (functional.matmul); tests pass the oracle on CPU."""
    if matmul is None:
        from .functional import matmul as gpu_matmul

        def matmul(a, b, out=None):
            return gpu_matmul(a, b, out=out)

    C_local = matmul(A_local, B, out=local_out)
    if full_out is not None:
        gather_rows(full_out, C_local, group)
        return full_out
    return C_local
