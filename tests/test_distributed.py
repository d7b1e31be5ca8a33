"""Row-sharded and batch-sharded GEMM + all-gather across ranks, on CPU with
gloo (world size 2 and 3): every rank must end with the full C equal to the
oracle's full product (rows, and the batches of a batched product, are
independent, so the sharded result is bit-identical)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle_bridge as ob
from macrograd_b200.sharded import row_block, sharded_matmul


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _oracle_matmul(a, b, out=None):
    c = torch.from_numpy(ob.oracle_matmul(a.numpy(), b.numpy()))
    if out is not None:
        out.copy_(c)
        return out
    return c


def _worker(rank, world, port, M, K, N, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        A = ob.seeded_uniform((M, K), 4)
        B = ob.seeded_uniform((K, N), 1004)
        r0, r1 = row_block(M, world, rank)
        full = torch.empty(M, N)
        sharded_matmul(torch.from_numpy(A[r0:r1].copy()), torch.from_numpy(B), full_out=full,
                       matmul=_oracle_matmul)
        ref = ob.oracle_matmul(A, B)
        q.put((rank, bool(np.array_equal(full.numpy(), ref))))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _batch_worker(rank, world, port, nb, shared_b, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        A = ob.seeded_uniform((nb, 9, 12), 6)
        B = ob.seeded_uniform((12, 10) if shared_b else (nb, 12, 10), 1006)
        b0, b1 = row_block(nb, world, rank)            # this rank's batches
        B_local = B if shared_b else B[b0:b1].copy()
        full = torch.empty(nb, 9, 10)
        sharded_matmul(torch.from_numpy(A[b0:b1].copy()), torch.from_numpy(B_local), full_out=full,
                       matmul=_oracle_matmul)
        q.put((rank, bool(np.array_equal(full.numpy(), ob.oracle_matmul(A, B)))))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def _spawn(target, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    return results


@pytest.mark.parametrize("world,nb,shared_b", [(2, 6, False), (2, 5, True), (3, 7, False)])
def test_batch_sharded_matmul_gathers_the_oracle_product(world, nb, shared_b):
    """A batched product split by its leading (batch) dim: each rank multiplies
    its batches (B per batch, or one broadcast B) and the slices are gathered
    along that dim."""
    results = _spawn(_batch_worker, world, nb, shared_b)
    assert all(v is True for v in results.values()), results


@pytest.mark.parametrize("world,M", [(2, 64), (2, 67), (3, 50)])
def test_row_sharded_matmul_gathers_the_oracle_product(world, M):
    results = _spawn(_worker, world, M, 48, 40)
    assert all(v is True for v in results.values()), results


def test_row_blocks_partition_the_rows():
    for rows in (1, 7, 64, 8192, 8193):
        for world in (1, 2, 3, 8):
            blocks = [row_block(rows, world, r) for r in range(world)]
            assert blocks[0][0] == 0 and blocks[-1][1] == rows
            assert all(blocks[i][1] == blocks[i + 1][0] for i in range(world - 1))
            sizes = [b - a for a, b in blocks]
            assert max(sizes) - min(sizes) <= 1
