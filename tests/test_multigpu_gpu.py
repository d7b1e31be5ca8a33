"""Row-sharded GEMM across GPUs (one process each, NCCL): every form of the
C-row all-gather leaves the full C on every GPU, matching the oracle on
sampled rows of every rank's block.

test_fused_all_gather_on_two_gpus (n = 1024, 1001 on 2 GPUs): the all-gather
fused into the GEMM kernel in both of its forms -- export warps copying
finished tiles to the peer (default) and the epilogue storing to every rank
itself (MG_GEMM_EXPORT=0) -- in both modes; with the K split forced
(MG_GEMM_SPLIT_MIN_KB=1) the last split level's rows go out through every
CTA's export warps; a 1001-wide C takes the 4-byte copy paths. The NCCL
gather of the same kernel's rows must be bit-identical. The copy-engine form
(MG_GEMM_EXPORT=2: the GEMM in column bands, each band copied to the peer by
cudaMemcpy2DAsync; once forced to 256-column bands, once in the planner's
tapering bands) may split bands along K where one launch does not, so its C
is compared bit for bit with every rank's own rows broadcast over NCCL.

test_row_sharded_gathers_on_2_4_8_gpus: config 4 itself (8192^2, the bench's
row shards, whose last wave is split along K) and an uneven M-tail case
(n = 1001) on 2, 4 and 8 GPUs, each form (export warps, epilogue stores, copy
engines, NCCL) against the oracle on the first and last row of every rank's
256-row m-tiles, and the gathered rows bit-identical on every rank.

Skipped when fewer GPUs than ranks are visible."""
import os
import socket

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, n, q):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        from macrograd_b200 import _lib, load
        from macrograd_b200.sharded import PeerRows, row_block, scatter_matmul, sharded_matmul

        lib = load()
        A = ob.seeded_uniform((n, n // 2), 4)
        B = ob.seeded_uniform((n // 2, n), 1004)
        r0, r1 = row_block(n, world, rank)
        A_local = torch.from_numpy(A[r0:r1].copy()).to(dev)
        Bg = torch.from_numpy(B).to(dev)
        report = {}
        # (mode, export warps, K-split allowed down to this many K-blocks per range)
        for mode, export, min_kb in ((_lib.MG_MODE_TF32X3, "1", "16"), (_lib.MG_MODE_TF32, "1", "16"),
                                     (_lib.MG_MODE_TF32X3, "0", "16"), (_lib.MG_MODE_TF32X3, "1", "1"),
                                     (_lib.MG_MODE_TF32X3, "2", "16"), (_lib.MG_MODE_TF32, "2", "1")):
            lib.mg_set_mode(mode)
            os.environ["MG_GEMM_EXPORT"] = export
            os.environ["MG_GEMM_SPLIT_MIN_KB"] = min_kb
            # copy engines: one case in bands of one 256-wide column, the other in the
            # planner's own tapering bands (two of two columns here, K split to 1 K-block)
            if export == "2" and min_kb == "1":
                os.environ.pop("MG_GEMM_BAND_COLS", None)
            else:
                os.environ["MG_GEMM_BAND_COLS"] = "1"
            full = torch.full((n, n), float("nan"), device=dev)
            peers = PeerRows(full)
            for _ in range(2):                       # two calls in a row into the same buffers
                scatter_matmul(A_local, Bg, peers, r0)
                fence = torch.zeros(1, device=dev)
                dist.all_reduce(fence)                # every rank's kernel (and its remote rows) done
            torch.cuda.synchronize()
            got = full.cpu().numpy()
            if export == "2":
                same = True
                for src in range(world):   # the rows each rank computed, as it holds them
                    s0, s1 = row_block(n, world, src)
                    own = full[s0:s1].clone()
                    dist.broadcast(own, src)
                    same = same and bool(torch.equal(own, full[s0:s1]))
            else:
                full_nccl = torch.empty((n, n), device=dev)
                sharded_matmul(A_local, Bg, full_out=full_nccl)
                torch.cuda.synchronize()
                same = bool(np.array_equal(got, full_nccl.cpu().numpy()))
            rows = [0, 5, n // 2 - 1, n // 2, n // 2 + 7, n - 1]
            ref = ob.oracle_matmul(A[rows], B)
            tol = 1e-5 if mode == _lib.MG_MODE_TF32X3 else 2e-3
            report[(mode, export, min_kb)] = (bool(np.all(np.isfinite(got))), ob.frob_rel_err(got[rows], ref) <= tol,
                                              same)
            dist.barrier()
            peers.close()
        q.put((rank, report))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("n", [1024, 1001])
def test_fused_all_gather_on_two_gpus(n):
    _run(_worker, 2, n)


def _run(target, world, n):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = dict(q.get(timeout=600) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, rep in results.items():
        assert isinstance(rep, dict), f"rank {rank}: {rep}"
        for key, val in rep.items():
            if key == "errors":
                print(f"rank {rank} frobenius errors against the oracle: {val}")
                continue
            finite, close, same = val
            what = f"rank {rank} {key}"
            assert finite, f"{what}: C has rows nobody wrote"
            assert close, f"{what}: rows differ from the oracle"
            assert same, f"{what}: gathered rows differ from the rows their rank computed"
    return results


def _sample_rows(n, world):
    """Every rank's first and last row and the first and last row of each of
    its 256-row (SM pair) m-tiles: full rows, so every column tile -- the last
    K-split level's included -- is compared."""
    from macrograd_b200.sharded import row_block

    rows = set()
    for r in range(world):
        r0, r1 = row_block(n, world, r)
        for m in range(r0, r1, 256):
            rows.update({m, min(m + 255, r1 - 1)})
        rows.update({r0, r1 - 1})
    return sorted(rows)


def _worker_sizes(rank, world, port, n, q):
    """A[n, n] @ B[n, n] row-sharded over `world` ranks (config 4 at n = 8192,
    seeds of the single-GPU config-4 test), gathered by each form in turn."""
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from macrograd_b200 import _lib, load
        from macrograd_b200.sharded import PeerRows, row_block, scatter_matmul, sharded_matmul

        lib = load()
        lib.mg_set_mode(_lib.MG_MODE_TF32X3)
        r0, r1 = row_block(n, world, rank)
        A_local = torch.from_numpy(ob.seeded_uniform((n, n), 4)[r0:r1].copy()).to(dev)
        Bh = ob.seeded_uniform((n, n), 1004)
        Bg = torch.from_numpy(Bh).to(dev)
        rows = _sample_rows(n, world)
        ref = None
        if rank == 0:
            A = ob.seeded_uniform((n, n), 4)
            ref = ob.oracle_matmul(A[rows], Bh)
        report, errors = {}, {}
        for form in ("export", "epilogue", "copy-engines", "nccl"):
            full = torch.full((n, n), float("nan"), device=dev)
            peers = None
            if form == "nccl":
                C_local = torch.empty((r1 - r0, n), device=dev)
                sharded_matmul(A_local, Bg, full_out=full, local_out=C_local)
            else:
                os.environ["MG_GEMM_EXPORT"] = {"export": "1", "epilogue": "0", "copy-engines": "2"}[form]
                peers = PeerRows(full)
                scatter_matmul(A_local, Bg, peers, r0)
                fence = torch.zeros(1, device=dev)
                dist.all_reduce(fence)                # every rank's kernel (and its remote rows) done
            torch.cuda.synchronize()
            finite = bool(torch.isfinite(full).all())
            # the rows each rank computed, as it holds them, reach every rank unchanged
            same = True
            for src in range(world):
                s0, s1 = row_block(n, world, src)
                own = full[s0:s1].clone()
                dist.broadcast(own, src)
                same = same and bool(torch.equal(own, full[s0:s1]))
            picked = full[rows].contiguous()
            first = picked.clone()
            dist.broadcast(first, 0)
            same = same and bool(torch.equal(first, picked))
            close = True
            if rank == 0:
                e = ob.frob_rel_err(picked.cpu().numpy(), ref)
                errors[form] = float(e)
                close = e <= 1e-5
            report[(n, world, form)] = (finite, close, same)
            dist.barrier()
            if peers is not None:
                peers.close()
            os.environ.pop("MG_GEMM_EXPORT", None)
        if rank == 0:
            report["errors"] = errors
        q.put((rank, report))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("n", [8192, 1001])
def test_row_sharded_gathers_on_2_4_8_gpus(world, n):
    """Config 4 (n = 8192: the bench's row shards, the last wave split along
    K) and an M-tail case (n = 1001: uneven row blocks, 4-byte copies) on 2, 4
    and 8 GPUs, each gather form against the oracle (3xTF32, 1e-5)."""
    _run(_worker_sizes, world, n)
