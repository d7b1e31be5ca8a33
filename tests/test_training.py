"""Data-parallel decoder training step on CPU (gloo): the reference's own
modules, autograd, loss and AdamW (the drop-in build's "cpu" path), with the
batch split over 2 ranks and the gradients all-reduced, give the gradient of
the single-process step on the whole batch. Uses a small model of the same
architecture so the reference CPU arithmetic finishes in seconds."""
import os
import socket
import subprocess

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle_bridge as ob
from macrograd_b200 import training

SMALL = dict(layers=2, heads=2, emb=32, ff=64, context=16, vocab=65)
BATCH, T, SEED = 4, 16, 11


def _seam_or_skip():
    if not os.path.exists(training.SEAM):
        # the drop-in build compiles the reference sources; where they are
        # absent it is not built (and the test skips)
        import __graft_entry__

        ref = __graft_entry__.reference_dir()
        if ref is not None:
            subprocess.run(["make", "-s", "-C", os.path.join(ob.ROOT, "macrograd_b200", "shim"), f"REF={ref}"],
                           capture_output=True)
    if not os.path.exists(training.SEAM):
        pytest.skip("drop-in build not available (needs the reference sources at build time)")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _single_process():
    m = training.DecoderStep(device="cpu", **SMALL)
    tok, tgt = m.make_batch(SEED, BATCH, T, 0, BATCH)
    loss = m.forward_backward()
    g = m.host_grads()
    m.close()
    return tok, tgt, loss, g


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        m = training.DecoderStep(device="cpu", **SMALL)
        first, count = training.shard(BATCH, world, rank)
        tok, tgt = m.make_batch(SEED, BATCH, T, first, count)
        loss = m.forward_backward()
        m.allreduce_grads()
        g = m.host_grads()
        p0 = m.host_params()
        m.optimizer_step()
        p1 = m.host_params()
        m.close()
        q.put((rank, (first, tok, tgt, loss, g, p0, p1)))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_batch_shards_cover_the_batch():
    assert [training.shard(64, 8, r) for r in range(8)] == [(8 * r, 8) for r in range(8)]
    assert [training.shard(5, 2, r) for r in range(2)] == [(0, 3), (3, 2)]


def test_data_parallel_step_equals_single_process_step():
    _seam_or_skip()
    tok, tgt, loss, g = _single_process()
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(results[r], tuple), f"rank {r}: {results[r]}"
    losses = []
    for r in range(world):
        first, rtok, rtgt, rloss, rg, p0, p1 = results[r]
        n = rtok.shape[0]
        # the rank's sequences are its share of the single-process batch
        assert np.array_equal(rtok, tok[first:first + n]) and np.array_equal(rtgt, tgt[first:first + n])
        losses.append(rloss)
        # every rank holds the same reduced gradient and takes the same step
        assert np.array_equal(rg, results[0][4])
        assert np.array_equal(p1, results[0][6])
        assert not np.array_equal(p1, p0)
    # mean of the ranks' mean losses (equal shares) = mean loss of the batch;
    # summed / world gradients = gradient of the batch's mean loss. The ranks'
    # GEMMs sum over half the rows each, so fp32 rounding differs slightly.
    assert abs(np.mean(losses) - loss) <= 1e-6 * abs(loss)
    err = np.linalg.norm(results[0][4] - g) / np.linalg.norm(g)
    assert err <= 1e-5, err
