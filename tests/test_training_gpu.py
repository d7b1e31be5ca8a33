"""The decoder training step on "cuda" through the drop-in build: the
reference's modules, autograd, loss and AdamW, with every GEMM of the forward
and backward pass on the sm_100a kernels.

* per GEMM (the configuration's dimensions, one rank's 8 sequences): GEMMs
  captured at the seam during the step are recomputed by the oracle on sampled
  output rows -- 3xTF32 within 1e-5 (Frobenius-normalised);
* whole step (a small model of the same architecture): loss and parameter
  gradients on "cuda" against the reference's own "cpu" step. The loss is
  held to 1e-5. Gradients are compared only downstream of the last GELU: the
  reference's GELU stores Phi(x) for its backward only on the CPU branch
  (tensor_ops.cpp:1374-1382); on "cuda" kernel_ops::gelu
  (cuda_backend.cu:1592-1645) writes the output alone, so GELUOp::_backward
  (tensor_ops.cpp:1347-1352) reads a Phi that was never filled and every
  gradient upstream of a GELU differs from the CPU step whatever the GEMMs
  do. Those GEMMs are covered by the per-GEMM check above;
* data parallel on 2 GPUs (NCCL): the all-reduced gradients of two ranks
  match the one-GPU gradient of the whole batch within 1e-5 (skipped with one
  GPU).
"""
import os
import socket

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
from macrograd_b200 import training  # noqa: E402

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, heads=2, emb=32, ff=64, context=16, vocab=65)


@pytest.fixture(scope="module", autouse=True)
def seam_built():
    if not os.path.exists(training.SEAM):
        pytest.skip("drop-in build not available (needs the reference sources at build time)")


def _rows_of(c, rows, batch_index, fn):
    """op(A) rows `rows` of batch element `batch_index` of a captured GEMM,
    recomputed by the oracle; returns (got, expected)."""
    r = c.out.ndim
    bidx = np.unravel_index(batch_index, c.out.shape[:-2]) if r > 2 else ()

    def pick(x):
        if x is None:
            return None
        idx = tuple(min(i, s - 1) for i, s in zip(bidx, x.shape[:-2]))
        return x[idx]

    A, B, bias = pick(c.A), pick(c.B), pick(c.bias)
    A_rows = A[:, rows] if c.trans_a else A[rows, :]
    bias_rows = None
    if bias is not None:
        bias_rows = bias[rows, :] if bias.shape[0] > 1 else np.broadcast_to(bias, (len(rows), bias.shape[1]))
        bias_rows = np.ascontiguousarray(bias_rows)
    exp = fn(np.ascontiguousarray(A_rows), np.ascontiguousarray(B), c.trans_a, c.trans_b, bias_rows)
    got = pick(c.out)[rows, :]
    return got, exp


def test_every_captured_gemm_of_a_step_matches_the_oracle():
    torch.cuda.set_device(0)
    m = training.DecoderStep(device="cuda", device_index=0)
    try:
        m.make_batch(5, training.BATCH, m.cfg["context"], 0, 8)
        m.observe(1)
        m.forward_backward()
        calls = m.gemm_calls()
        assert calls > 100, calls                      # 6 layers x (6 fwd + 12 bwd) + unembed
        want = list(range(0, 10)) + list(range(calls - 14, calls))
        m.observe(2, want)
        m.forward_backward()
        caps = m.captured()
        m.observe(0)
        assert [c.index for c in caps] == want
        for c in caps:
            M = c.out.shape[-2]
            nb = int(np.prod(c.out.shape[:-2])) if c.out.ndim > 2 else 1
            rows = sorted({0, M // 2, M - 1})
            got, exp = [], []
            for b in sorted({0, nb - 1}):
                g, e = _rows_of(c, rows, b, ob.oracle_matmul)
                got.append(g)
                exp.append(e)
            got, exp = np.concatenate(got), np.concatenate(exp)
            # the causal mask puts -inf into the attention scores: those
            # entries must match exactly, the rest within the tolerance
            fin = np.isfinite(exp)
            assert np.array_equal(got[~fin], exp[~fin]), c.index
            err = ob.frob_rel_err(got[fin], exp[fin])
            assert err <= 1e-5, (c.index, c.out.shape, c.trans_a, c.trans_b, err)
    finally:
        m.close()


def test_small_step_on_gpu_matches_the_reference_cpu_step():
    results = {}
    for dev in ("cpu", "cuda"):
        m = training.DecoderStep(device=dev, device_index=0 if dev == "cuda" else -1, **SMALL)
        try:
            m.make_batch(7, 4, SMALL["context"], 0, 4)
            loss = m.forward_backward()
            results[dev] = (loss, m.host_grads(), m.param_sizes())
        finally:
            m.close()
    (lc, gc, sizes), (lg, gg, _) = results["cpu"], results["cuda"]
    assert abs(lg - lc) <= 1e-5 * abs(lc), (lg, lc)
    # parameters per layer: q, k, v, o (weight, bias), attention norm (2),
    # feed-forward linear0, linear1 (weight, bias), feed-forward norm (2);
    # after the last GELU: the last layer's linear1 and its norm
    per_layer = 16
    last = (SMALL["layers"] - 1) * per_layer
    offs = np.concatenate([[0], np.cumsum(sizes)])
    for i in range(last + 12, last + 16):
        a, b = gc[offs[i]:offs[i + 1]], gg[offs[i]:offs[i + 1]]
        err = np.linalg.norm(b - a) / np.linalg.norm(a)
        assert err <= 1e-5, (i, err)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _dp_worker(rank, world, port, batch, q):
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
        m = training.DecoderStep(device="cuda", device_index=rank)
        first, count = training.shard(batch, world, rank)
        m.make_batch(9, batch, m.cfg["context"], first, count)
        m.forward_backward()
        m.allreduce_grads()
        g = m.host_grads()
        m.close()
        q.put((rank, g))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_two_gpu_data_parallel_gradients_match_one_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    batch = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, 2, port, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(results[r], np.ndarray), f"rank {r}: {results[r]}"
    assert np.array_equal(results[0], results[1])
    torch.cuda.set_device(0)
    m = training.DecoderStep(device="cuda", device_index=0)
    try:
        m.make_batch(9, batch, m.cfg["context"], 0, batch)
        m.forward_backward()
        g = m.host_grads()
    finally:
        m.close()
    err = np.linalg.norm(results[0] - g) / np.linalg.norm(g)
    assert err <= 1e-5, err
