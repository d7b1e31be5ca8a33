"""Benchmark: fp32-accurate matmul TFLOP/s on B200 (square 8192^3 GEMM).

Workload: C = A @ B, A and B [8192, 8192] fp32 ~ U(-1, 1). The rows of A (and
so of C) are split across the N ranks (one process per GPU), B is replicated,
and when N > 1 every GPU ends the step holding all of C: by default the GEMM
kernel copies each finished tile into every GPU's C over NVLink (the
all-gather fused into the kernel); --gather ce computes the rows in column
bands and has the copy engines send each finished band beside the next one's
GEMM; --gather nccl uses an NCCL all-gather after the GEMM.
Work is fixed as N grows ("strong" scaling). Default mode 3xTF32
(fp32-accurate); --mode tf32 times the fast mode.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--mode 3xtf32|tf32]
    python -m torch.distributed.run --nproc-per-node N bench.py --gpus N ...
    python bench.py --impl reference ...   # the reference's CPU matmul, host cores

Prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
SIZE = 8192
METRIC = "fp32-accurate matmul TFLOP/s & % TF32 roofline at 1/2/4/8 B200 vs host CPU"
UNIT = "TFLOP/s"
def workload(n):
    return f"square fp32 GEMM {n}x{n}x{n}, rows of A sharded over the GPUs, C rows all-gathered"

# DRAM bytes (read + write) of one 8192^3 launch of the GEMM kernel, measured
# with ncu (dram__bytes_read.sum + dram__bytes_write.sum of the 3xTF32 launch;
# null where not captured).
NCU_TRAFFIC_BYTES_PER_LAUNCH = {"3xtf32": 2566900992 + 255566848, "tf32": None}


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--mode", choices=["3xtf32", "tf32"], default="3xtf32")
    p.add_argument("--size", type=int, default=SIZE)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="N=1: skip the sub-records (the 8192^3 GEMM in the other mode, and the batched, "
                        "linear-layer and attention workloads)")
    p.add_argument("--workload", choices=["gemm", "decoder", "batched", "linear", "attention"], default="gemm",
                   help="gemm: the square 8192^3 GEMM (default); decoder: the decoder-only character "
                        "model's training step through the drop-in build, batch-sharded over the GPUs; "
                        "batched / linear / attention: the one-GPU forward + backward GEMM workloads "
                        "(batched A[8,256,384] @ W[384,384]; linear layer X[16384,384] @ W[1536,384]^T + b; "
                        "causal attention Q, K, V [64,6,256,64] with the softmax fused)")
    p.add_argument("--gather", choices=["fused", "ce", "nccl"], default="fused",
                   help="N>1: C rows reach every GPU from the GEMM kernel over NVLink (fused), by the "
                        "copy engines band by band beside the GEMM (ce), or by an NCCL all-gather after it")
    return p.parse_args()


GATHER_NAMES = {"fused": " + all-gather fused into the GEMM kernel (NVLink peer stores)",
                "ce": " + all-gather by the copy engines, column band by band beside the GEMM",
                "nccl": " + NCCL all-gather"}


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), \
            float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# ------------------------------------------------------------------ CPU side
def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:  # pragma: no cover
        return os.cpu_count() or 1


def reference_cpu_sample(n, rows_per_core, cores, seed=4):
    """Times the reference's own CPU matmul (oracle/_ref, compiled from the
    reference sources) on `cores` processes, each multiplying its own
    rows_per_core rows of A by the full B. Falls back to the C restatement
    (one thread) when the reference build is absent. Returns (tflops, kind,
    cores_used, seconds, rows)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_bridge as ob
    rows = rows_per_core * cores
    A = ob.seeded_uniform((rows, n), seed)
    B = ob.seeded_uniform((n, n), seed + 1000)
    C = np.empty((rows, n), np.float32)
    if ob.ref_available():
        lib = ob.ref()
        t0 = time.perf_counter()
        rc = lib.ref_matmul_rows_mp(ob._ptr(C), ob._ptr(A), ob._ptr(B), rows, n, n, cores)
        dt = time.perf_counter() - t0
        if rc != 0:
            raise RuntimeError(f"reference row-sliced matmul failed ({rc})")
        kind, used = "reference", cores
    else:
        rows = rows_per_core
        t0 = time.perf_counter()
        C = ob.oracle_matmul(A[:rows], B)
        dt = time.perf_counter() - t0
        kind, used = "port", 1
    flops = 2.0 * rows * n * n
    return flops / dt / 1e12, kind, used, dt, rows


def run_reference_arm(args):
    rank, _, world = env_rank()
    if rank != 0:
        return 0
    n = args.size
    cores = cpu_cores()
    rows_per_core = 8
    vals = []
    kind = "reference"
    used = cores
    rows = rows_per_core * cores
    for i in range(args.warmup + args.steps):
        v, kind, used, dt, rows = reference_cpu_sample(n, rows_per_core, cores, seed=4 + i)
        if i >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    sample = (f"{rows} rows of A x full B[{n},{n}] per step ({rows_per_core} rows per process, "
              f"{used} processes), the reference's Functional::matmul CPU loop")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (reference CPU RNG, U(-1,1))",
        "config": {"workload": workload(n), "size": n, "mode": "fp32 (reference CPU loop)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": used, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ GPU side
def main():
    args = parse_args()
    if args.workload == "decoder":
        return run_decoder(args)
    if args.workload in ("batched", "linear", "attention"):
        return run_small_workload(args)
    if args.impl == "reference":
        return run_reference_arm(args)

    rank, local_rank, world = env_rank()
    if world != args.gpus:
        print(f"--gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
        return 2
    n = args.size
    if n % world != 0:
        print("size must divide evenly over the ranks", file=sys.stderr)
        return 2

    # CPU baselines first, before any CUDA call in this process (the
    # reference's row-sliced matmul forks worker processes).
    cpu = None
    small_cpu = {}
    one_gpu_extras = world == 1 and n == SIZE and not args.no_extras
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = cpu_cores()
        v, kind, used, dt, rows = reference_cpu_sample(n, 8, cores)
        cpu = {"value": v, "unit": UNIT, "cores": used, "kind": kind,
               "sample": f"{rows} rows of A x full B[{n},{n}] ({2.0 * rows * n * n / 1e9:.1f} GFLOP) "
                         f"in {dt:.2f} s over {used} processes"}
        if one_gpu_extras:
            for w in ("batched", "linear", "attention"):
                small_cpu[w] = small_reference_rate(w, 2, 1)

    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    import macrograd_b200 as mg
    from macrograd_b200 import _lib
    from macrograd_b200.sharded import PeerRows, gather_rows, row_block, scatter_matmul, sharded_matmul

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    lib = mg.load()
    mode = _lib.MG_MODE_TF32X3 if args.mode == "3xtf32" else _lib.MG_MODE_TF32
    _lib.check(lib.mg_set_mode(mode))

    r0, r1 = row_block(n, world, rank)
    rows = r1 - r0
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    A = torch.empty(rows, n, device=dev).uniform_(-1, 1, generator=g)
    g.manual_seed(4321)
    B = torch.empty(n, n, device=dev).uniform_(-1, 1, generator=g)
    C_local = torch.empty(rows, n, device=dev)
    C_full = torch.empty(n, n, device=dev) if world > 1 else C_local
    stream = torch.cuda.current_stream(dev)
    fused = world > 1 and args.gather in ("fused", "ce")
    if fused:
        # the library reads its export switch at every call
        os.environ["MG_GEMM_EXPORT"] = "2" if args.gather == "ce" else os.environ.get("MG_GEMM_EXPORT", "1")
    peers = PeerRows(C_full) if fused else None
    fence = torch.zeros(1, device=dev)

    def gemm():
        if fused:
            scatter_matmul(A, B, peers, r0)               # rows into every GPU's C while the GEMM runs
        else:
            sharded_matmul(A, B, local_out=C_local)       # this rank's rows (one GEMM launch)

    def exchange():
        if fused:
            dist.all_reduce(fence)                        # every rank's rows have landed
        elif world > 1:
            gather_rows(C_full, C_local)                  # C rows to every GPU (NCCL)

    def step():
        gemm()
        exchange()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, device-timed with events on the launching stream
    clocks = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    launches0 = lib.mg_launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    kern_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    ev0.record(stream)
    for i in range(args.steps):
        kern_ev[i][0].record(stream)
        gemm()
        kern_ev[i][1].record(stream)
        exchange()
        kern_ev[i][2].record(stream)
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = lib.mg_launch_count() - launches0
    clk = clocks.stop()
    elapsed_ms = ev0.elapsed_time(ev1)
    kern_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in kern_ev)
    gather_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in kern_ev)

    t = torch.tensor([elapsed_ms, kern_ms, gather_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    elapsed_ms, kern_ms, gather_ms = float(t[0]), float(t[1]), float(t[2])
    ms_per_step = elapsed_ms / args.steps
    flops = 2.0 * n * n * n
    value = flops / (ms_per_step * 1e-3) / 1e12

    # ---- end to end through the public API from pinned host memory
    # Every step copies its A rows in from pinned host memory, runs the GEMM
    # (and the all-gather) and copies its C rows back out; consecutive steps
    # are pipelined on three streams with double buffers (copy-in of step i+1
    # and copy-out of step i-1 run while step i computes), the way a stream of
    # GEMMs on host data would be driven.
    e2e = None
    if not args.no_e2e:
        A_h = A.cpu().pin_memory()
        C_h = torch.empty(rows, n, dtype=torch.float32).pin_memory()
        A_d = [torch.empty_like(A) for _ in range(2)]
        if fused:
            C_e = [C_full] + [torch.empty(n, n, device=dev)]
            peers_e = [peers, PeerRows(C_e[1])]
        elif world > 1:
            C_e = [C_full, torch.empty(n, n, device=dev)]
        else:
            C_e = [C_local, torch.empty(rows, n, device=dev)]
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in", "comp", "out")}
        used = [False, False]

        def e2e_step(i):
            b = i % 2
            if used[b]:
                s_in.wait_event(ev["comp"][b])          # the GEMM that read A_d[b] is done
            with torch.cuda.stream(s_in):
                A_d[b].copy_(A_h, non_blocking=True)
                ev["in"][b].record(s_in)
            stream.wait_event(ev["in"][b])
            if used[b]:
                stream.wait_event(ev["out"][b])         # C[b]'s previous rows are on the host
            if fused:
                scatter_matmul(A_d[b], B, peers_e[b], r0)
                dist.all_reduce(fence)
                src = C_e[b][r0:r1]
            elif world > 1:
                sharded_matmul(A_d[b], B, full_out=C_e[b], local_out=C_local)
                src = C_e[b][r0:r1]
            else:
                sharded_matmul(A_d[b], B, local_out=C_e[b])
                src = C_e[b]
            ev["comp"][b].record(stream)
            s_out.wait_event(ev["comp"][b])
            with torch.cuda.stream(s_out):
                C_h.copy_(src, non_blocking=True)
                ev["out"][b].record(s_out)
            used[b] = True

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_event(e0)
        for i in range(args.steps):
            e2e_step(i)
        stream.wait_stream(s_out)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        te = torch.tensor([e0.elapsed_time(e1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e_ms = float(te[0]) / args.steps
        e2e = {"value": flops / (e_ms * 1e-3) / 1e12, "unit": UNIT,
               "h2d_bytes_per_step": int(A_h.numel() * 4 * world),
               "d2h_bytes_per_step": int(C_h.numel() * 4 * world),
               "ms_per_step": e_ms,
               "note": "per step: A row shard host->device (pinned), GEMM, all-gather, own C rows "
                       "device->host; B resident like weights; steps pipelined on three streams "
                       "(double-buffered A and C)"}
        if fused:
            dist.barrier(device_ids=[local_rank])
            peers_e[1].close()

    # ---- N = 1 sub-records: the same GEMM in the other mode (kernel time),
    # and the other configurations' workloads (measure_small)
    extras = None
    if one_gpu_extras and rank == 0:
        other = "tf32" if args.mode == "3xtf32" else "3xtf32"
        _lib.check(lib.mg_set_mode(_lib.MG_MODE_TF32 if other == "tf32" else _lib.MG_MODE_TF32X3))
        for _ in range(max(3, args.warmup)):
            gemm()
        torch.cuda.synchronize()
        kev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
        oclk = ClockSampler(local_rank)
        oclk.start()
        for i in range(args.steps):
            kev[i][0].record(stream)
            gemm()
            kev[i][1].record(stream)
        torch.cuda.synchronize()
        oclk_rec = oclk.stop()
        o_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in kev)
        bf16_, _, _, src_ = peaks()
        o_peak = bf16_ / 2.0 / (3.0 if other == "3xtf32" else 1.0)
        o_tf = 2.0 * n * n * n / (o_ms * 1e-3) / 1e12
        extras = {other: {"value": o_tf, "unit": UNIT, "ms": o_ms, "mode": other,
                          "roofline": {"bound": "tensor", "achieved": o_tf, "peak": o_peak, "unit": UNIT,
                                       "frac": o_tf / o_peak,
                                       "peak_source": f"{src_} bf16 dense {bf16_:.1f} / 2"
                                                      + (" / 3" if other == "3xtf32" else "")},
                          "note": "the same 8192^3 GEMM in the other mode, kernel time (CUDA events), "
                                  "operands resident, larger than L2", "clocks": oclk_rec}}
        _lib.check(lib.mg_set_mode(mode))
        del A, B, C_local, C_full
        torch.cuda.empty_cache()
        extras["workloads"] = {w: measure_small(w, args.mode, args.steps, args.warmup, dev, lib, small_cpu.get(w))
                               for w in ("batched", "linear", "attention")}

    if world > 1:
        dist.barrier(device_ids=[local_rank])             # no rank still writes into a peer's C
        if peers is not None:
            peers.close()
        dist.destroy_process_group()
    if rank != 0:
        return 0

    bf16, bf16_sus, hbm, src = peaks()
    tf32_peak = bf16 / 2.0
    peak = tf32_peak / 3.0 if args.mode == "3xtf32" else tf32_peak
    per_launch_flops = 2.0 * rows * n * n
    achieved = per_launch_flops / (kern_ms * 1e-3) / 1e12
    # captured for the one-GPU 8192^3 launch only; a row shard's launch has
    # its own L2 reuse, so other shapes report none rather than a scaled guess
    traffic = NCU_TRAFFIC_BYTES_PER_LAUNCH.get(args.mode) if (world == 1 and n == SIZE) else None
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic U(-1,1) (torch generator, seeded), resident in HBM",
        "config": {"workload": workload(n), "size": n, "rows_per_gpu": rows,
                   "mode": args.mode,
                   "parallelism": f"row-shard x{world}" + (GATHER_NAMES[args.gather] if world > 1 else ""),
                   "l2": (f"operands 2 x {n * n * 4 / 1e6:.0f} MB, output {n * n * 4 / 1e6:.0f} MB: "
                          + ("each larger than the 126 MB L2" if n * n * 4 > 126e6
                             else "smaller than the 126 MB L2 and not flushed (not a contract measurement)"))},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": UNIT,
                     "frac": achieved / peak, "traffic": traffic,
                     "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one 8192^3 launch "
                                        "(profiles/dram_mg_gemm_tc_kernel_8192.md)" if traffic is not None
                                        else "not captured for this shape"),
                     "peak_source": (f"{src} bf16 dense {bf16:.1f} TFLOP/s / 2 = TF32 {tf32_peak:.1f}"
                                     + (" / 3 products per fp32-accurate term" if args.mode == "3xtf32" else "")),
                     "kernel": "mg_gemm_tc_kernel", "kernel_ms": kern_ms},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": int(launches),
        "gemm_only": {"value": flops / (kern_ms * 1e-3) / 1e12, "unit": UNIT, "ms": kern_ms,
                      "note": "max over ranks of the per-rank GEMM time; the step adds the exchange "
                              "(the fence of the fused all-gather, or the NCCL all-gather)"},
        "exchange_ms": gather_ms if world > 1 else 0.0,
        "clocks": clk,
    }
    if extras is not None:
        line["other_mode"] = extras.pop("tf32" if args.mode == "3xtf32" else "3xtf32")
        line["workloads"] = extras["workloads"]
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ small workloads
SMALL = {
    "batched": (3 * 2.0 * 8 * 256 * 384 * 384,
                {"workload": "batched fp32 matmul A[8,256,384] @ W[384,384], backward with dC = ones",
                 "gemms": "C = A W; dA = dC W^T; dW = A^T dC (batch folded into K = 2048)"}),
    "linear": (3 * 2.0 * 16384 * 1536 * 384,
               {"workload": "linear layer X[16384,384] @ W[1536,384]^T + b[1536], backward with dY ~ N(0,1)",
                "gemms": "Y = X W^T + b (bias fused); dX = dY W; dW = dY^T X (transposed views in place)"}),
    "attention": (6 * 2.0 * 64 * 6 * 256 * 256 * 64,
                  {"workload": "causal attention Q, K, V [64,6,256,64]: P = softmax(Q K^T / 8 + causal) fused, "
                               "O = P V, backward with dO = ones",
                   "gemms": "P (score product + mask + row softmax in the epilogue), O = P V, "
                            "dS = P (dP - rowsum(P dP)) with dP = dO V^T (softmax backward in the epilogue), "
                            "dV = P^T dO, dQ/8 = dS K, dK = dS^T (Q/8): 6 products, 6 launches"}),
}


def small_desc(workload):
    flops, desc = SMALL[workload]
    return flops, dict(desc)


def small_reference_rate(workload, steps, warmup):
    """A one-GPU workload's step through the reference's own CPU
    Functional::matmul and autograd backward (oracle/_ref, built from the
    reference sources; the C restatement when that build is absent), on a
    bounded sample of the step (a slice of its rows or sequences), one core --
    the reference's CPU path is single-threaded. Returns the cpu_baseline
    record: GEMM TFLOP/s over the sample (median of `steps` after `warmup`)."""
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_bridge as ob
    use_ref = ob.ref_available()
    kind = "reference" if use_ref else "port"

    def fwd_bwd(A, B, dC, transB=False, bias=None):   # forward + the backward's two GEMMs
        if use_ref:
            ob.ref_matmul_backward(A, B, dC, False, transB, bias)
        else:
            ob.oracle_matmul(A, B, False, transB, bias)
            ob.oracle_matmul_backward(A, B, dC, False, transB, None if bias is None else bias.shape)

    mm = ob.ref_matmul if use_ref else ob.oracle_matmul
    if workload == "batched":
        A, W = ob.seeded_uniform((8, 256, 384), 20), ob.seeded_uniform((384, 384), 21)
        dC = np.ones((8, 256, 384), np.float32)
        flops, sample = SMALL["batched"][0], "the whole step"

        def step():
            t0 = time.perf_counter()
            fwd_bwd(A, W, dC)
            return time.perf_counter() - t0
    elif workload == "linear":
        rows = 1024
        bound = (6.0 / 384) ** 0.5
        X = ob.seeded_uniform((rows, 384), 22)
        W, b = ob.seeded_uniform((1536, 384), 23, -bound, bound), ob.seeded_uniform((1536,), 24, -bound, bound)
        dY = ob.seeded_normal((rows, 1536), 25)
        flops, sample = 3 * 2.0 * rows * 1536 * 384, f"{rows} of the 16384 rows of X (and dY)"

        def step():
            t0 = time.perf_counter()
            fwd_bwd(X, W, dY, True, b)
            return time.perf_counter() - t0
    else:
        nb = 4
        Q = ob.seeded_normal((nb, 6, 256, 64), 26, 0.0, 0.125)
        K = ob.seeded_normal((nb, 6, 256, 64), 27, 0.0, 0.125)
        V = ob.seeded_normal((nb, 6, 256, 64), 28)
        dO = np.ones_like(V)
        Qs = Q * np.float32(0.125)
        mask = ob.oracle_causal_mask(256)
        flops = 6 * 2.0 * nb * 6 * 256 * 256 * 64
        sample = (f"{nb} of the 64 sequences; the Q K^T product that the last forward + backward call "
                  f"recomputes is subtracted (its time taken from the step's first product)")

        def step():
            t0 = time.perf_counter()
            S = mm(Qs, K, False, True, mask)                        # scores + mask
            t_qk = time.perf_counter() - t0
            P = ob.ref_softmax_rows(S) if use_ref else ob.oracle_softmax_rows(S)
            if use_ref:
                dP, _, _ = ob.ref_matmul_backward(P, V, dO)         # O = P V; dP = dO V^T, dV = P^T dO
            else:
                mm(P, V)
                dP = mm(dO, V, False, True)
                mm(P, dO, True, False)
            dS = P * (dP - (P * dP).sum(-1, keepdims=True))         # SoftOp::_backward
            fwd_bwd(Qs, K, dS, True)                                 # dQ/8, dK, after Q K^T again
            return time.perf_counter() - t0 - t_qk                  # less the repeated Q K^T
    vals = []
    for i in range(max(1, warmup) + max(1, steps)):
        dt = step()
        if i >= max(1, warmup):
            vals.append(flops / dt / 1e12)
    return {"value": statistics.median(vals), "unit": "TFLOP/s", "cores": 1, "kind": kind,
            "sample": f"{sample}: {flops / 1e9:.2f} GFLOP per step"}


def run_small_reference(args):
    """--impl reference for the one-GPU GEMM workloads (small_reference_rate)."""
    rank, _, _ = env_rank()
    if rank != 0:
        return 0
    full_flops, desc = small_desc(args.workload)
    cpu = small_reference_rate(args.workload, args.steps, args.warmup)
    value = cpu["value"]
    print(json.dumps({
        "impl": "reference", "metric": f"{args.workload} fwd+bwd GEMM TFLOP/s", "value": value,
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (reference CPU RNG)",
        "config": {**desc, "mode": "fp32 (reference CPU loop)", "gflop_per_step": full_flops / 1e9},
        "cpu_baseline": cpu,
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)
    return 0


def small_step_calls(workload, dev):
    """The library calls of one forward + backward step of a one-GPU workload
    (every GEMM through the public API, functional.py), on seeded synthetic
    inputs resident in HBM: (flops, config, [(name, fn)]) -- each fn makes
    one library call and returns its output."""
    import torch
    from macrograd_b200 import functional as F

    g = torch.Generator(device=dev)
    g.manual_seed(20)
    flops, desc = small_desc(workload)
    if workload == "batched":
        A = torch.empty(8, 256, 384, device=dev).uniform_(-1, 1, generator=g)
        W = torch.empty(384, 384, device=dev).uniform_(-1, 1, generator=g)
        dC = torch.ones(8, 256, 384, device=dev)
        calls = [("C = A W", lambda: F.matmul(A, W)),
                 ("dA, dW", lambda: F.matmul_backward(A, W, dC))]
    elif workload == "linear":
        bound = (6.0 / 384) ** 0.5
        X = torch.empty(16384, 384, device=dev).uniform_(-1, 1, generator=g)
        W = torch.empty(1536, 384, device=dev).uniform_(-bound, bound, generator=g)
        b = torch.empty(1536, device=dev).uniform_(-bound, bound, generator=g)
        dY = torch.empty(16384, 1536, device=dev).normal_(0, 1, generator=g)
        calls = [("Y = X W^T + b", lambda: F.matmul(X, W, b, False, True)),
                 ("dX, dW, db", lambda: F.matmul_backward(X, W, dY, False, True, True, (1536,)))]
    else:
        Q = torch.empty(64, 6, 256, 64, device=dev).normal_(0, 0.125, generator=g)
        K = torch.empty(64, 6, 256, 64, device=dev).normal_(0, 0.125, generator=g)
        V = torch.empty(64, 6, 256, 64, device=dev).normal_(0, 1, generator=g)
        dO = torch.ones(64, 6, 256, 64, device=dev)
        Qs = Q * 0.125
        st = {}
        calls = [("P = softmax(Q K^T / 8 + causal)", lambda: st.__setitem__("P", F.attention_scores(Q, K, 0.125, True))),
                 ("O = P V", lambda: F.matmul(st["P"], V)),
                 ("dS = P (dP - rowsum(P dP)), dP = dO V^T",
                  lambda: st.__setitem__("dS", F.attention_softmax_backward(dO, V, st["P"]))),
                 ("dV = P^T dO", lambda: F.matmul(st["P"], dO, None, True, False)),
                 ("dQ/8 = dS K", lambda: F.matmul(st["dS"], K)),
                 ("dK = dS^T Q/8", lambda: F.matmul(st["dS"], Qs, None, True, False))]
    return flops, desc, calls


def measure_small(workload, mode, steps, warmup, dev, lib, cpu=None):
    """Times one workload's step on this GPU. Every library call is captured
    in a CUDA graph of its own (the launch-bound small calls pay no host
    overhead) and the graphs are replayed back to back between CUDA events on
    the launching stream, L2 flushed before every step (a 512 MB write,
    untimed): per-call device times, their sum the step's GEMM time. The same
    step run eagerly through the Python API is timed beside it. Returns the
    workload's record (TFLOP/s against TF32 / 3 or TF32; HBM rate of the
    attention score product and of its fused softmax backward)."""
    import torch
    from macrograd_b200 import _lib

    _lib.check(lib.mg_set_mode(_lib.MG_MODE_TF32X3 if mode == "3xtf32" else _lib.MG_MODE_TF32))
    flops, desc, calls = small_step_calls(workload, dev)
    flush = torch.empty(128 * 1024 * 1024, device=dev)
    for _ in range(max(3, warmup)):
        for _, fn in calls:
            fn()
    torch.cuda.synchronize()
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    graphs = []
    for _, fn in calls:
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=side):
            fn()
        graphs.append(gr)
    torch.cuda.synchronize()
    for gr in graphs:
        gr.replay()
    torch.cuda.synchronize()
    launches0 = lib.mg_launch_count()
    clocks = ClockSampler(dev.index or 0)
    clocks.start()
    each_ms = []
    for _ in range(steps):
        flush.fill_(1.0)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(len(graphs) + 1)]
        ev[0].record()
        for i, gr in enumerate(graphs):
            gr.replay()
            ev[i + 1].record()
        torch.cuda.synchronize()
        each_ms.append([ev[i].elapsed_time(ev[i + 1]) for i in range(len(graphs))])
    eager_ms = []
    for _ in range(steps):
        flush.fill_(1.0)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _, fn in calls:
            fn()
        e1.record()
        torch.cuda.synchronize()
        eager_ms.append(e0.elapsed_time(e1))
    clk = clocks.stop()
    # graph replays make no library call: the eager steps give the kernels per step
    launches = (lib.mg_launch_count() - launches0) // max(1, steps)
    per_call = [statistics.mean(x) for x in zip(*each_ms)]
    gms = sum(per_call)
    bf16, _, hbm, src = peaks()
    peak = bf16 / 2.0 / (3.0 if mode == "3xtf32" else 1.0)
    tf = flops / (gms * 1e-3) / 1e12
    rec = {
        "metric": f"{workload} fwd+bwd GEMM TFLOP/s", "value": tf, "unit": "TFLOP/s", "mode": mode,
        "gemm_ms_per_step": gms, "eager_ms_per_step": statistics.mean(eager_ms),
        "config": {**desc, "mode": mode, "gflop_per_step": flops / 1e9,
                   "l2": "flushed before every step (512 MB write, untimed)",
                   "timing": "each library call captured in its own CUDA graph, replayed back to back between "
                             "CUDA events (device time); eager_ms_per_step: the same step through the Python API"},
        "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                     "peak_source": f"{src} bf16 dense {bf16:.1f} / 2" + (" / 3" if mode == "3xtf32" else "")},
        "per_call_ms": dict(zip([n for n, _ in calls], per_call)),
        "gpu_launches_per_step": int(launches),
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    if workload == "attention":
        L, nbh = 256, 64 * 6
        sbytes = 4.0 * nbh * (2 * L * 64 + L * L)            # Q, K read; P written
        bbytes = 4.0 * nbh * (2 * L * 64 + 2 * L * L)        # dO, V, P read; dS written
        for key, i, b, what in (("score_product", 0, sbytes, "Q, K read + P written, one fused launch"),
                                ("softmax_backward", 2, bbytes, "dO, V, P read + dS written, one fused launch")):
            ms = per_call[i]
            rec[key] = {"bound": "hbm", "ms": ms, "achieved": b / (ms * 1e-3) / 1e9, "peak": hbm, "unit": "GB/s",
                        "frac": b / (ms * 1e-3) / 1e9 / hbm, "bytes": b, "note": what}
    del graphs
    torch.cuda.synchronize()
    return rec


def run_small_workload(args):
    """One-GPU forward + backward GEMM workloads of the matmul path (the
    parity configurations, timed) as their own JSON line: measure_small."""
    if args.impl == "reference":
        return run_small_reference(args)
    rank, local_rank, world = env_rank()
    if world != 1:
        print("the small workloads run on one GPU", file=sys.stderr)
        return 2
    cpu = None if args.no_cpu_baseline else small_reference_rate(args.workload, 3, 1)   # before any CUDA call
    import torch

    sys.path.insert(0, ROOT)
    import macrograd_b200 as mg

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    lib = mg.load()
    rec = measure_small(args.workload, args.mode, args.steps, args.warmup, dev, lib, cpu)
    line = {"metric": rec.pop("metric"), "value": rec.pop("value"), "unit": rec.pop("unit"), "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": rec["gemm_ms_per_step"],
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (torch generator, seeded), resident in HBM", **rec}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ decoder step
DECODER_METRIC = "decoder training step tokens/s (6 layers, d_model 384, batch 64 x 256 tokens)"


def decoder_reference_rate(T, steps, warmup):
    """The reference's own CPU training step (its modules, autograd and AdamW
    through the drop-in build on "cpu") on one of the batch's sequences, one
    core (the reference's CPU path is single-threaded): the cpu_baseline
    record, tokens/s, median of `steps` after `warmup`."""
    from macrograd_b200 import training

    m = training.DecoderStep(device="cpu")
    try:
        m.make_batch(5, training.BATCH, T, 0, 1)
        vals = []
        for i in range(max(1, warmup) + max(1, steps)):
            t0 = time.perf_counter()
            m.forward_backward()
            m.optimizer_step()
            dt = time.perf_counter() - t0
            if i >= max(1, warmup):
                vals.append(T / dt)
    finally:
        m.close()
    return {"value": statistics.median(vals), "unit": "tokens/s", "cores": 1, "kind": "reference",
            "sample": f"1 sequence of {T} tokens per step (full model, forward + backward + AdamW), 1 core"}


def run_decoder(args):
    """The decoder-only character model's training step (6 layers, 6 heads,
    d_model 384, MLP 1536, context 256, vocab 65, batch 64), built from the
    reference's own modules through the drop-in build: forward, cross-entropy,
    backward (every GEMM on the sm_100a kernels), gradient all-reduce over the
    ranks (NCCL), AdamW step. The 64 sequences are split over the ranks (the
    global batch stays 64: "strong" scaling). Reports
    tokens/s, the step time, and the GEMMs' share of it (CUDA events around
    every GEMM on the library stream, one extra observed step)."""
    rank, local_rank, world = env_rank()
    sys.path.insert(0, ROOT)
    from macrograd_b200 import training

    cfg = training.CONFIG
    T = cfg["context"]
    tokens_per_step = training.BATCH * T
    if args.impl == "reference":
        # the reference's own CPU step on one of its sequences (it is single-threaded)
        if rank != 0:
            return 0
        cpu = decoder_reference_rate(T, args.steps, args.warmup)
        v = cpu["value"]
        print(json.dumps({"impl": "reference", "metric": DECODER_METRIC, "value": v, "unit": "tokens/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                          "data": "synthetic token ids (reference CPU RNG)",
                          "config": {"workload": "decoder training step", **cfg, "batch": training.BATCH},
                          "cpu_baseline": cpu,
                          "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}), flush=True)
        return 0

    import torch
    import torch.distributed as dist

    # the reference's CPU step, timed before any CUDA work (rank 0 of a one-GPU run)
    cpu = decoder_reference_rate(T, 1, 1) if (world == 1 and not args.no_cpu_baseline) else None
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    import macrograd_b200 as mg
    from macrograd_b200 import _lib

    lib = mg.load()
    _lib.check(lib.mg_set_mode(_lib.MG_MODE_TF32X3 if args.mode == "3xtf32" else _lib.MG_MODE_TF32))
    m = training.DecoderStep(device="cuda", device_index=local_rank)
    first, count = training.shard(training.BATCH, world, rank)
    m.make_batch(5, training.BATCH, T, first, count)
    flat = torch.empty(m.numel, dtype=torch.float32, device=dev)

    def step():
        loss = m.forward_backward()
        if world > 1:
            m.allreduce_grads(flat=flat)
        m.optimizer_step()
        return loss

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(max(3, args.warmup)):
        step()
    # GEMM share: one observed step
    m.observe(1)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    step()
    m.lib.c5_synchronize()
    t1.record()
    torch.cuda.synchronize()
    obs_step_ms = t0.elapsed_time(t1)
    gemm_ms, gemm_flop, calls = m.gemm_ms(), m.gemm_flop(), m.gemm_calls()
    m.observe(0)
    launches0 = lib.mg_launch_count()

    clocks = ClockSampler(local_rank)
    clocks.start()
    torch.cuda.synchronize()
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record()
    losses = []
    for _ in range(args.steps):
        losses.append(step())
    m.lib.c5_synchronize()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = lib.mg_launch_count() - launches0
    t = torch.tensor([ev0.elapsed_time(ev1) / args.steps, gemm_ms, obs_step_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step, gemm_ms, obs_step_ms = float(t[0]), float(t[1]), float(t[2])
    m.close()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    value = tokens_per_step / (ms_per_step * 1e-3)
    line = {
        "metric": DECODER_METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic token ids (reference CPU RNG), random init",
        "config": {"workload": "decoder training step (reference modules through the drop-in build)", **cfg,
                   "batch": training.BATCH, "mode": args.mode,
                   "parallelism": f"data-parallel x{world}" + (" + NCCL gradient all-reduce" if world > 1 else "")},
        "gemm": {"calls_per_step": calls, "ms_per_step": gemm_ms, "share_of_step": gemm_ms / obs_step_ms,
                 "tflops": gemm_flop / (gemm_ms * 1e-3) / 1e12 if gemm_ms > 0 else None,
                 "gflop_per_step_per_rank": gemm_flop / 1e9,
                 "note": "CUDA events around every GEMM on the library stream, one observed step (max over ranks)"},
        "loss": losses[-1] if losses else None,
        "gpu_launches": int(launches),
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
