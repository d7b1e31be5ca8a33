"""The decoder-only character-model training step, data-parallel over ranks.

The model, autograd, loss and optimizer are the reference's own C++ code
(mini_shakespeare/include/transformer.h modules, macrograd/source/nn.cpp
AdamW, Functional::cross_entropy_loss), compiled with the matmul seam into
macrograd_b200/shim/_build/libmacrograd_seam.so (train_driver.cpp), so on
"cuda" every GEMM of the forward and backward pass runs on the sm_100a
kernels; on "cpu" the same step is the reference's CPU arithmetic.

Data parallel: every rank builds the same seeded model, draws the same
seeded batch and keeps its contiguous share of the sequences; after the
backward pass the parameter gradients are summed over the ranks (one flat
all-reduce: NCCL over NVLink on GPUs, gloo on CPU) and divided by the world
size -- the gradient of the mean loss over the whole batch -- and then every
rank takes the same optimizer step. The reference itself is single-process
(README.md:538); this is the data-parallel layer its training loop gains.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence, Tuple

import numpy as np

SEAM = os.path.join(os.path.dirname(os.path.abspath(__file__)), "shim", "_build", "libmacrograd_seam.so")

# The configuration the training step is measured on: 6 layers, 6 heads,
# d_model 384, MLP 4 x 384, context 256, 65 characters, batch 64.
CONFIG = dict(layers=6, heads=6, emb=384, ff=1536, context=256, vocab=65)
BATCH = 64

_c = ctypes
_SIG = {
    "c5_create": (_c.c_int, [_c.c_int] * 6 + [_c.c_ulonglong, _c.c_float, _c.c_float, _c.c_char_p, _c.c_int]),
    "c5_destroy": (None, []),
    "c5_make_batch": (_c.c_int, [_c.c_ulonglong, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_void_p, _c.c_void_p]),
    "c5_forward_backward": (_c.c_float, []),
    "c5_optimizer_step": (_c.c_int, []),
    "c5_synchronize": (None, []),
    "c5_param_count": (_c.c_int, []),
    "c5_param_numel": (_c.c_longlong, []),
    "c5_param_sizes": (_c.c_int, [_c.c_void_p]),
    "c5_copy_out": (_c.c_int, [_c.c_int, _c.c_void_p]),
    "c5_load_grads": (_c.c_int, [_c.c_void_p]),
    "c5_observe": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int]),
    "c5_calls": (_c.c_int, []),
    "c5_gemm_flop": (_c.c_double, []),
    "c5_gemm_ms": (_c.c_double, []),
    "c5_captured": (_c.c_int, []),
    "c5_capture_meta": (_c.c_int, [_c.c_int, _c.c_void_p]),
    "c5_capture_data": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p]),
}

_lib = None


def seam_library():
    """Loads the drop-in build (the sm_100a library first, so the seam binds
    to this package's copy). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(SEAM):
            raise FileNotFoundError(f"{SEAM} is missing: build it with `make -C macrograd_b200/shim REF=/path/to/macrograd`")
        from . import _lib as mglib

        mglib.load()
        lib = ctypes.CDLL(SEAM)
        for name, (res, args) in _SIG.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class CapturedGemm:
    """Operands and result of one GEMM seen at the seam (storage shapes,
    rank-equalised as kernel_ops::matmul receives them)."""

    def __init__(self, index, trans_a, trans_b, out, A, B, bias):
        self.index, self.trans_a, self.trans_b = index, trans_a, trans_b
        self.out, self.A, self.B, self.bias = out, A, B, bias


class DecoderStep:
    """One process's model (the C side holds a single model per process)."""

    def __init__(self, device: str = "cuda", device_index: int = -1, seed: int = 5, lr: float = 1e-3,
                 weight_decay: float = 0.05, **dims):
        cfg = dict(CONFIG)
        cfg.update(dims)
        self.cfg = cfg
        self.device = device
        self.lib = seam_library()
        rc = self.lib.c5_create(cfg["layers"], cfg["heads"], cfg["emb"], cfg["ff"], cfg["context"], cfg["vocab"],
                                seed, lr, weight_decay, device.encode(), device_index)
        if rc != 0:
            raise RuntimeError("a model already exists in this process (close() it first)")
        self.numel = int(self.lib.c5_param_numel())

    def close(self):
        self.lib.c5_destroy()

    def make_batch(self, seed: int, batch_total: int, T: int, first: int, count: int) -> Tuple[np.ndarray, np.ndarray]:
        tok = np.empty((count, T), np.int32)
        tgt = np.empty((count, T), np.int32)
        rc = self.lib.c5_make_batch(seed, batch_total, T, first, count, tok.ctypes.data, tgt.ctypes.data)
        if rc != 0:
            raise ValueError("invalid batch slice")
        return tok, tgt

    def forward_backward(self) -> float:
        return float(self.lib.c5_forward_backward())

    def optimizer_step(self) -> None:
        self.lib.c5_optimizer_step()

    def copy_out(self, which: int, dst_ptr: int) -> None:
        if self.lib.c5_copy_out(which, ctypes.c_void_p(dst_ptr)) != 0:
            raise RuntimeError("copy of the parameters / gradients failed")

    def param_sizes(self) -> np.ndarray:
        out = np.zeros(int(self.lib.c5_param_count()), np.int64)
        self.lib.c5_param_sizes(out.ctypes.data)
        return out

    def host_grads(self) -> np.ndarray:
        """All parameter gradients, flattened in parameter-list order."""
        return self._host(0)

    def host_params(self) -> np.ndarray:
        return self._host(1)

    def _host(self, which: int) -> np.ndarray:
        out = np.empty(self.numel, np.float32)
        if self.device == "cuda":
            import torch

            buf = torch.empty(self.numel, dtype=torch.float32, device="cuda")
            self.copy_out(which, buf.data_ptr())
            out[:] = buf.cpu().numpy()
        else:
            self.copy_out(which, out.ctypes.data)
        return out

    def allreduce_grads(self, group=None, flat=None):
        """Sum the gradients over the ranks, divide by the world size, load
        them back. `flat` (a float32 tensor of numel elements on this rank's
        device, or on CPU for gloo) is reused across steps when given."""
        import torch
        import torch.distributed as dist

        world = dist.get_world_size(group)
        if flat is None:
            dev = torch.device("cuda", torch.cuda.current_device()) if self.device == "cuda" else "cpu"
            flat = torch.empty(self.numel, dtype=torch.float32, device=dev)
        self.copy_out(0, flat.data_ptr())
        dist.all_reduce(flat, group=group)
        flat.div_(world)
        if flat.is_cuda:
            torch.cuda.synchronize()
        if self.lib.c5_load_grads(ctypes.c_void_p(flat.data_ptr())) != 0:
            raise RuntimeError("loading the reduced gradients failed")
        return flat

    # -- seam observer: GEMM timing and operand capture --------------------
    def observe(self, mode: int, indices: Optional[Sequence[int]] = None) -> None:
        idx = np.asarray(list(indices or []), np.int32)
        self.lib.c5_observe(mode, idx.ctypes.data if idx.size else None, int(idx.size))

    def gemm_calls(self) -> int:
        return int(self.lib.c5_calls())

    def gemm_flop(self) -> float:
        return float(self.lib.c5_gemm_flop())

    def gemm_ms(self) -> float:
        return float(self.lib.c5_gemm_ms())

    def captured(self):
        out = []
        meta = np.zeros(69, np.int32)
        for j in range(int(self.lib.c5_captured())):
            self.lib.c5_capture_meta(j, meta.ctypes.data)
            index, rank, ta, tb, has_bias = (int(x) for x in meta[:5])
            shapes = [tuple(int(x) for x in meta[5 + 16 * i: 5 + 16 * i + rank]) for i in range(4)]
            o = np.empty(shapes[0], np.float32)
            A = np.empty(shapes[1], np.float32)
            B = np.empty(shapes[2], np.float32)
            bias = np.empty(shapes[3], np.float32) if has_bias else None
            self.lib.c5_capture_data(j, o.ctypes.data, A.ctypes.data, B.ctypes.data,
                                     bias.ctypes.data if bias is not None else None)
            out.append(CapturedGemm(index, bool(ta), bool(tb), o, A, B, bias))
        return out


def shard(batch_total: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous share of the sequences: (first, count)."""
    base, extra = divmod(batch_total, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)
