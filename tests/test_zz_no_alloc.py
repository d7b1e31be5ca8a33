"""mg_matmul_noalloc: the allocation-free form of mg_matmul, for callers that
cannot let the library allocate device memory during a call (runtimes that
plan and own all device memory up front, latency-critical loops that must not
touch an allocator). It takes its scratch -- the padded copy of an operand whose
rows are not a multiple of 16 bytes -- from a fixed device buffer inside the
library instead of allocating it.

Checked through the C ABI against mg_matmul on cases that need that scratch,
on two calls in a row (the buffer keeps the previous call's contents), with a
counting allocator registered to show that mg_matmul allocates and
mg_matmul_noalloc does not, and with an oversized request that must be
refused before anything runs.
"""
import ctypes

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
import macrograd_b200 as mg  # noqa: E402
from macrograd_b200 import _lib  # noqa: E402
from macrograd_b200._lib import i32_array  # noqa: E402

pytestmark = pytest.mark.gpu

ALLOC_FN = ctypes.CFUNCTYPE(ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p)
FREE_FN = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p)


class CountingAllocator:
    """Workspace allocator that counts calls (test only; backs blocks with torch)."""

    def __init__(self):
        self.allocs = 0
        self.live = {}
        self.alloc_fn = ALLOC_FN(self._alloc)
        self.free_fn = FREE_FN(self._free)

    def _alloc(self, nbytes, stream, ctx):
        self.allocs += 1
        t = torch.empty(int(nbytes), dtype=torch.uint8, device="cuda")
        self.live[t.data_ptr()] = t
        return t.data_ptr()

    def _free(self, ptr, stream, ctx):
        self.live.pop(ptr, None)


def call(fn, A, B, ta=False, tb=False):
    """Runs mg_matmul or mg_matmul_noalloc on CUDA tensors A, B (storage shapes,
    rank-equalised by the caller) and returns (status, out)."""
    a, b = list(A.shape), list(B.shape)
    out_shape = [max(x, y) for x, y in zip(a[:-2], b[:-2])] + [a[-1] if ta else a[-2], b[-2] if tb else b[-1]]
    out = torch.full(out_shape, float("nan"), device="cuda")
    st = fn(ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
            i32_array(out_shape), i32_array(a), i32_array(b), len(out_shape), int(ta), int(tb),
            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    return st, out


CASES = [
    # (A storage shape, B storage shape, transA, transB): every case has an
    # operand with rows of 65 or 130 floats, which mg_matmul re-lays out in scratch
    ((3, 1000, 65), (1, 65, 130), False, False),
    ((2048, 65), (384, 65), False, True),
    ((65, 701), (65, 96), True, False),
]


@pytest.mark.parametrize("sa,sb,ta,tb", CASES)
def test_noalloc_matches_mg_matmul_two_calls_in_a_row(sa, sb, ta, tb):
    lib = mg.load()
    counter = CountingAllocator()
    lib.mg_set_allocator(ctypes.cast(counter.alloc_fn, ctypes.c_void_p),
                         ctypes.cast(counter.free_fn, ctypes.c_void_p), None)
    try:
        for call_no in range(2):
            A = torch.from_numpy(ob.seeded_uniform(sa, 900 + 10 * call_no)).cuda()
            B = torch.from_numpy(ob.seeded_uniform(sb, 901 + 10 * call_no)).cuda()
            before = counter.allocs
            st_ref, ref = call(lib.mg_matmul, A, B, ta, tb)
            assert st_ref == _lib.MG_OK, lib.mg_last_error()
            assert counter.allocs > before, "mg_matmul was expected to need scratch here"
            before = counter.allocs
            st, got = call(lib.mg_matmul_noalloc, A, B, ta, tb)
            assert st == _lib.MG_OK, lib.mg_last_error()
            assert counter.allocs == before, "mg_matmul_noalloc allocated"
            got, ref = got.cpu().numpy(), ref.cpu().numpy()
            assert np.all(np.isfinite(got))
            assert ob.frob_rel_err(got, ref) <= 1e-5, f"call {call_no}"
    finally:
        lib.mg_set_allocator(None, None, None)


def test_noalloc_refuses_requests_beyond_its_buffer():
    lib = mg.load()
    rows = (_lib_scratch_bytes() // (68 * 4)) + 64        # padded copy of A just too large
    A = torch.zeros(rows, 65, device="cuda")
    B = torch.zeros(65, 32, device="cuda")
    st, out = call(lib.mg_matmul_noalloc, A, B)
    assert st == _lib.MG_ERR_INVALID
    assert "MG_NOALLOC_SCRATCH_BYTES" in lib.mg_last_error().decode()
    assert torch.isnan(out).all(), "nothing may run when the request is refused"


def _lib_scratch_bytes():
    import os
    import re
    text = open(os.path.join(ob.ROOT, "include", "mg_gemm.h")).read()
    m = re.search(r"#define MG_NOALLOC_SCRATCH_BYTES \((\d+)u << (\d+)\)", text)
    return int(m.group(1)) << int(m.group(2))
