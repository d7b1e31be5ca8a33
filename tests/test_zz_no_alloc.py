"""mg_matmul_noalloc: the allocation-free form of mg_matmul, for callers that
cannot let the library allocate device memory during a call (runtimes that
plan and own all device memory up front, latency-critical loops that must not
touch an allocator). It takes its scratch -- the padded copy of an operand whose
rows are not a multiple of 16 bytes, and the partial tiles of a K-split last
wave with their counters -- from a fixed device buffer inside the library
instead of allocating it.

Checked through the C ABI against mg_matmul on cases that need that scratch,
on two calls in a row (the buffer keeps the previous call's contents), with a
counting allocator registered to show that mg_matmul allocates and
mg_matmul_noalloc does not; on a long-K product whose single tile is split
along K with its partial slots in the buffer (against the oracle, and bit for
bit against mg_matmul's own split); on one whose re-laid-out operands leave no
room for the slots, which must run unsplit; and with an oversized request that
must be refused before anything runs.
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


def _split_slots_bytes(bn, slots):
    """Scratch of a K split with `slots` partial ranges: two 128 x bn fp32
    tiles per slot, then two counters per slot (mg_gemm.cu setup_split)."""
    return slots * 2 * 128 * bn * 4 + slots * 2 * 4


@pytest.mark.parametrize("K", [8192])
def test_noalloc_k_split_from_the_buffer_matches_oracle(K, monkeypatch):
    """A[K,65]^T B[K,65]: one 65 x 65 output tile (single-SM kernel, tile width
    128) on a 148-SM GPU, so the launch splits that tile into 8 K-ranges whose
    7 partial tiles go through the fixed buffer, after both operands' padded
    copies (rows of 65 floats): 2 x 8192 x 68 x 4 B + the slots, well inside it."""
    lib = mg.load()
    relayout = 2 * (K * 68 * 4 + 16)
    assert relayout + 512 + _split_slots_bytes(128, 7) < _lib_scratch_bytes()
    results = []
    for call_no in range(2):
        A_h = ob.seeded_uniform((K, 65), 950 + 10 * call_no)
        B_h = ob.seeded_uniform((K, 65), 951 + 10 * call_no)
        A, B = torch.from_numpy(A_h).cuda(), torch.from_numpy(B_h).cuda()
        st, got = call(lib.mg_matmul_noalloc, A, B, True, False)
        assert st == _lib.MG_OK, lib.mg_last_error()
        st, split = call(lib.mg_matmul, A, B, True, False)
        assert st == _lib.MG_OK, lib.mg_last_error()
        monkeypatch.setenv("MG_GEMM_SPLIT", "0")
        st, unsplit = call(lib.mg_matmul, A, B, True, False)
        monkeypatch.delenv("MG_GEMM_SPLIT")
        assert st == _lib.MG_OK, lib.mg_last_error()
        got, split, unsplit = (x.cpu().numpy() for x in (got, split, unsplit))
        ref = ob.oracle_matmul(A_h, B_h, True, False)
        assert ob.frob_rel_err(got, ref) <= 1e-5, f"call {call_no}"
        # the same plan as mg_matmul's: the partial ranges added in the same order
        assert np.array_equal(got, split), f"call {call_no}: not mg_matmul's split result"
        # ... and a different summation from the one-range launch: the split ran
        assert not np.array_equal(got, unsplit), f"call {call_no}: the launch did not split"
        results.append(got)
    assert not np.array_equal(results[0], results[1])


def test_noalloc_runs_unsplit_when_the_slots_do_not_fit(monkeypatch):
    """The same product with K = 29312: the two padded copies take all but
    ~0.7 MiB of the buffer, less than the 7 partial slots need, so the launch
    must run without its K split -- bit for bit mg_matmul with the split off."""
    lib = mg.load()
    K = 29312
    relayout = 2 * (K * 68 * 4 + 16) + 256
    cap = _lib_scratch_bytes()
    assert relayout <= cap < relayout + _split_slots_bytes(128, 7)
    A_h = ob.seeded_uniform((K, 65), 970)
    B_h = ob.seeded_uniform((K, 65), 971)
    A, B = torch.from_numpy(A_h).cuda(), torch.from_numpy(B_h).cuda()
    for call_no in range(2):
        st, got = call(lib.mg_matmul_noalloc, A, B, True, False)
        assert st == _lib.MG_OK, lib.mg_last_error()
        monkeypatch.setenv("MG_GEMM_SPLIT", "0")
        st, unsplit = call(lib.mg_matmul, A, B, True, False)
        monkeypatch.delenv("MG_GEMM_SPLIT")
        assert st == _lib.MG_OK, lib.mg_last_error()
        got, unsplit = got.cpu().numpy(), unsplit.cpu().numpy()
        assert np.array_equal(got, unsplit), f"call {call_no}"
        assert ob.frob_rel_err(got, ob.oracle_matmul(A_h, B_h, True, False)) <= 1e-5


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
