"""Parity of the sm_100a kernels (through the C ABI) with the oracle.

Tolerances (Frobenius-normalised relative error ||x - ref||_F / ||ref||_F):
    3xTF32 (default mode) <= 1e-5      TF32 (fast mode) <= 2e-3
At the full config sizes the oracle runs on row / column / head slices: rows
of C depend only on the same rows of op(A) (and all of op(B)), so a slice of
the oracle equals the same slice of the full product bit for bit.
"""
import ctypes

import numpy as np
import pytest

import oracle_bridge as ob

torch = pytest.importorskip("torch")
import macrograd_b200 as mg  # noqa: E402
from macrograd_b200 import _lib, functional as F  # noqa: E402

pytestmark = pytest.mark.gpu

TOL = {_lib.MG_MODE_TF32X3: 1e-5, _lib.MG_MODE_TF32: 2e-3}
MODES = [_lib.MG_MODE_TF32X3, _lib.MG_MODE_TF32]
GOLDEN = np.load(__import__("os").path.join(ob.ROOT, "tests", "golden", "matmul_golden.npz"))


@pytest.fixture(autouse=True)
def _mode_guard():
    lib = mg.load()
    old = lib.mg_get_mode()
    yield
    lib.mg_set_mode(old)


def set_mode(m):
    assert mg.load().mg_set_mode(m) == 0


def cuda(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def gpu_matmul(A, B, ta=False, tb=False, bias=None):
    return host(F.matmul(cuda(A), cuda(B), cuda(bias) if bias is not None else None, ta, tb))


def assert_close(x, ref, mode, what=""):
    """Non-finite entries (e.g. the -inf of a causal mask) must match exactly;
    the Frobenius error is taken over the finite ones."""
    assert x.shape == ref.shape, f"{what}: shape {x.shape} vs {ref.shape}"
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(x), fin), f"{what}: non-finite positions differ"
    assert np.array_equal(x[~fin], ref[~fin], equal_nan=True), f"{what}: non-finite values differ"
    x, ref = x[fin], ref[fin]
    e = ob.frob_rel_err(x, ref)
    assert e <= TOL[mode], f"{what}: frobenius rel err {e:.3e} > {TOL[mode]:.0e} (max/rms {ob.max_rel_err(x, ref):.3e})"
    return e


def status_ok():
    detail = ctypes.c_int32(0)
    return mg.load().mg_device_status(ctypes.byref(detail), 1), detail.value


# ---------------------------------------------------------------- basics
def test_device_is_b200():
    assert torch.cuda.get_device_capability() == (10, 0)


@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 1)])
def test_tf32_operands_are_truncated(ta, tb):
    """The 3xTF32 split relies on this: a TF32 MMA reads an fp32 operand with
    its 13 low mantissa bits dropped (x = 1 + 2^-11 + 2^-12 is read as 1, not
    rounded to 1 + 2^-10), so the raw tile serves as hi and only lo = x - hi
    is formed. Checked for A and B, K-major and MN-major."""
    x = np.float32(1 + 2.0 ** -11 + 2.0 ** -12)
    A = np.zeros((128, 8), np.float32)
    B = np.zeros((8, 16), np.float32)
    A[0, 0], B[0, 0] = x, 1.0
    A[1, 1], B[1, 1] = 1.0, x
    At = np.ascontiguousarray(A.T) if ta else A
    Bt = np.ascontiguousarray(B.T) if tb else B
    set_mode(_lib.MG_MODE_TF32)
    c = gpu_matmul(At, Bt, bool(ta), bool(tb))
    assert c[0, 0] == np.float32(1.0) and c[1, 1] == np.float32(1.0)
    set_mode(_lib.MG_MODE_TF32X3)
    c = gpu_matmul(At, Bt, bool(ta), bool(tb))
    assert c[0, 0] == x and c[1, 1] == x


def test_accumulation_error_does_not_grow_with_k():
    """The MMA's accumulate into TMEM truncates; the kernel promotes a TMEM
    partial into an fp32 master every 256 K-elements, so the 3xTF32 error
    against exact arithmetic stays flat as K grows."""
    set_mode(_lib.MG_MODE_TF32X3)
    errs = []
    for K in (512, 4096, 16384):
        A = ob.seeded_uniform((128, K), 70 + K)
        B = ob.seeded_uniform((K, 64), 71 + K)
        exact = A.astype(np.float64) @ B.astype(np.float64)
        errs.append(ob.frob_rel_err(gpu_matmul(A, B), exact))
    assert max(errs) < 4e-6, errs


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", sorted({k.split("/")[1] for k in GOLDEN.files if k.startswith("fwd/")}))
def test_forward_vs_reference_golden(name, mode):
    set_mode(mode)
    g = lambda k: GOLDEN[f"fwd/{name}/{k}"]
    ta, tb = (bool(x) for x in g("flags"))
    bias = GOLDEN[f"fwd/{name}/bias"] if f"fwd/{name}/bias" in GOLDEN.files else None
    assert_close(gpu_matmul(g("A"), g("B"), ta, tb, bias), g("C"), mode, name)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("name", sorted({k.split("/")[1] for k in GOLDEN.files if k.startswith("bwd/")}))
def test_backward_vs_reference_golden(name, mode):
    set_mode(mode)
    g = lambda k: GOLDEN[f"bwd/{name}/{k}"]
    ta, tb = (bool(x) for x in g("flags"))
    has_bias = f"bwd/{name}/bias" in GOLDEN.files
    dA, dB, db = F.matmul_backward(cuda(g("A")), cuda(g("B")), cuda(g("dC")), ta, tb, has_bias,
                                   g("bias").shape if has_bias else None)
    assert_close(host(dA), g("dA"), mode, name + " dA")
    assert_close(host(dB), g("dB"), mode, name + " dB")
    if has_bias:
        assert_close(host(db), g("dbias"), mode, name + " dbias")


def test_attention_golden_fused_softmax():
    set_mode(_lib.MG_MODE_TF32X3)
    P = host(F.attention_scores(cuda(GOLDEN["attn/Q"]), cuda(GOLDEN["attn/K"]), 0.5, causal=True))
    assert_close(P, GOLDEN["attn/P"], _lib.MG_MODE_TF32X3, "attn P")
    P2 = host(F.attention_scores(cuda(GOLDEN["attn/Q"]), cuda(GOLDEN["attn/K"]), 0.5, causal=False,
                                 mask=cuda(GOLDEN["attn/mask"])))
    assert_close(P2, GOLDEN["attn/P"], _lib.MG_MODE_TF32X3, "attn P (mask tensor)")


# ---------------------------------------------------------------- shapes
ODD = [1, 7, 17, 65, 129]


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,K", [(m, n, k) for m in ODD for n in ODD for k in ODD
                                   if (ODD.index(m) + ODD.index(n) + ODD.index(k)) % 3 == 0])
def test_odd_shapes_all_layouts(M, N, K, ta, tb):
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform((K, M) if ta else (M, K), M * 1000 + K)
    B = ob.seeded_uniform((N, K) if tb else (K, N), N * 1000 + K + 1)
    assert_close(gpu_matmul(A, B, bool(ta), bool(tb)), ob.oracle_matmul(A, B, bool(ta), bool(tb)),
                 _lib.MG_MODE_TF32X3, f"{M}x{N}x{K} t{ta}{tb}")


@pytest.mark.parametrize("sa,sb,ta,tb", [
    ((2, 3, 1, 40, 36), (1, 3, 5, 36, 20), False, False),   # 5-D, broadcast on both sides
    ((6, 1, 48, 32), (6, 32, 70), False, False),
    ((3, 33, 20), (1, 33, 44), True, False),                  # transposed A, broadcast B
    ((4, 130, 66), (4, 70, 66), False, True),                 # odd N tail with transB
    ((2, 2, 300, 260), (260, 257), False, False),             # N > 256: two n-tiles
])
@pytest.mark.parametrize("mode", MODES)
def test_batched_broadcast_layouts(sa, sb, ta, tb, mode):
    set_mode(mode)
    A = ob.seeded_uniform(sa, 101)
    B = ob.seeded_uniform(sb, 102)
    assert_close(gpu_matmul(A, B, ta, tb), ob.oracle_matmul(A, B, ta, tb), mode, f"{sa}x{sb}")


@pytest.fixture(params=[("0", None), ("1", "256"), ("1", "224")],
                ids=["single_sm", "sm_pair_256", "sm_pair_224"])
def kernel_variant(request, monkeypatch):
    """Forces the single-SM (M=128 tiles) or the SM-pair (M=256 tiles,
    cta_group::2) kernel through MG_GEMM_PAIR, and for pairs the tile width
    (256, or 224 -- 112 B columns per SM, a partly filled last MN-major box)
    through MG_GEMM_BN; the library reads both on every call."""
    pair, bn = request.param
    monkeypatch.setenv("MG_GEMM_PAIR", pair)
    if bn is not None:
        monkeypatch.setenv("MG_GEMM_BN", bn)
    return f"pair={pair} bn={bn}"


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("sa,sb,ta,tb,bias_shape", [
    ((300, 520), (520, 200), False, False, None),          # M, N tails in both tiles
    ((2, 260, 96), (2, 300, 96), False, True, (300,)),     # K-major B, bias
    ((3, 64, 400), (64, 130), True, False, None),          # MN-major A and B
    ((520, 70), (40, 520), True, True, (70, 1)),           # both transposed, column bias
    ((4, 256, 64), (4, 256, 64), False, True, None),       # attention-score shape
])
def test_kernel_variants_agree_with_oracle(kernel_variant, mode, sa, sb, ta, tb, bias_shape):
    set_mode(mode)
    A = ob.seeded_uniform(sa, 801)
    B = ob.seeded_uniform(sb, 802)
    bias = ob.seeded_uniform(bias_shape, 803) if bias_shape else None
    assert_close(gpu_matmul(A, B, ta, tb, bias), ob.oracle_matmul(A, B, ta, tb, bias), mode,
                 f"variant {kernel_variant}")


@pytest.mark.parametrize("presplit", ["0", "1"], ids=["split_in_kernel", "lo_planes"])
@pytest.mark.parametrize("sa,sb,ta,tb,bias_shape", [
    ((600, 520), (520, 700), False, False, None),
    ((3, 520, 300), (1, 520, 260), True, False, (260,)),     # broadcast B, MN-major A
    ((2, 2, 300, 96), (2, 1, 270, 96), False, True, None),  # 4-D, broadcast B over one dim
    ((700, 33), (333, 700), True, True, None),               # odd K-major / MN-major widths
])
def test_presplit_paths_agree_with_oracle(kernel_variant, monkeypatch, presplit, sa, sb, ta, tb, bias_shape):
    """3xTF32 with lo computed per tile in the kernel, and with lo planes
    precomputed once in HBM (MG_GEMM_PRESPLIT forces either path)."""
    monkeypatch.setenv("MG_GEMM_PRESPLIT", presplit)
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform(sa, 821)
    B = ob.seeded_uniform(sb, 822)
    bias = ob.seeded_uniform(bias_shape, 823) if bias_shape else None
    assert_close(gpu_matmul(A, B, ta, tb, bias), ob.oracle_matmul(A, B, ta, tb, bias), 0,
                 f"presplit={presplit} variant={kernel_variant}")


def test_kernel_variants_softmax_and_accumulate(kernel_variant):
    set_mode(_lib.MG_MODE_TF32X3)
    q = ob.seeded_normal((3, 2, 200, 64), 811, 0.0, 0.125)
    k = ob.seeded_normal((3, 2, 200, 64), 812, 0.0, 0.125)
    P = host(F.attention_scores(cuda(q), cuda(k), 0.125, causal=True))
    mask = ob.oracle_causal_mask(200)
    for b in range(3):
        for h in range(2):
            S = ob.oracle_matmul(q[b, h] * np.float32(0.125), k[b, h], False, True, mask)
            assert_close(P[b, h], ob.oracle_softmax_rows(S), 0, f"softmax {kernel_variant}")
    A = ob.seeded_uniform((4, 300, 48), 813)
    W = ob.seeded_uniform((48, 80), 814)
    dC = ob.seeded_normal((4, 300, 80), 815)
    prev = ob.seeded_normal((48, 80), 816)
    g = cuda(prev)
    F.matmul_backward(cuda(A), cuda(W), cuda(dC), need_a=False, grad_b=g)
    _, dW, _ = ob.oracle_matmul_backward(A, W, dC)
    assert_close(host(g), prev + dW, 0, f"beta=1 {kernel_variant}")


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("M,N", [(40, 17), (64, 64), (100, 100), (70, 130), (256, 256), (300, 250)])
@pytest.mark.parametrize("scale", [0.125, -0.5])
def test_row_softmax_widths_and_scales(mode, M, N, scale):
    """The fused row softmax at every tile width it runs at (N up to 64, 128
    and 256 columns, ragged ends, M != N), its two warps' alternating 32-column
    blocks, causal and not, a negative scale (the per-column path) and an
    additive mask (the bias path), against the oracle."""
    set_mode(mode)
    q = ob.seeded_normal((2, 3, M, 40), 871 + M, 0.0, 0.5)
    k = ob.seeded_normal((2, 3, N, 40), 872 + N, 0.0, 0.5)
    add = ob.seeded_normal((M, N), 873 + M + N)
    causal_mask = np.where(np.arange(N)[None, :] > np.arange(M)[:, None], -np.inf, 0.0).astype(np.float32)
    for what, causal, mask in (("causal", True, None), ("full", False, None), ("mask", False, add)):
        P = host(F.attention_scores(cuda(q), cuda(k), scale, causal=causal,
                                    mask=cuda(mask) if mask is not None else None))
        ref_mask = causal_mask if causal else mask
        for b in range(2):
            for h in range(3):
                S = ob.oracle_matmul(q[b, h] * np.float32(scale), k[b, h], False, True, ref_mask)
                assert_close(P[b, h], ob.oracle_softmax_rows(S), mode, f"{what} softmax {M}x{N} scale {scale}")


@pytest.mark.parametrize("pair", ["1", "0"], ids=["sm_pair", "single_sm"])
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("sa,sb,ta,tb,bias_shape", [
    ((512, 1024), (1024, 1024), False, False, None),      # few tiles: one level, up to 8 K-ranges a tile
    ((2048, 256), (256, 4096), False, False, None),       # 128 pair tiles: whole wave + 2- and 4-way levels
    ((300, 1000), (700, 1000), False, True, (700,)),      # tails in M and N, bias added once
    ((1000, 640), (1000, 520), True, False, (1, 520)),    # MN-major A
])
def test_k_split_of_the_last_wave(monkeypatch, pair, mode, sa, sb, ta, tb, bias_shape):
    """The last, partial wave of tiles split over K (ranges summed in fp32 by
    the final range of each tile); MG_GEMM_SPLIT_MIN_KB=1 lets short K split
    too. Same tolerance as unsplit, and the unsplit launch agrees."""
    monkeypatch.setenv("MG_GEMM_PAIR", pair)
    monkeypatch.setenv("MG_GEMM_SPLIT_MIN_KB", "1")
    set_mode(mode)
    A = ob.seeded_uniform(sa, 841)
    B = ob.seeded_uniform(sb, 842)
    bias = ob.seeded_uniform(bias_shape, 843) if bias_shape else None
    ref = ob.oracle_matmul(A, B, ta, tb, bias)
    split = gpu_matmul(A, B, ta, tb, bias)
    assert_close(split, ref, mode, "split")
    monkeypatch.setenv("MG_GEMM_SPLIT", "0")
    unsplit = gpu_matmul(A, B, ta, tb, bias)
    assert_close(unsplit, ref, mode, "unsplit")
    # the split launch really ran: its ranges are summed in another order
    assert not np.array_equal(split, unsplit)


@pytest.mark.parametrize("mode", MODES)
def test_attention_head_split_as_strided_views(mode):
    """The multi-head attention's head split / merge (transformer.h:226-228,
    244) as strides of the GEMM operands and output: Q, K, V stay [B, L, E]
    tensors, the [B, H, L, d] heads are views, and O is written straight into
    its merged [B, L, E] layout -- against the oracle on materialised heads."""
    set_mode(mode)
    B_, L, H, d = 3, 96, 6, 64
    E = H * d
    q = ob.seeded_normal((B_, L, E), 861, 0.0, 0.125)
    k = ob.seeded_normal((B_, L, E), 862, 0.0, 0.125)
    v = ob.seeded_normal((B_, L, E), 863)
    heads = lambda x: x.view(B_, L, H, d).transpose(1, 2)     # [B, H, L, d], no copy
    qg, kg, vg = cuda(q), cuda(k), cuda(v)
    S = F.matmul_view(heads(qg), heads(kg).transpose(-1, -2), alpha=0.125)
    O = torch.empty(B_, L, E, device="cuda")
    F.matmul_view(S, heads(vg), out=heads(O))
    qh = np.ascontiguousarray(q.reshape(B_, L, H, d).transpose(0, 2, 1, 3))
    kh = np.ascontiguousarray(k.reshape(B_, L, H, d).transpose(0, 2, 1, 3))
    vh = np.ascontiguousarray(v.reshape(B_, L, H, d).transpose(0, 2, 1, 3))
    S_ref = ob.oracle_matmul(qh * np.float32(0.125), kh, False, True)
    assert_close(host(S), S_ref, mode, "scores on head views")
    O_ref = ob.oracle_matmul(host(S), vh).transpose(0, 2, 1, 3).reshape(B_, L, E)
    assert_close(host(O), O_ref, mode, "output merged in place")


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("shape", [(4, 6, 256, 64), (3, 2, 200, 64), (2, 96, 40)])
def test_fused_softmax_backward(mode, shape):
    """dS = P * (dP - rowsum(P * dP)), dP = dO V^T, from one launch, against
    the same expression in float64 from the oracle's GEMM inputs (the
    reference's SoftOp::_backward, tensor_ops.cpp:2056-2059; test_oracle.py
    checks the expression against the reference's own autograd)."""
    set_mode(mode)
    L = shape[-2]
    q = ob.seeded_normal(shape, 871, 0.0, 0.125)
    k = ob.seeded_normal(shape, 872, 0.0, 0.125)
    v = ob.seeded_normal(shape, 873)
    dO = ob.seeded_normal(shape, 874)
    P = host(F.attention_scores(cuda(q), cuda(k), 0.125, causal=True))
    dS = host(F.attention_softmax_backward(cuda(dO), cuda(v), cuda(P)))
    dP = np.matmul(dO.astype(np.float64), np.swapaxes(v.astype(np.float64), -1, -2))
    P64 = P.astype(np.float64)
    ref = P64 * (dP - (P64 * dP).sum(-1, keepdims=True))
    assert dS.shape == ref.shape == P.shape[:-1] + (L,)
    assert_close(dS, ref.astype(np.float32), mode, "softmax backward")


def test_k_split_with_accumulate(monkeypatch):
    """beta = 1 (gradient accumulation) is applied once, by the final range."""
    monkeypatch.setenv("MG_GEMM_SPLIT_MIN_KB", "1")
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform((6, 400, 96), 851)
    W = ob.seeded_uniform((96, 300), 852)
    dC = ob.seeded_normal((6, 400, 300), 853)
    prev = ob.seeded_normal((96, 300), 854)
    g = cuda(prev)
    F.matmul_backward(cuda(A), cuda(W), cuda(dC), need_a=False, grad_b=g)
    _, dW, _ = ob.oracle_matmul_backward(A, W, dC)
    assert_close(host(g), prev + dW, 0, "beta=1 split")


@pytest.mark.parametrize("b2", ["1", "0"])
@pytest.mark.parametrize("sa,sb,ta,tb", [
    ((100, 1000), (1000, 50), False, False),     # one m-tile, K over 4 promotion chunks
    ((1000, 100), (50, 1000), True, True),       # both operands transposed views
    ((3, 128, 256), (3, 256, 64), False, False), # batched, one chunk (two accumulators)
    ((3, 256, 128), (3, 256, 40), True, False),  # MN-major A, N tail
])
def test_narrow_tiles_a_in_tmem(monkeypatch, b2, sa, sb, ta, tb):
    """3xTF32 tiles of width 64 with A in tensor memory: [B hi | B lo] as one
    operand of width 128 (two MMAs a K-step, the accumulator's halves added)
    or three MMAs of width 64 (MG_GEMM_B2=0); with promotion chunks and with
    two accumulators, against the oracle. The pre-split A/B path agrees."""
    monkeypatch.setenv("MG_GEMM_B2", b2)
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform(sa, 891)
    B = ob.seeded_uniform(sb, 892)
    ref = ob.oracle_matmul(A, B, ta, tb)
    assert_close(gpu_matmul(A, B, ta, tb), ref, _lib.MG_MODE_TF32X3, f"b2={b2}")
    monkeypatch.setenv("MG_GEMM_A_TMEM", "0")
    assert_close(gpu_matmul(A, B, ta, tb), ref, _lib.MG_MODE_TF32X3, "A in shared memory")


@pytest.mark.parametrize("blocks", ["1", "2"])
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("sa,sb,ta,tb", [
    ((3, 300, 96), (96, 200), False, False),     # M and N tails, short K, broadcast B
    ((2, 129, 64), (2, 250, 64), False, True),   # transposed B, widths below 256
    ((640, 1000), (1000, 72), False, False),     # long K, narrow N
])
def test_staging_blocks_forced(monkeypatch, blocks, mode, sa, sb, ta, tb):
    """One or two epilogue staging blocks per warp (MG_GEMM_STAGE_BLOCKS;
    with two, consecutive TMA stores of C alternate blocks and a store waits
    only for the store before last), against the oracle."""
    monkeypatch.setenv("MG_GEMM_STAGE_BLOCKS", blocks)
    set_mode(mode)
    A = ob.seeded_uniform(sa, 881)
    B = ob.seeded_uniform(sb, 882)
    assert_close(gpu_matmul(A, B, ta, tb), ob.oracle_matmul(A, B, ta, tb), mode, f"stage blocks {blocks}")
    q = ob.seeded_normal((2, 3, 150, 40), 883, 0.0, 0.5)
    k = ob.seeded_normal((2, 3, 150, 40), 884, 0.0, 0.5)
    P = host(F.attention_scores(cuda(q), cuda(k), 0.25, causal=True))
    mask = ob.oracle_causal_mask(150)
    for b in range(2):
        for h in range(3):
            S = ob.oracle_matmul(q[b, h] * np.float32(0.25), k[b, h], False, True, mask)
            assert_close(P[b, h], ob.oracle_softmax_rows(S), mode, f"softmax, stage blocks {blocks}")


@pytest.mark.parametrize("bias_shape", [(40,), (1, 40), (30, 1), (30, 40), (3, 1, 40), (3, 30, 40)])
def test_bias_broadcast_forms(bias_shape):
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform((3, 30, 50), 201)
    B = ob.seeded_uniform((50, 40), 202)
    bias = ob.seeded_uniform(bias_shape, 203)
    assert_close(gpu_matmul(A, B, bias=bias), ob.oracle_matmul(A, B, bias=bias), _lib.MG_MODE_TF32X3,
                 str(bias_shape))


def test_unaligned_rows_take_the_relayout_path():
    # vocab-65 logits: rows of 260 bytes are not 16-byte multiples (TMA rule)
    set_mode(_lib.MG_MODE_TF32X3)
    dC = ob.seeded_normal((512, 65), 301)
    table = ob.seeded_uniform((65, 384), 302)
    x = ob.seeded_uniform((512, 384), 303)
    assert_close(gpu_matmul(dC, table), ob.oracle_matmul(dC, table), 0, "dx = dC table")
    assert_close(gpu_matmul(dC, x, True, False), ob.oracle_matmul(dC, x, True, False), 0, "dtable")
    assert_close(gpu_matmul(x, table, False, True), ob.oracle_matmul(x, table, False, True), 0, "logits")


def test_vector_operands_squeeze_like_reference():
    A = ob.seeded_uniform((5, 7), 401)
    v = ob.seeded_uniform((7,), 402)
    r = gpu_matmul(A, v)
    assert r.shape == (5,)
    assert_close(r, ob.oracle_matmul(A, v), 0, "gemv")
    r = gpu_matmul(v, ob.seeded_uniform((7, 3), 403))
    assert r.shape == (3,)


def test_k_zero_gives_bias_or_zero():
    A = np.zeros((3, 5, 0), np.float32)
    B = np.zeros((0, 4), np.float32)
    assert np.array_equal(gpu_matmul(A, B), np.zeros((3, 5, 4), np.float32))
    bias = ob.seeded_uniform((4,), 7)
    assert np.array_equal(gpu_matmul(A, B, bias=bias), np.broadcast_to(bias, (3, 5, 4)))


def test_empty_outputs():
    assert gpu_matmul(np.zeros((0, 5), np.float32), np.ones((5, 3), np.float32)).shape == (0, 3)
    assert gpu_matmul(np.zeros((2, 0, 5), np.float32), np.ones((5, 3), np.float32)).shape == (2, 0, 3)


def test_beta_accumulate_into_existing_gradient():
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform((4, 64, 48), 501)
    W = ob.seeded_uniform((48, 80), 502)
    dC = ob.seeded_normal((4, 64, 80), 503)
    prev = ob.seeded_normal((48, 80), 504)
    g = cuda(prev)
    F.matmul_backward(cuda(A), cuda(W), cuda(dC), need_a=False, grad_b=g)
    _, dW, _ = ob.oracle_matmul_backward(A, W, dC)
    assert_close(host(g), prev + dW, 0, "grad += dW (beta = 1)")


def test_nonfinite_inputs_propagate():
    set_mode(_lib.MG_MODE_TF32X3)
    A = ob.seeded_uniform((128, 32), 601)
    B = ob.seeded_uniform((32, 64), 602)
    A[3, 5] = np.inf
    A[9, 0] = np.nan
    C = gpu_matmul(A, B)
    R = ob.oracle_matmul(A, B)
    assert np.array_equal(np.isnan(C), np.isnan(R))
    assert np.array_equal(np.isinf(C), np.isinf(R))
    fin = np.isfinite(R)
    assert ob.frob_rel_err(C[fin], R[fin]) <= 1e-5


def test_readme_known_answer_on_gpu():
    from test_oracle import (README_FINAL_GRAD, README_FINAL_PARAMS, README_LOSSES,
                             readme_least_squares)
    set_mode(_lib.MG_MODE_TF32X3)
    losses, params, grad = readme_least_squares(
        lambda A, x: gpu_matmul(A, x),
        lambda A, dC: gpu_matmul(A, dC.reshape(4, 1), True, False).reshape(4))
    assert np.allclose(losses, README_LOSSES, atol=5e-5)
    assert np.allclose(params, README_FINAL_PARAMS, atol=5e-5)
    assert np.allclose(grad, README_FINAL_GRAD, atol=5e-5)


# ---------------------------------------------------------------- configs
@pytest.mark.parametrize("mode", MODES)
def test_config1_forward_and_backward(mode):
    """A[8,256,384] @ W[384,384], U(-1,1) seed 1; backward with dC = ones."""
    set_mode(mode)
    A = ob.seeded_uniform((8, 256, 384), 1)
    W = ob.seeded_uniform((384, 384), 1001)
    dC = np.ones((8, 256, 384), np.float32)
    C = gpu_matmul(A, W)
    assert_close(C, ob.oracle_matmul(A, W), mode, "cfg1 C")
    dA, dW, _ = F.matmul_backward(cuda(A), cuda(W), cuda(dC))
    rA, rW, _ = ob.oracle_matmul_backward(A, W, dC)
    assert_close(host(dA), rA, mode, "cfg1 dA")
    assert_close(host(dW), rW, mode, "cfg1 dW")


@pytest.mark.parametrize("mode", MODES)
def test_config2_linear_layer(mode):
    """X[16384,384] @ W[1536,384]^T + b, Kaiming-uniform W and b (bound
    1/sqrt(384)*sqrt(6)... as sqrt(6/384)), dY ~ N(0,1); checked on row and
    column slices of the oracle."""
    set_mode(mode)
    bound = float(np.sqrt(6.0 / 384))
    X = ob.seeded_uniform((16384, 384), 2)
    W = ob.seeded_uniform((1536, 384), 1002, -bound, bound)
    b = ob.seeded_uniform((1536,), 2002, -bound, bound)
    dY = ob.seeded_normal((16384, 1536), 3002)
    Xg, Wg, dYg = cuda(X), cuda(W), cuda(dY)
    Y = host(F.matmul(Xg, Wg, cuda(b), False, True))
    rows = slice(8000, 8192)
    assert_close(Y[rows], ob.oracle_matmul(X[rows], W, False, True, b), mode, "cfg2 Y rows")
    # the weight and bias gradients accumulate into existing ones (beta = 1),
    # as `internal_gradient() += ...` does in MatMulBiasOp::_backward
    prevW = ob.seeded_normal((1536, 384), 4002)
    prevb = ob.seeded_normal((1536,), 5002)
    gW, gb = cuda(prevW), cuda(prevb)
    dX, dW, db = F.matmul_backward(Xg, Wg, dYg, False, True, True, (1536,), grad_b=gW, grad_bias=gb)
    assert dW.data_ptr() == gW.data_ptr() and db.data_ptr() == gb.data_ptr()
    assert_close(host(dX)[rows], ob.oracle_matmul(dY[rows], W), mode, "cfg2 dX rows")
    cols = slice(96, 160)
    rdW = ob.oracle_matmul(dY, np.ascontiguousarray(X[:, cols]), True, False)
    assert_close(host(dW)[:, cols], prevW[:, cols] + rdW, mode, "cfg2 dW cols (+=)")
    assert_close(host(db), prevb + ob.oracle_reduce_to(dY, [1, 1536]).reshape(1536), _lib.MG_MODE_TF32X3,
                 "cfg2 db (+=)")


def test_config3_attention_forward_and_backward():
    """Q,K ~ N(0, 1/8), V ~ N(0,1) [64,6,256,64]; S = QK^T/8 + causal, P =
    softmax(S) fused; O = P V; backward with dO ~ N(0,1) through both GEMMs.
    The oracle runs on 3 of the 384 (batch, head) slices."""
    set_mode(_lib.MG_MODE_TF32X3)
    shp = (64, 6, 256, 64)
    Q = ob.seeded_normal(shp, 3, 0.0, 0.125)
    K = ob.seeded_normal(shp, 1003, 0.0, 0.125)
    V = ob.seeded_normal(shp, 2003)
    dO = ob.seeded_normal(shp, 4003)
    Qg, Kg, Vg, dOg = cuda(Q), cuda(K), cuda(V), cuda(dO)
    P = F.attention_scores(Qg, Kg, 0.125, causal=True)
    O = F.matmul(P, Vg)
    dP, dV, _ = F.matmul_backward(P, Vg, dOg)
    Ph, Oh, dPh, dVh = host(P), host(O), host(dP), host(dV)
    mask = ob.oracle_causal_mask(256)
    for (bi, hi) in [(0, 0), (31, 4), (63, 5)]:
        q, k, v, do = Q[bi, hi], K[bi, hi], V[bi, hi], dO[bi, hi]
        S = ob.oracle_matmul(q * np.float32(0.125), k, False, True, mask)
        Pr = ob.oracle_softmax_rows(S)
        assert_close(Ph[bi, hi], Pr, 0, "cfg3 P")
        assert_close(Oh[bi, hi], ob.oracle_matmul(Pr, v), 0, "cfg3 O")
        rdP, rdV, _ = ob.oracle_matmul_backward(Pr, v, do)
        assert_close(dPh[bi, hi], rdP, 0, "cfg3 dP")
        assert_close(dVh[bi, hi], rdV, 0, "cfg3 dV")
    # score-GEMM backward: dQs = dS K, dK = dS^T Qs
    dS = ob.seeded_normal(shp[:3] + (256,), 5003)
    Qs = cuda(Q * np.float32(0.125))
    dQs, dK, _ = F.matmul_backward(Qs, Kg, cuda(dS), False, True)
    dQh, dKh = host(dQs), host(dK)
    for (bi, hi) in [(5, 1), (40, 3)]:
        rQ, rK, _ = ob.oracle_matmul_backward(Q[bi, hi] * np.float32(0.125), K[bi, hi], dS[bi, hi], False, True)
        assert_close(dQh[bi, hi], rQ, 0, "cfg3 dQs")
        assert_close(dKh[bi, hi], rK, 0, "cfg3 dK")


@pytest.mark.parametrize("mode", MODES)
def test_config4_square_8192_row_slices(mode):
    """A,B[8192,8192] ~ U(-1,1) seed 4; rows 0..31, 4096..4127 and the last
    m-tile's 8160..8191 (the last wave's tiles) of C against the oracle on the
    same row slices (bit-identical to its full product)."""
    set_mode(mode)
    n = 8192
    A = ob.seeded_uniform((n, n), 4)
    B = ob.seeded_uniform((n, n), 1004)
    C = F.matmul(cuda(A), cuda(B))
    torch.cuda.synchronize()
    for r0 in (0, 4096, 8160):
        rows = slice(r0, r0 + 32)
        got = C[rows].cpu().numpy()
        assert_close(got, ob.oracle_matmul(A[rows], B), mode, f"cfg4 rows {r0}")
        # and against exact (float64) arithmetic: the GPU is at least as close as the oracle
        exact = A[rows].astype(np.float64) @ B.astype(np.float64)
        if mode == _lib.MG_MODE_TF32X3:
            assert ob.frob_rel_err(got, exact) <= 1e-5


def test_no_kernel_timed_out():
    st, detail = status_ok()
    assert st == 0, f"device status {st}, wait site {detail}"


def test_native_launches_counted():
    lib = mg.load()
    before = lib.mg_launch_count()
    gpu_matmul(np.ones((4, 4), np.float32), np.ones((4, 4), np.float32))
    assert lib.mg_launch_count() == before + 1
