"""GPU parity of the tensor-core GEMM (the hot path) through the C ABI.

Tolerances (written per test):
  * bf16-weight path (gemm_nt_bf16): relative Frobenius error <= 2e-3 against the
    reference CPU GEMM (north-star gate per GEMM); the GPU rounds A to bf16 as the
    reference backend does (backend_cuda.cu:466-467), the CPU keeps A exact.
  * fp32-weight path (gemm_nt_f32, tf32 tensor cores): relative Frobenius <= 2e-3.
  * M <= 16 (memory-bound fp32 kernel, exact operands): relative Frobenius <= 1e-5.
  * bf16 A given directly (gemm_nt_bf16a): same operands as the CPU on the widened
    values, so only summation order differs: relative Frobenius <= 1e-5.
"""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_golden, rel_fro

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-3
TOL_TF32 = 2e-3
TOL_EXACT = 1e-5


def _t(a, dtype=None):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def _bf16_t(bits):
    """uint16 bf16 bit patterns -> torch.bfloat16 CUDA tensor with the same bits."""
    import torch

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).cuda().view(torch.bfloat16)


def _np(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture(autouse=True)
def _auto_tile(sdb):
    sdb.check(sdb.lib().sdb200_set_gemm_tile(0))
    yield
    sdb.check(sdb.lib().sdb200_set_gemm_tile(0))


def test_golden_gemm_f32(sdb):
    """test_ops.cpp gemm shapes: padded ld, bias, accumulate, fp32 weights."""
    import torch

    be = sdb.backend
    for f in sorted(glob.glob(os.path.join(GOLDEN, "gemm_[0-9]*.npz"))):
        g = np.load(f)
        M, N, K, bias, acc = (int(v) for v in g["dims"])
        A, B = _t(g["A"]), _t(g["B"])
        C = _t(g["C0"]) if acc else torch.zeros((M, N + 2), device="cuda")
        be.gemm_nt_f32(A, B, _t(g["bias"]) if bias else None, C, bool(acc), M=M, N=N, K=K,
                       lda=K + 3, ldb=K + 5, ldc=N + 2)
        got = _np(C)
        tol = TOL_EXACT if M <= 16 else TOL_TF32
        assert rel_fro(got[:, :N], g["C"][:, :N]) <= tol, f
        assert np.array_equal(got[:, N:], g["C"][:, N:]), f  # padding columns untouched


def test_golden_gemm_bf16(sdb):
    be = sdb.backend
    for f in sorted(glob.glob(os.path.join(GOLDEN, "gemm_bf16_*.npz"))):
        g = np.load(f)
        C = be.gemm_nt_bf16(_t(g["A"]), _bf16_t(g["Bh"]), _t(g["bias"]))
        assert rel_fro(_np(C), g["C"]) <= TOL_BF16, f


@pytest.mark.parametrize("bn", [64, 128, 192, 256])
@pytest.mark.parametrize("M,N,K", [(129, 257, 300), (300, 500, 200), (256, 512, 64), (1000, 77, 40), (17, 96, 4000)])
def test_gemm_bf16_tiles_and_edges(sdb, orc, bn, M, N, K):
    """Every tile width, ragged M/N/K, padded lda/ldb (B repacked when its pitch breaks
    TMA's 16-byte rule), bias and accumulate."""
    import torch

    sdb.check(sdb.lib().sdb200_set_gemm_tile(bn))
    rng = np.random.default_rng(M + N + K + bn)
    A = rng.standard_normal((M, K + 3)).astype(np.float32)
    Bh = orc.to_bf16(rng.standard_normal((N, K + 5)).astype(np.float32))
    bias = rng.standard_normal(N).astype(np.float32)
    C0 = rng.standard_normal((M, N + 2)).astype(np.float32)
    want = orc.gemm_nt_bf16(A, Bh, bias, C0, M, N, K)
    C = _t(C0)
    sdb.backend.gemm_nt_bf16(_t(A), _bf16_t(Bh), _t(bias), C, True, M=M, N=N, K=K, lda=K + 3, ldb=K + 5,
                             ldc=N + 2)
    got = _np(C)
    assert rel_fro(got[:, :N], want[:, :N]) <= TOL_BF16
    assert np.array_equal(got[:, N:], C0[:, N:])
    # no accumulate, no bias, aligned operands (B used in place by TMA)
    A2 = np.ascontiguousarray(A[:, :K])
    B2 = np.ascontiguousarray(Bh[:, :K]) if K % 8 == 0 else None
    if B2 is not None:
        want2 = orc.gemm_nt_bf16(A2, B2)
        got2 = _np(sdb.backend.gemm_nt_bf16(_t(A2), _bf16_t(B2)))
        assert rel_fro(got2, want2) <= TOL_BF16
    del torch


@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("M,N,K", [(130, 320, 320), (4096 // 8, 2560, 320), (200, 77, 768), (320, 512, 2880)])
def test_gemm_f32_tf32(sdb, orc, bn, M, N, K):
    """fp32 weights (SD1.5 shapes: attention projections, GEGLU proj, cross k/v, conv)."""
    sdb.check(sdb.lib().sdb200_set_gemm_tile(bn))
    rng = np.random.default_rng(M * 3 + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32)
    want = orc.gemm_nt(A, B, bias)
    got = _np(sdb.backend.gemm_nt_f32(_t(A), _t(B), _t(bias)))
    assert rel_fro(got, want) <= TOL_TF32


def test_gemm_bf16a_exact_operands(sdb, orc):
    rng = np.random.default_rng(7)
    M, N, K = 384, 640, 512
    Ah = orc.to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    Bh = orc.to_bf16(rng.standard_normal((N, K)).astype(np.float32))
    Aw = (Ah.astype(np.uint32) << 16).view(np.float32)
    want = orc.gemm_nt_bf16(Aw, Bh)
    got = _np(sdb.backend.gemm_nt_bf16a(_bf16_t(Ah), _bf16_t(Bh)))
    assert rel_fro(got, want) <= TOL_EXACT


@pytest.mark.parametrize("M,N,K", [(1, 15360, 256), (3, 3840, 256), (16, 1000, 1024), (5, 77, 40)])
def test_gemm_small_m(sdb, orc, M, N, K):
    """adaLN GEMV (M=1, N=4*3840, K=256) and other small-M shapes: exact fp32 kernel."""
    rng = np.random.default_rng(M + N)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Bf = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    Bh = orc.to_bf16(Bf)
    bias = rng.standard_normal(N).astype(np.float32)
    got = _np(sdb.backend.gemm_nt_bf16(_t(A), _bf16_t(Bh), _t(bias)))
    assert rel_fro(got, orc.gemm_nt_bf16(A, Bh, bias)) <= TOL_EXACT
    got = _np(sdb.backend.gemm_nt_f32(_t(A), _t(Bf), _t(bias)))
    assert rel_fro(got, orc.gemm_nt(A, Bf, bias)) <= TOL_EXACT


def test_gemm_k_zero_is_bias(sdb):
    import torch

    bias = torch.arange(10, dtype=torch.float32, device="cuda")
    A = torch.zeros((300, 8), device="cuda")
    B = torch.zeros((10, 8), device="cuda", dtype=torch.bfloat16)
    C = sdb.backend.gemm_nt_bf16(A, B, bias, K=0)
    assert torch.equal(C, bias.expand(300, 10))


def test_cfg1_fused_qkv_full_size(sdb, orc):
    """BASELINE config 1 at full size: X [4096,3840] ~N(0,1), W bf16 [11520,3840]
    ~N(0,0.02), bias ~N(0,0.01), seed 0. Checked against the committed reference rows,
    against the oracle on 512 sampled rows, and by size-independent properties on the
    full output: a second run with accumulate=1 gives C + (C - bias), and repeated
    runs are bit-identical."""
    import torch

    from sdb200.workloads import cfg1_inputs

    X, W, b = cfg1_inputs()
    Wh = orc.to_bf16(W)
    g = load_golden("cfg1_rows")
    Xt, Wt, bt = _t(X), _bf16_t(Wh), _t(b)
    C = sdb.backend.gemm_nt_bf16(Xt, Wt, bt)
    got = _np(C)
    assert np.isfinite(got).all()
    assert rel_fro(got[g["rows"]], g["C"]) <= TOL_BF16
    rows = np.sort(np.random.default_rng(1).choice(4096, 512, replace=False))
    want = orc.gemm_nt_bf16(np.ascontiguousarray(X[rows]), Wh, b)
    assert rel_fro(got[rows], want) <= TOL_BF16
    C2 = sdb.backend.gemm_nt_bf16(Xt, Wt, bt)
    assert torch.equal(C, C2), "GEMM is not deterministic"
    C3 = C.clone()
    sdb.backend.gemm_nt_bf16(Xt, Wt, None, C3, accumulate=True)
    exp = C.double() * 2 - bt.double()
    assert float(((C3.double() - exp).norm() / exp.norm()).item()) <= 1e-6


@pytest.mark.parametrize("M,N,K", [(4224, 3840, 3840), (4224, 3840, 10240), (128, 3840, 2560)])
def test_dit_shapes_sampled(sdb, orc, M, N, K):
    """Z-Image block GEMM shapes at 1024^2 (q/k/v/out, w2, cap_embed), 256 rows checked."""
    rng = np.random.default_rng(N + K)
    X = rng.standard_normal((M, K), dtype=np.float32)
    Wh = orc.to_bf16((0.02 * rng.standard_normal((N, K), dtype=np.float32)).astype(np.float32))
    got = _np(sdb.backend.gemm_nt_bf16(_t(X), _bf16_t(Wh)))
    rows = np.sort(np.random.default_rng(2).choice(M, min(M, 256), replace=False))
    want = orc.gemm_nt_bf16(np.ascontiguousarray(X[rows]), Wh)
    assert rel_fro(got[rows], want) <= TOL_BF16


@pytest.mark.parametrize("N,K", [(11520, 3840), (20480, 3840), (3840, 10240)])
def test_dit_shapes_full_output_vs_reference(sdb, ref, N, K):
    """Every output element of the Z-Image block GEMMs of one 1024^2 image (M = 4224 rows:
    the fused q/k/v projection, the w1/w3 pair, w2) against the reference's own CPU
    gemm_nt_bf16 (tensor.cpp:412-474, compiled from its sources, all host cores): the
    per-GEMM gate on whole outputs, not on sampled rows."""
    M = 4224
    ref.set_num_threads(0)
    rng = np.random.default_rng(N + 3 * K)
    X = rng.standard_normal((M, K), dtype=np.float32)
    Wh = ref.to_bf16((0.02 * rng.standard_normal((N, K), dtype=np.float32)).astype(np.float32))
    bias = (0.01 * rng.standard_normal(N)).astype(np.float32)
    got = _np(sdb.backend.gemm_nt_bf16(_t(X), _bf16_t(Wh), _t(bias)))
    want = ref.gemm_nt_bf16(X, Wh, bias)
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= TOL_BF16


@pytest.mark.parametrize("epi", [1, 2])
@pytest.mark.parametrize("y_bf16", [False, True])
def test_fused_gated_epilogue(sdb, orc, epi, y_bf16):
    """SwiGLU (w1/w3 interleaved, zimage.cpp:130) and GEGLU (modules.cpp:65) fused into
    the GEMM epilogue vs GEMM + activation on the CPU reference path."""
    import torch

    rng = np.random.default_rng(11 + epi)
    M, D, K = 300, 320, 256
    A = rng.standard_normal((M, K)).astype(np.float32)
    W1 = orc.to_bf16((0.05 * rng.standard_normal((D, K))).astype(np.float32))
    W2 = orc.to_bf16((0.05 * rng.standard_normal((D, K))).astype(np.float32))
    b1 = rng.standard_normal(D).astype(np.float32)
    b2 = rng.standard_normal(D).astype(np.float32)
    y1 = orc.gemm_nt_bf16(A, W1, b1)
    y2 = orc.gemm_nt_bf16(A, W2, b2)
    if epi == 1:
        want = orc.swiglu(y1, y2)
    else:
        want = orc.geglu(np.concatenate([y1, y2], axis=1))
    Wi = sdb.backend.interleave_gated(_bf16_t(W1), _bf16_t(W2))
    bi = sdb.backend.interleave_gated(_t(b1), _t(b2))
    Y = sdb.backend.gemm_bf16_epilogue(_t(A), Wi, bi, epi=epi, y_bf16=y_bf16)
    got = _np(Y.float()) if y_bf16 else _np(Y)
    tol = TOL_BF16 + (4e-3 if y_bf16 else 0.0)  # + bf16 rounding of the stored output
    assert rel_fro(got, want) <= tol
    del torch


def test_no_device_wait_expired(sdb):
    assert sdb.backend.device_error_word() == 0
    sdb.backend.synchronize()


@pytest.mark.parametrize("M,N,K,f32", [(128, 3840, 10240, False), (128, 3840, 2560, False), (77, 1000, 3000, False),
                                       (200, 1000, 4096, True)])
def test_gemm_split_k(sdb, orc, M, N, K, f32):
    """Few-tile, long-K GEMMs (the context refiner and caption embedder at one image: M =
    128 text tokens against 3840 x 10240 / 3840 x 2560 weights) run as split-K: each K
    split of each tile on its own SM, partial tiles added in split order with the bias by a
    reduction kernel. Checked against the oracle (bias, accumulate, padded ldc), for
    determinism, and against the unsplit kernel (forced tile width; same operands, only the
    fp32 summation order differs)."""
    import torch

    rng = np.random.default_rng(M + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    bias = (0.01 * rng.standard_normal(N)).astype(np.float32)
    C0 = rng.standard_normal((M, N + 4)).astype(np.float32)
    rows = np.sort(np.random.default_rng(K).choice(M, 24, replace=False))
    be = sdb.backend
    if f32:
        Wd = _t(W)
        run = lambda C, acc, b: be.gemm_nt_f32(_t(A), Wd, b, C, acc, M=M, N=N, K=K, ldc=N + 4)  # noqa: E731
        want = orc.gemm_nt(np.ascontiguousarray(A[rows]), W, bias, C0[rows], len(rows), N, K)
        tol = TOL_TF32
    else:
        Wh = orc.to_bf16(W)
        Wd = _bf16_t(Wh)
        run = lambda C, acc, b: be.gemm_nt_bf16(_t(A), Wd, b, C, acc, M=M, N=N, K=K, ldc=N + 4)  # noqa: E731
        want = orc.gemm_nt_bf16(np.ascontiguousarray(A[rows]), Wh, bias, C0[rows], len(rows), N, K)
        tol = TOL_BF16
    C = _t(C0)
    run(C, True, _t(bias))
    got = _np(C)
    assert rel_fro(got[rows, :N], want[:, :N]) <= tol
    assert np.array_equal(got[:, N:], C0[:, N:])  # padding columns untouched
    C2 = _t(C0)
    run(C2, True, _t(bias))
    assert torch.equal(C, C2)  # deterministic
    sdb.check(sdb.lib().sdb200_set_gemm_tile(256))
    C3 = _t(C0)
    run(C3, True, _t(bias))
    sdb.check(sdb.lib().sdb200_set_gemm_tile(0))
    assert rel_fro(got[:, :N], _np(C3)[:, :N]) <= TOL_EXACT


@pytest.mark.parametrize("M", [1, 3, 16])
@pytest.mark.parametrize("N,K,pad,f32", [(15360, 256, 0, False), (3841, 1000, 0, False), (1001, 2560, 3, False),
                                         (777, 320, 0, True), (500, 700, 1, True)])
def test_gemv_small_m(sdb, orc, M, N, K, pad, f32):
    """M <= 16: the memory-bound GEMV (exact fp32 A, weights read once; the adaLN
    modulation is M = 1, N = 15360, K = 256). Ragged N, a K tail outside the 16-byte body,
    and a weight pitch that rules the vector loads out; bias and accumulate."""
    rng = np.random.default_rng(M * 7 + N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    W = (0.02 * rng.standard_normal((N, K + pad))).astype(np.float32)
    bias = (0.01 * rng.standard_normal(N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    be = sdb.backend
    C = _t(C0)
    if f32:
        want = orc.gemm_nt(A, W, bias, C0, M, N, K, ldb=K + pad)
        be.gemm_nt_f32(_t(A), _t(W), _t(bias), C, True, M=M, N=N, K=K, ldb=K + pad)
    else:
        Wh = orc.to_bf16(W)
        want = orc.gemm_nt_bf16(A, Wh, bias, C0, M, N, K, ldb=K + pad)
        be.gemm_nt_bf16(_t(A), _bf16_t(Wh), _t(bias), C, True, M=M, N=N, K=K, ldb=K + pad)
    assert rel_fro(_np(C), want) <= TOL_EXACT


def _qkv_rope_oracle(orc, X, Wh, bias, Dq, cos, sin, gq, gk, eps, rows):
    """The reference's sequence for the fused projection (zimage.cpp:113-120): linear,
    rms_norm_heads, then rope() with the interleaved pairs, on the given rows only (row m
    at position m % S)."""
    y = orc.gemm_nt_bf16(np.ascontiguousarray(X[rows]), Wh, bias)
    pos = rows % cos.shape[0]
    out = []
    for part, g in ((0, gq), (1, gk)):
        x = orc.rms_norm_heads(y[:, part * Dq:(part + 1) * Dq], 128, g, eps)
        out.append(orc.rope(x[None], 128, cos[pos], sin[pos], True)[0])
    out.append(y[:, 2 * Dq:])
    return out


@pytest.mark.parametrize("case", ["bf16_x", "f32_x", "unaligned_gamma", "zimage_1024"])
def test_fused_qkv_rope_epilogue(sdb, orc, case):
    """sdb200_gemm_bf16_qkv_rope (the DiT's QKV projection with QK-norm, RoPE and the fp16
    attention-operand pack in the GEMM epilogue) against the reference's separate linear,
    rms_norm_heads and rope on the CPU oracle. With bf16 X both sides use the same operand
    values, so the gate is the fp16 rounding of the outputs (1e-3); with fp32 X the GEMM
    gate applies (2e-3) plus the fp16 rounding. Covers ragged M, rows wrapping the rotary
    table (S < M), bias, absent and unaligned gammas, and the Z-Image width at 1024^2
    (30 heads, 4224 tokens, sampled rows)."""
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    rng = np.random.default_rng({"bf16_x": 1, "f32_x": 2, "unaligned_gamma": 3, "zimage_1024": 4}[case])
    if case == "zimage_1024":
        M, K, Dq, S = 4224, 3840, 3840, 4224
    else:
        M, K, Dq, S = 300, 256, 256, 150
    eps = 1e-5
    X = rng.standard_normal((M, K)).astype(np.float32)
    if case != "f32_x":
        X = f32_to_bf16_bits(X).astype(np.uint32) << 16
        X = X.view(np.float32)
    Wh = f32_to_bf16_bits((0.02 * rng.standard_normal((3 * Dq, K))).astype(np.float32))
    bias = (0.05 * rng.standard_normal(3 * Dq)).astype(np.float32)
    ang = rng.uniform(0.0, 40.0, (S, 64))
    cos = np.repeat(np.cos(ang), 2, axis=1).astype(np.float32)
    sin = np.repeat(np.sin(ang), 2, axis=1).astype(np.float32)
    gq = (1.0 + 0.3 * rng.standard_normal(128)).astype(np.float32)
    gk = (1.0 + 0.3 * rng.standard_normal(128)).astype(np.float32)
    if case == "f32_x":
        gq = gk = None
    Xd = _t(X) if case == "f32_x" else _t(X).to(torch.bfloat16)
    if case == "unaligned_gamma":
        buf = _t(np.concatenate([[0.0], gq, gk]).astype(np.float32))
        gqd, gkd = buf[1:129], buf[129:257]  # 4-byte aligned only: the per-element gamma loads
    else:
        gqd = None if gq is None else _t(gq)
        gkd = None if gk is None else _t(gk)
    q, k, v = sdb.backend.gemm_bf16_qkv_rope(Xd, _bf16_t(Wh), _t(cos), _t(sin), gqd, gkd, _t(bias), eps)
    rows = np.arange(M) if M <= 1024 else np.sort(np.random.default_rng(9).choice(M, 64, replace=False))
    want = _qkv_rope_oracle(orc, X, Wh, bias, Dq, cos, sin, gq, gk, eps, rows)
    tol = 1e-3 if case != "f32_x" else TOL_BF16 + 1e-3
    for name, got, w in zip("qkv", (q, k, v), want):
        g = _np(got).astype(np.float32)[rows]
        assert np.isfinite(g).all(), name
        assert rel_fro(g, w) <= tol, (case, name, rel_fro(g, w))
    assert sdb.backend.device_error_word() == 0


@pytest.mark.parametrize("epi,y_bf16", [(0, False), (0, True), (1, True)])
def test_epilogue_bias_alignment_paths(sdb, epi, y_bf16):
    """The epilogue adds the bias with float4 loads when it is 16-byte aligned and per
    element otherwise; both add the same values in the same order, so the outputs must be
    bit-identical. The ragged N (not a multiple of 32 output columns for epi 0) also covers
    the masked tail chunk."""
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    rng = np.random.default_rng(31 + epi)
    M, K = 260, 192
    N = 1000 if epi == 0 else 1024
    A = _t(rng.standard_normal((M, K)).astype(np.float32))
    W = _bf16_t(f32_to_bf16_bits((0.05 * rng.standard_normal((N, K))).astype(np.float32)))
    b = rng.standard_normal(N).astype(np.float32)
    aligned = _t(b)
    buf = _t(np.concatenate([[0.0], b]).astype(np.float32))
    unaligned = buf[1:]
    assert unaligned.data_ptr() % 16 != 0
    y0 = sdb.backend.gemm_bf16_epilogue(A, W, aligned, epi=epi, y_bf16=y_bf16)
    y1 = sdb.backend.gemm_bf16_epilogue(A, W, unaligned, epi=epi, y_bf16=y_bf16)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)


def test_gemm_output_beyond_2g_elements(sdb, orc):
    """An output of more than 2^31 elements (65541 x 33000 fp32, 8.65 GB): every store
    offset past 2^31 must be formed in 64 bits. Sampled rows, the last ones included, are
    checked against the oracle at the GEMM gate."""
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    M, N, K = 65541, 33000, 64
    if torch.cuda.mem_get_info()[0] < 12 * (1 << 30):
        pytest.skip("needs 12 GB of free device memory")
    rng = np.random.default_rng(77)
    A = rng.standard_normal((M, K)).astype(np.float32)
    Wh = f32_to_bf16_bits((0.05 * rng.standard_normal((N, K))).astype(np.float32))
    bias = (0.1 * rng.standard_normal(N)).astype(np.float32)
    C = torch.empty((M, N), device="cuda")
    sdb.backend.gemm_nt_bf16(_t(A), _bf16_t(Wh), _t(bias), C=C, M=M, N=N, K=K, lda=K, ldb=K, ldc=N)
    rows = np.concatenate([np.sort(rng.choice(M - 8, 24, replace=False)), np.arange(M - 8, M)])
    got = _np(C[torch.from_numpy(rows).cuda()])
    del C
    torch.cuda.empty_cache()
    want = orc.gemm_nt_bf16(np.ascontiguousarray(A[rows]), Wh, bias)
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= TOL_BF16
