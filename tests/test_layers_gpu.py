"""GPU parity of attention and of the layer / elementwise / layout ops against the
golden vectors the reference produced, through the C ABI.

Tolerances follow the reference's own GPU-vs-CPU checks (tests/test_ops.cpp:356-477):
norms 1e-4, rope / swiglu / geglu / activations 1e-5, row helpers 1e-6, layout ops
exact. conv2d runs on the tf32 tensor-core GEMM, so it is held to the GEMM gate
(relative Frobenius <= 2e-3) instead of the reference's fp32-SGEMM 1e-3 abs.
"""
import glob
import os

import numpy as np
import pytest

from conftest import GOLDEN, load_golden, rel_fro

pytestmark = pytest.mark.gpu


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture
def attention_path(sdb):
    """Selects the attention kernel for one test and restores the default after."""
    def use(path):
        sdb.check(sdb.lib().sdb200_set_attention_path(path))
    yield use
    sdb.check(sdb.lib().sdb200_set_attention_path(0))


def test_golden_attention_exact_path(sdb, attention_path):
    """fp32 streaming kernel: the reference's own GPU tolerance (test_ops.cpp:439-451, 1e-4)."""
    attention_path(1)
    for f in sorted(glob.glob(os.path.join(GOLDEN, "attention_*.npz"))):
        g = np.load(f)
        N, Sq, Skv, H, KVH, d, causal = (int(v) for v in g["dims"])
        o = sdb.backend.attention(_t(g["q"]), _t(g["k"]), _t(g["v"]), H, bool(causal), KVH)
        assert np.abs(_np(o) - g["out"]).max() <= 1e-4, f


def test_golden_attention_tensor_cores(sdb, attention_path):
    """tcgen05 kernel (fp16 operands, fp32 softmax/accumulate): relative Frobenius <= 2e-3,
    the per-contraction parity gate. Covers MHA, causal, GQA 4/2 and 8/2, head dims 4..128
    (padded to 64/128), Skv != Sq and ragged tiles."""
    attention_path(0)
    for f in sorted(glob.glob(os.path.join(GOLDEN, "attention_*.npz"))):
        g = np.load(f)
        N, Sq, Skv, H, KVH, d, causal = (int(v) for v in g["dims"])
        o = sdb.backend.attention(_t(g["q"]), _t(g["k"]), _t(g["v"]), H, bool(causal), KVH)
        assert rel_fro(_np(o), g["out"]) <= 2e-3, f


@pytest.mark.parametrize("path", [0, 1])
@pytest.mark.parametrize("d", [40, 128, 160])
def test_attention_no_keys_is_zero(sdb, orc, attention_path, path, d):
    """Skv = 0: the reference's score matrix is empty and its P V product a K = 0 GEMM, so
    the output is zero (the oracle agrees). Every path (flash kernel, wide-head GEMM form,
    exact kernel) writes zeros over whatever the buffer held; N = 0 and Sq = 0 are no-ops."""
    import torch

    attention_path(path)
    L = sdb.lib()
    N, Sq, H, KVH = 2, 37, 4, 2
    q = torch.randn((N, Sq, H * d), device="cuda")
    k = torch.empty((N, 0, KVH * d), device="cuda")
    out = torch.full((N, Sq, H * d), float("nan"), device="cuda")
    sdb.backend.bind_stream()
    for causal in (0, 1):
        out.fill_(float("nan"))
        sdb.check(L.sdb200_attention(q.data_ptr(), k.data_ptr(), k.data_ptr(), out.data_ptr(), N, Sq, 0, H, KVH, d,
                                     causal))
        torch.cuda.synchronize()
        assert torch.count_nonzero(out).item() == 0
    want = orc.attention(_np(q), np.zeros((N, 0, KVH * d), np.float32), np.zeros((N, 0, KVH * d), np.float32), H,
                         KVH, False)
    assert np.array_equal(_np(out), want)
    out.fill_(7.0)
    sdb.check(L.sdb200_attention(q.data_ptr(), k.data_ptr(), k.data_ptr(), out.data_ptr(), 0, Sq, 5, H, KVH, d, 0))
    sdb.check(L.sdb200_attention(q.data_ptr(), k.data_ptr(), k.data_ptr(), out.data_ptr(), N, 0, 5, H, KVH, d, 0))
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())
    if d <= 128:  # the fp16-operand entry point
        dp = 64 if d <= 64 else 128
        for bf16 in (0, 1):
            o = torch.full((N * Sq * H * d,), -1, dtype=torch.int16 if bf16 else torch.int32, device="cuda")
            sdb.check(L.sdb200_attention_f16(q.data_ptr(), k.data_ptr(), k.data_ptr(), o.data_ptr(), bf16, N, Sq, 0, H,
                                             KVH, d, dp, 0))
            torch.cuda.synchronize()
            assert torch.count_nonzero(o).item() == 0


@pytest.mark.parametrize("N,Sq,Skv,H,KVH,d,causal", [
    (1, 4224, 4224, 4, 4, 128, False),   # Z-Image joint sequence at 1024^2 (4 of 30 heads)
    (1, 640, 640, 30, 30, 128, False),   # all 30 heads, shorter sequence
    (2, 300, 300, 32, 8, 128, True),     # Qwen3-like GQA 32/8, causal
    (1, 1024, 77, 8, 8, 40, False),      # SD1.5 cross-attention (d=40 padded to 64)
    (2, 1000, 1000, 8, 8, 40, False),    # SD1.5 self-attention, ragged tiles
    (1, 129, 700, 2, 1, 64, True),       # Skv > Sq, causal, 2/1 GQA
])
def test_attention_tensor_cores_vs_oracle(sdb, orc, attention_path, N, Sq, Skv, H, KVH, d, causal):
    attention_path(0)
    rng = np.random.default_rng(Sq + Skv + H)
    q = rng.standard_normal((N, Sq, H * d)).astype(np.float32)
    k = rng.standard_normal((N, Skv, KVH * d)).astype(np.float32)
    v = rng.standard_normal((N, Skv, KVH * d)).astype(np.float32)
    want = orc.attention(q, k, v, H, KVH, causal)
    got = _np(sdb.backend.attention(_t(q), _t(k), _t(v), H, causal, KVH))
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= 2e-3


def test_attention_d256_paths(sdb, orc, attention_path):
    """Head dims above 128: tf32 GEMMs around a softmax by default (GEMM gate), the exact
    fp32 kernel on path 1 (the reference's 1e-4)."""
    rng = np.random.default_rng(12)
    q = rng.standard_normal((1, 40, 2 * 256)).astype(np.float32)
    k = rng.standard_normal((1, 50, 2 * 256)).astype(np.float32)
    v = rng.standard_normal((1, 50, 2 * 256)).astype(np.float32)
    want = orc.attention(q, k, v, 2, 2, False)
    got = _np(sdb.backend.attention(_t(q), _t(k), _t(v), 2))
    assert rel_fro(got, want) <= 2e-3
    attention_path(1)
    got = _np(sdb.backend.attention(_t(q), _t(k), _t(v), 2))
    assert np.abs(got - want).max() <= 1e-4


@pytest.mark.parametrize("N,Sq,Skv,H,KVH,d,causal", [
    # small score matrices (N * heads * Sq * Skv <= 2^24): the exact streaming kernel
    (1, 1024, 1024, 1, 1, 512, False),   # the VAE mid-block attention shape at a reduced size
    (2, 130, 67, 4, 2, 160, True),       # GQA, causal, Skv not a multiple of 4
    (1, 7, 300, 3, 3, 200, False),       # few query rows
    # above that: tf32 GEMMs around the row softmax
    (1, 2100, 2100, 4, 2, 160, True),    # GQA, causal, Skv not a multiple of 4 (padded rows)
])
def test_attention_wide_heads_vs_oracle(sdb, orc, N, Sq, Skv, H, KVH, d, causal):
    rng = np.random.default_rng(Sq + d)
    q = rng.standard_normal((N, Sq, H * d)).astype(np.float32)
    k = rng.standard_normal((N, Skv, KVH * d)).astype(np.float32)
    v = rng.standard_normal((N, Skv, KVH * d)).astype(np.float32)
    got = _np(sdb.backend.attention(_t(q), _t(k), _t(v), H, causal=causal, kv_heads=KVH))
    want = orc.attention(q, k, v, H, KVH, causal)
    assert rel_fro(got, want) <= 2e-3


def test_attention_gemm_path_row_chunks(sdb, ref, attention_path):
    """Skv large enough that the 256 MB score block holds fewer rows than Sq: several
    query-row chunks, with the causal mask offset per chunk; against the reference's own
    CPU attention (tensor.cpp:771-810, compiled from its sources) and the exact kernel."""
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    Sq, Skv, d = 1000, 70000, 136
    q = torch.randn((1, Sq, d), generator=g, device="cuda")
    k = torch.randn((1, Skv, d), generator=g, device="cuda")
    v = torch.randn((1, Skv, d), generator=g, device="cuda")
    ref.set_num_threads(0)
    qh, kh, vh = _np(q), _np(k), _np(v)
    for causal in (False, True):
        attention_path(0)
        got = _np(sdb.backend.attention(q, k, v, 1, causal=causal))
        assert rel_fro(got, ref.attention(qh, kh, vh, 1, 1, causal)) <= 2e-3, causal
        attention_path(1)
        want = _np(sdb.backend.attention(q, k, v, 1, causal=causal))
        assert rel_fro(got, want) <= 2e-3, causal


@pytest.mark.parametrize("rows,C", [(1000, 320), (77, 1280), (40, 2048), (40, 2052), (33, 322)])
def test_row_norms_widths(sdb, rows, C):
    """LayerNorm / RMSNorm at the UNet's widths (one warp per row, the row in registers) and
    at widths that take the block-per-row kernel (C > 2048, C % 4 != 0), against float64."""
    be = sdb.backend
    rng = np.random.default_rng(C)
    x = (3.0 + 2.0 * rng.standard_normal((rows, C))).astype(np.float32)
    g = rng.standard_normal(C).astype(np.float32)
    b = rng.standard_normal(C).astype(np.float32)
    xd = x.astype(np.float64)
    mu = xd.mean(1, keepdims=True)
    ln = (xd - mu) / np.sqrt(((xd - mu) ** 2).mean(1, keepdims=True) + 1e-5) * g + b
    rms = xd / np.sqrt((xd ** 2).mean(1, keepdims=True) + 1e-6) * g
    assert np.abs(_np(be.layer_norm(_t(x), _t(g), _t(b), 1e-5)) - ln).max() <= 1e-4
    assert np.abs(_np(be.rms_norm(_t(x), _t(g), 1e-6)) - rms).max() <= 1e-4


def test_golden_layers(sdb):
    g = load_golden("layers")
    be = sdb.backend
    assert np.abs(_np(be.rms_norm(_t(g["rms_x"]), _t(g["rms_g"]), 1e-6)) - g["rms_y"]).max() <= 1e-4
    assert np.abs(_np(be.layer_norm(_t(g["ln_x"]), _t(g["ln_g"]), _t(g["ln_b"]), 1e-5)) - g["ln_y"]).max() <= 1e-4
    assert np.abs(_np(be.layer_norm(_t(g["ln_x"]), None, None, 1e-6)) - g["ln_y_noaff"]).max() <= 1e-4
    x = _t(g["rms_x"])
    be.rms_norm_heads_(x, 8, _t(g["rmsh_g"]), 1e-6)
    assert np.abs(_np(x) - g["rmsh_y"]).max() <= 1e-4
    for inter, key in ((False, "rope_half"), (True, "rope_inter")):
        x = _t(g["rope_x"])
        be.rope_(x, 8, _t(g["rope_cos"]), _t(g["rope_sin"]), inter)
        assert np.abs(_np(x) - g[key]).max() <= 1e-5, key
    assert np.abs(_np(be.swiglu(_t(g["swiglu_g"]), _t(g["swiglu_u"]))) - g["swiglu_y"]).max() <= 1e-5
    assert np.abs(_np(be.geglu(_t(g["geglu_x"]))) - g["geglu_y"]).max() <= 1e-5
    for causal, key in ((False, "softmax_y"), (True, "softmax_y_causal")):
        x = _t(g["softmax_x"])
        be.softmax_rows_(x, 0.37, causal)
        assert np.abs(_np(x) - g[key]).max() <= 1e-6, key
    assert np.abs(_np(be.group_norm(_t(g["gn_x"]), 32, _t(g["gn_g"]), _t(g["gn_b"]), 1e-6)) - g["gn_y"]).max() <= 1e-4
    x = _t(g["rows_x"])
    be.mul_rows_(x, _t(g["rows_v"]))
    assert np.abs(_np(x) - g["mul_rows"]).max() <= 1e-6
    x = _t(g["rows_x"])
    be.add_rows_scaled_(x, _t(g["rows_y"]), _t(g["rows_v"]))
    assert np.abs(_np(x) - g["add_rows_scaled"]).max() <= 1e-6


def test_golden_conv2d(sdb):
    for f in sorted(glob.glob(os.path.join(GOLDEN, "conv2d_*.npz"))):
        g = np.load(f)
        stride, pad = (int(v) for v in g["dims"])
        got = _np(sdb.backend.conv2d(_t(g["x"]), _t(g["w"]), _t(g["b"]), stride, pad))
        assert rel_fro(got, g["y"]) <= 2e-3, f


def test_conv2d_sd15_shape(sdb, orc):
    """BASELINE config 2 conv: 3x3, 320 -> 320 on a 64x64 latent (GEMM 320 x 4096 x 2880)."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 320, 64, 64)).astype(np.float32)
    w = (0.02 * rng.standard_normal((320, 320, 3, 3))).astype(np.float32)
    b = (0.02 * rng.standard_normal(320)).astype(np.float32)
    want = orc.conv2d(x, w, b, 1, 1)
    got = _np(sdb.backend.conv2d(_t(x), _t(w), _t(b), 1, 1))
    assert rel_fro(got, want) <= 2e-3


@pytest.fixture
def conv_setup(sdb):
    """Selects the conv2d lowering and GEMM tile width for one test; restores defaults."""
    def use(implicit, bn=0, pair=1):
        sdb.check(sdb.lib().sdb200_set_conv_implicit(1 if implicit else 0))
        sdb.check(sdb.lib().sdb200_set_gemm_tile(bn))
        sdb.check(sdb.lib().sdb200_set_gemm_pair(pair))
    yield use
    sdb.check(sdb.lib().sdb200_set_conv_implicit(1))
    sdb.check(sdb.lib().sdb200_set_gemm_tile(0))
    sdb.check(sdb.lib().sdb200_set_gemm_pair(1))


# (N, Cin, H, W, Cout, k, pad): ragged channel counts, Wo below and above 32, batches,
# 1x1 kernels, pad 2, a one-pixel image, and UNet / VAE channel widths.
CONV_CASES = [
    (1, 3, 5, 7, 8, 3, 1),
    (2, 40, 9, 33, 130, 3, 1),
    (1, 8, 70, 40, 5, 1, 0),
    (2, 5, 12, 20, 7, 3, 2),
    (1, 33, 17, 65, 129, 3, 1),
    (1, 4, 1, 1, 2, 3, 1),
    (1, 16, 48, 48, 512, 3, 1),
    (1, 128, 96, 96, 128, 3, 1),
    (2, 256, 24, 24, 128, 1, 0),
    (1, 64, 5, 300, 256, 3, 1),     # SM pairs: one-row 256-pixel rectangles split left / right
    (1, 40, 20, 70, 320, 3, 1),     # SM pairs: 128 x 2 rectangles split top / bottom, ragged Cout
    (2, 640, 8, 8, 1280, 3, 1),     # few tiles, long K (the UNet's deepest level): split-K
    (1, 1280, 16, 12, 640, 3, 1),   # split-K with a ragged pixel rectangle
    (2, 128, 45, 38, 3, 3, 1),      # few output channels (the VAE's conv_out): direct fp32 kernel
    (1, 20, 17, 19, 6, 5, 2),       # direct kernel, 5 x 5 taps
]


@pytest.mark.parametrize("case", CONV_CASES)
def test_conv2d_implicit_gemm(sdb, orc, conv_setup, case):
    """Stride-1 conv2d as an implicit GEMM (NHWC boxes by TMA, zero-filled halo) against the
    oracle's im2col convolution, at every tile width, and against the im2col lowering on
    the same tf32 tensor cores (same rounded operands: only the summation order differs)
    where that lowering uses them."""
    N, Cin, H, W, Cout, k, pad = case
    rng = np.random.default_rng(sum(case))
    x = rng.standard_normal((N, Cin, H, W)).astype(np.float32)
    w = (0.05 * rng.standard_normal((Cout, Cin, k, k))).astype(np.float32)
    b = (0.05 * rng.standard_normal(Cout)).astype(np.float32)
    want = orc.conv2d(x, w, b, 1, pad)
    conv_setup(False)
    lowered = _np(sdb.backend.conv2d(_t(x), _t(w), _t(b), 1, pad))
    # automatic choice, each single-SM tile width, and SM pairs wherever the shape allows
    for bn, pair in ((0, 1), (64, 1), (128, 1), (256, 1), (0, 2)):
        conv_setup(True, bn, pair)
        got = _np(sdb.backend.conv2d(_t(x), _t(w), _t(b), 1, pad))
        assert got.shape == want.shape
        assert rel_fro(got, want) <= 2e-3, (bn, pair)
        if Cout > 16:  # the lowering's GEMM runs on tf32 tensor cores (exact SIMT for M <= 16)
            # same rounded operands, fp32 sums in another order (split-K partials at K = 5760
            # differ by about 1e-5)
            assert rel_fro(got, lowered) <= 5e-5, (bn, pair)


def test_conv2d_nhwc_packed_with_residual(sdb, orc):
    """The packed-operand entry points: pack x (channel pitch above C) and w once, then
    out = conv + bias + res in one kernel; res is read in the output layout."""
    import torch

    rng = np.random.default_rng(21)
    N, Cin, H, W, Cout = 2, 37, 19, 45, 70
    x = rng.standard_normal((N, Cin, H, W)).astype(np.float32)
    w = (0.05 * rng.standard_normal((Cout, Cin, 3, 3))).astype(np.float32)
    b = (0.05 * rng.standard_normal(Cout)).astype(np.float32)
    res = rng.standard_normal((N, Cout, H, W)).astype(np.float32)
    want = orc.conv2d(x, w, b, 1, 1) + res
    cp, cq = 40, 64
    L = sdb.lib()
    xd, wd, bd, rd = _t(x), _t(w), _t(b), _t(res)
    xh = torch.empty(N * H * W * cp, device="cuda")
    wp = torch.empty(Cout * 9 * cq, device="cuda")
    out = torch.empty((N, Cout, H, W), device="cuda")
    sdb.check(L.sdb200_conv_pack_input(xd.data_ptr(), xh.data_ptr(), N, Cin, H * W, cp))
    sdb.check(L.sdb200_conv_pack_weight(wd.data_ptr(), wp.data_ptr(), Cout, Cin, 9, cq))
    sdb.check(L.sdb200_conv2d_nhwc(xh.data_ptr(), N, Cin, cp, H, W, wp.data_ptr(), cq, Cout, 3, 3, 1, bd.data_ptr(),
                                   rd.data_ptr(), out.data_ptr(), H, W))
    assert rel_fro(_np(out), want) <= 2e-3
    # a channel pitch that is not a multiple of 4 is refused before any launch
    assert L.sdb200_conv2d_nhwc(xh.data_ptr(), N, Cin, 38, H, W, wp.data_ptr(), cq, Cout, 3, 3, 1, None, None,
                                out.data_ptr(), H, W) != 0


@pytest.mark.parametrize("Cout,Cin,taps,cq", [
    (70, 37, 9, 64),     # channel pitch above Cin: zero columns
    (64, 320, 1, 320),   # 1 x 1
    (16, 2560, 9, 2560),  # 92 KB slab (opt-in shared memory)
    (8, 4000, 9, 4000),  # slab above the kernel's shared-memory bound: the gather form
])
def test_conv_pack_weight_layout(sdb, Cout, Cin, taps, cq):
    """w [Cout, Cin, taps] -> wp [Cout, taps, cq] rounded to tf32 (nearest even, low 13 bits
    cleared), zero for channels Cin..cq-1: bit-exact against numpy."""
    import torch

    rng = np.random.default_rng(Cin)
    w = rng.standard_normal((Cout, Cin, taps)).astype(np.float32)
    w.reshape(-1)[:4] = [np.inf, -np.inf, 1.0 + 2.0 ** -11, 1.0 + 3 * 2.0 ** -11]  # ties to even
    u = w.view(np.uint32)
    r = ((u + np.uint32(0xFFF) + ((u >> 13) & 1)) & np.uint32(0xFFFFE000)).view(np.float32)
    r = np.where(np.isinf(w), w, r)
    want = np.zeros((Cout, taps, cq), np.float32)
    want[:, :, :Cin] = r.transpose(0, 2, 1)
    wd = _t(w)
    wp = torch.full((Cout * taps * cq,), 7.0, device="cuda")
    sdb.check(sdb.lib().sdb200_conv_pack_weight(wd.data_ptr(), wp.data_ptr(), Cout, Cin, taps, cq))
    got = _np(wp).reshape(Cout, taps, cq)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_conv2d_nhwc_split_k_with_residual(sdb, orc):
    """A convolution with few output tiles and a long K runs as split-K; the reduction adds
    the bias and the residual (here the output buffer itself, in place)."""
    import torch

    rng = np.random.default_rng(23)
    N, Cin, H, W, Cout = 2, 1280, 8, 8, 1280
    x = rng.standard_normal((N, Cin, H, W)).astype(np.float32)
    w = (0.02 * rng.standard_normal((Cout, Cin, 3, 3))).astype(np.float32)
    b = (0.05 * rng.standard_normal(Cout)).astype(np.float32)
    res = rng.standard_normal((N, Cout, H, W)).astype(np.float32)
    want = orc.conv2d(x, w, b, 1, 1) + res
    L = sdb.lib()
    xd, wd, bd = _t(x), _t(w), _t(b)
    xh = torch.empty(N * H * W * Cin, device="cuda")
    wp = torch.empty(Cout * 9 * Cin, device="cuda")
    out = _t(res)  # residual = output, in place
    sdb.check(L.sdb200_conv_pack_input(xd.data_ptr(), xh.data_ptr(), N, Cin, H * W, Cin))
    sdb.check(L.sdb200_conv_pack_weight(wd.data_ptr(), wp.data_ptr(), Cout, Cin, 9, Cin))
    sdb.check(L.sdb200_conv2d_nhwc(xh.data_ptr(), N, Cin, Cin, H, W, wp.data_ptr(), Cin, Cout, 3, 3, 1, bd.data_ptr(),
                                   out.data_ptr(), out.data_ptr(), H, W))
    assert rel_fro(_np(out), want) <= 2e-3


def test_conv2d_strided_uses_im2col(sdb, orc):
    """Stride 2 (the UNet's downsamplers) keeps the im2col lowering."""
    rng = np.random.default_rng(11)
    x = rng.standard_normal((1, 64, 33, 31)).astype(np.float32)
    w = (0.05 * rng.standard_normal((96, 64, 3, 3))).astype(np.float32)
    b = (0.05 * rng.standard_normal(96)).astype(np.float32)
    want = orc.conv2d(x, w, b, 2, 1)
    got = _np(sdb.backend.conv2d(_t(x), _t(w), _t(b), 2, 1))
    assert rel_fro(got, want) <= 2e-3


@pytest.mark.parametrize("shape,groups", [
    ((1, 128, 256, 256), 32),   # VAE last-stage width: 4 channels x 65536 values per group
    ((2, 320, 37, 29), 32),     # odd plane (no 16-byte rows), several chunks per group
    ((1, 64, 3, 3), 32),        # groups smaller than one chunk
    ((3, 96, 17, 16), 8),       # one launch: the group in shared memory
    ((2, 320, 64, 64), 32),     # SD 1.x UNet groups at 512^2, one launch (160 KB group)
    ((2, 640, 32, 32), 32),
    ((2, 1280, 8, 8), 32),
])
def test_group_norm_split_statistics(sdb, orc, shape, groups):
    """GroupNorm with chunked statistics combined in double (large groups), or in one launch
    with the group in shared memory and two-pass fp32 statistics (groups up to 48K values),
    against the oracle's double two-pass statistics (the reference's GPU-vs-CPU norm
    tolerance, 1e-4)."""
    rng = np.random.default_rng(shape[1])
    # A large common offset makes single-pass fp32 statistics fail; the split form must not.
    x = (3.0 + rng.standard_normal(shape)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(shape[1])).astype(np.float32)
    beta = (0.1 * rng.standard_normal(shape[1])).astype(np.float32)
    want = orc.group_norm(x, groups, gamma, beta, 1e-6)
    got = _np(sdb.backend.group_norm(_t(x), groups, _t(gamma), _t(beta), 1e-6))
    assert np.abs(got - want).max() <= 1e-4


def test_elementwise_and_layout(sdb):
    import torch

    rng = np.random.default_rng(8)
    a = rng.standard_normal(1000).astype(np.float32)
    for name, fn in (("silu", lambda v: v / (1 + np.exp(-v))), ("tanh", np.tanh),
                     ("quick_gelu", lambda v: v / (1 + np.exp(-1.702 * v)))):
        x = _t(a)
        sdb.backend.unary_(name, x)
        assert np.abs(_np(x) - fn(a.astype(np.float64))).max() <= 1e-5, name
    L = sdb.lib()
    img = rng.standard_normal((2, 3, 4, 5)).astype(np.float32)
    x = _t(img)
    y = torch.empty((2, 20, 3), device="cuda")
    sdb.check(L.sdb200_nchw_to_nlc(x.data_ptr(), y.data_ptr(), 2, 3, 20))
    assert np.array_equal(_np(y), img.reshape(2, 3, 20).transpose(0, 2, 1))
    z = torch.empty_like(x)
    sdb.check(L.sdb200_nlc_to_nchw(y.data_ptr(), z.data_ptr(), 2, 3, 20))
    assert np.array_equal(_np(z), img)
    up = torch.empty((2, 3, 8, 10), device="cuda")
    sdb.check(L.sdb200_upsample_nearest2x(x.data_ptr(), up.data_ptr(), 6, 4, 5))
    assert np.array_equal(_np(up), img.repeat(2, axis=2).repeat(2, axis=3))
    lat = rng.standard_normal((16, 6, 8)).astype(np.float32)
    lt = _t(lat)
    tok = torch.empty((12, 64), device="cuda")
    sdb.check(L.sdb200_patchify(lt.data_ptr(), tok.data_ptr(), 16, 6, 8, 2))
    want = lat.reshape(16, 3, 2, 4, 2).transpose(1, 3, 2, 4, 0).reshape(12, 64)
    assert np.array_equal(_np(tok), want)
    back = torch.empty_like(lt)
    sdb.check(L.sdb200_unpatchify(tok.data_ptr(), back.data_ptr(), 16, 6, 8, 2))
    assert np.array_equal(_np(back), lat)


def test_empty_shapes_are_no_ops(sdb):
    """Zero-size problems through the C ABI return SDB200_OK and touch nothing, as the
    reference's CPU loops do (its GPU backend would launch an empty grid): GEMMs with M or N
    zero, convolution with no images, norms, softmax, RoPE and the value-wise and layout ops
    with no rows or elements."""
    import torch

    L = sdb.lib()
    buf = torch.full((4096,), 5.0, device="cuda")
    w16 = torch.zeros((4096,), dtype=torch.int16, device="cuda")
    p, h = buf.data_ptr(), w16.data_ptr()
    calls = [
        lambda: L.sdb200_gemm_nt_f32(0, 64, 32, p, 32, p, 32, p, 64, None, 0),
        lambda: L.sdb200_gemm_nt_f32(64, 0, 32, p, 32, p, 32, p, 1, None, 0),
        lambda: L.sdb200_gemm_nt_bf16(0, 64, 32, p, 32, h, 32, p, 64, None, 0),
        lambda: L.sdb200_gemm_nt_bf16(16, 0, 32, p, 32, h, 32, p, 1, None, 0),
        lambda: L.sdb200_conv2d(p, 0, 4, 8, 8, p, 4, 3, 3, None, 1, 1, p, 8, 8),
        lambda: L.sdb200_group_norm(p, p, 0, 32, 64, 32, p, p, 1e-6),
        lambda: L.sdb200_layer_norm(p, p, 0, 64, p, p, 1e-5),
        lambda: L.sdb200_rms_norm(p, p, 0, 64, p, 1e-5),
        lambda: L.sdb200_rms_norm_heads(p, 0, 64, p, 1e-5),
        lambda: L.sdb200_softmax_rows(p, 0, 64, 1.0, 0),
        lambda: L.sdb200_rope(p, 0, 8, 64, 64, p, p, 1),
        lambda: L.sdb200_geglu(p, p, 0, 32),
        lambda: L.sdb200_swiglu(p, p, p, 0),
        lambda: L.sdb200_silu(p, 0),
        lambda: L.sdb200_add(p, p, 0),
        lambda: L.sdb200_mul_rows(p, p, 0, 64),
        lambda: L.sdb200_add_channel_bias(p, p, 0, 4, 64),
        lambda: L.sdb200_upsample_nearest2x(p, p, 0, 8, 8),
        lambda: L.sdb200_nchw_to_nlc(p, p, 0, 4, 64),
    ]
    for i, call in enumerate(calls):
        rc = call()
        assert rc == sdb.OK, (i, rc, L.sdb200_last_error())
    torch.cuda.synchronize()
    assert bool((buf == 5.0).all())
    assert sdb.backend.device_error_word() == 0


def test_attention_output_beyond_2g_elements(sdb, orc, attention_path):
    """More than 2^31 output elements: 520 samples of the 1024^2 joint sequence (4224 tokens)
    with 8 heads of 128, 2.25 G elements (9 GB fp32) per tensor, so the last samples' offsets
    need 64 bits. Two heads of the first and the last sample are checked against the oracle
    at the contraction gate."""
    import torch

    attention_path(0)
    N, S, H, d = 520, 4224, 8, 128
    if torch.cuda.mem_get_info()[0] < 48 * (1 << 30):
        pytest.skip("needs 48 GB of free device memory")
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    q = torch.randn((N, S, H * d), generator=g, device="cuda")
    k = torch.randn((N, S, H * d), generator=g, device="cuda")
    v = torch.randn((N, S, H * d), generator=g, device="cuda")
    out = sdb.backend.attention(q, k, v, H, False, H)
    torch.cuda.synchronize()
    assert N * S * H * d > 2 ** 31
    for n in (0, N - 1):
        qs, ks, vs = (_np(t[n:n + 1, :, :2 * d]) for t in (q, k, v))  # heads 0 and 1
        want = orc.attention(qs, ks, vs, 2, 2, False)
        got = _np(out[n:n + 1, :, :2 * d])
        assert np.isfinite(got).all()
        assert rel_fro(got, want) <= 2e-3, n
    del q, k, v, out
    torch.cuda.empty_cache()
