"""Generates the golden vectors under tests/golden/ from the reference itself.

Runs the reference's own CPU path (StableDiffusion-cpp src/tensor.cpp, compiled from
its sources by oracle/Makefile into oracle/_ref/libsdref.so) on seeded inputs and
stores inputs + outputs as small .npz fixtures. The cases mirror the reference's
kernel tests (tests/test_ops.cpp:481-505: odd sizes, padded leading dimensions,
bias / accumulate, causal and grouped-query attention, both RoPE conventions) plus a
sample of BASELINE config 1 (the fused-QKV bf16 GEMM, seed 0).

Run in a container that has the reference tree:  python tests/golden/make_golden.py
(`python tests/golden/make_golden.py flow` writes only the sampler fixture). The fixtures
it writes are committed; the tests never need the reference at run time.
"""
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "stablediffusion-cpp_b200"))

from oracle import REF_SO, RefCPU  # noqa: E402
from sdb200.workloads import cfg1_inputs  # noqa: E402,F401  (seeded BASELINE config 1 inputs)


def rn(rng, *shape, scale=1.0):
    return (scale * rng.standard_normal(shape)).astype(np.float32)


def main():
    if not os.path.exists(REF_SO):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    ref = RefCPU()
    rng = np.random.default_rng(1234)
    out = {}

    # gemm_nt, test_ops.cpp:35-54 shapes, padded ld: lda=K+3, ldb=K+5, ldc=N+2
    for i, (M, N, K, bias, acc) in enumerate(
        [(4, 4, 4, 0, 0), (37, 53, 129, 1, 0), (70, 130, 300, 0, 1), (1, 77, 40, 1, 0), (129, 5, 1000, 1, 1),
         (200, 300, 96, 1, 0)]):
        A = rn(rng, M, K + 3)
        B = rn(rng, N, K + 5)
        C0 = rn(rng, M, N + 2)
        bv = rn(rng, N)
        Cm = ref.gemm_nt(A, B, bv if bias else None, C0 if acc else None, M, N, K, ldc=N + 2)
        np.savez(os.path.join(HERE, f"gemm_{i}.npz"), A=A, B=B, C0=C0, bias=bv, C=Cm,
                 dims=np.array([M, N, K, bias, acc]))

    # gemm_nt_bf16, test_ops.cpp:157-169 shapes (+ bias)
    for i, (M, N, K) in enumerate([(37, 53, 129), (130, 257, 300), (300, 500, 200)]):
        A = rn(rng, M, K)
        Bh = ref.to_bf16(rn(rng, N, K))
        bv = rn(rng, N)
        Cm = ref.gemm_nt_bf16(A, Bh, bv)
        np.savez(os.path.join(HERE, f"gemm_bf16_{i}.npz"), A=A, Bh=Bh, bias=bv, C=Cm, dims=np.array([M, N, K]))

    # BASELINE config 1 sample: rows 0..7 and 4088..4095 of the full 4096 x 11520 x 3840 GEMM
    X, W, b = cfg1_inputs()
    Wh = ref.to_bf16(W)
    rows = np.r_[0:8, 4088:4096]
    Cs = ref.gemm_nt_bf16(np.ascontiguousarray(X[rows]), Wh, b)
    np.savez(os.path.join(HERE, "cfg1_rows.npz"), rows=rows, C=Cs,
             x_sum=np.float64(X.astype(np.float64).sum()), w_sum=np.float64(Wh.astype(np.float64).sum()))

    # attention, test_ops.cpp:85-115 and :260-277, :439-451 shapes
    for i, (N, Sq, Skv, H, KVH, d, causal) in enumerate(
        [(2, 9, 9, 3, 3, 8, 0), (1, 11, 5, 2, 2, 4, 0), (1, 7, 7, 1, 1, 16, 1), (1, 6, 6, 4, 2, 4, 1),
         (2, 37, 37, 8, 2, 16, 1), (1, 100, 100, 2, 2, 32, 0), (1, 150, 150, 2, 2, 128, 0),
         (1, 130, 77, 8, 8, 40, 0)]):
        q = rn(rng, N, Sq, H * d)
        k = rn(rng, N, Skv, KVH * d)
        v = rn(rng, N, Skv, KVH * d)
        o = ref.attention(q, k, v, H, KVH, bool(causal))
        np.savez(os.path.join(HERE, f"attention_{i}.npz"), q=q, k=k, v=v, out=o,
                 dims=np.array([N, Sq, Skv, H, KVH, d, causal]))

    # norms, rope, gated activations, softmax (test_ops.cpp:119-257)
    x = rn(rng, 5, 24)
    g24 = rn(rng, 24)
    g8 = rn(rng, 8)
    out["rms_x"], out["rms_g"] = x, g24
    out["rms_y"] = ref.rms_norm(x, g24, 1e-6)
    z = rn(rng, 21, 64)
    g64, b64 = rn(rng, 64), rn(rng, 64)
    out["ln_x"], out["ln_g"], out["ln_b"] = z, g64, b64
    out["ln_y"] = ref.layer_norm(z, g64, b64, 1e-5)
    out["ln_y_noaff"] = ref.layer_norm(z, None, None, 1e-6)
    out["rmsh_y"] = ref.rms_norm_heads(x, 8, g8, 1e-6)
    out["rmsh_g"] = g8
    S, H, D = 5, 3, 8
    xr = rn(rng, 1, S, H * D)
    cs = np.cos(0.1 * np.arange(S)[:, None] * (np.arange(D)[None, :] % (D // 2) + 1)).astype(np.float32)
    sn = np.sin(0.1 * np.arange(S)[:, None] * (np.arange(D)[None, :] % (D // 2) + 1)).astype(np.float32)
    out["rope_x"], out["rope_cos"], out["rope_sin"] = xr, cs, sn
    out["rope_half"] = ref.rope(xr, D, cs, sn, False)
    out["rope_inter"] = ref.rope(xr, D, cs, sn, True)
    gg, uu = rn(rng, 1000), rn(rng, 1000)
    out["swiglu_g"], out["swiglu_u"] = gg, uu
    out["swiglu_y"] = ref.swiglu(gg, uu)
    ge = rn(rng, 6, 40)
    out["geglu_x"], out["geglu_y"] = ge, ref.geglu(ge)
    sm = rn(rng, 12, 33)
    out["softmax_x"] = sm
    out["softmax_y"] = ref.softmax_rows(sm, 0.37, False)
    out["softmax_y_causal"] = ref.softmax_rows(sm, 0.37, True)
    gx = rn(rng, 2, 64, 5, 7)
    out["gn_x"], out["gn_g"], out["gn_b"] = gx, g64, b64
    out["gn_y"] = ref.group_norm(gx, 32, g64, b64, 1e-6)
    ma = rn(rng, 4, 6)
    mv, my = rn(rng, 6), rn(rng, 4, 6)
    out["rows_x"], out["rows_v"], out["rows_y"] = ma, mv, my
    out["mul_rows"] = ref.mul_rows(ma, mv)
    out["add_rows_scaled"] = ref.add_rows_scaled(ma, my, mv)
    # bf16 rounding incl. ties, inf, NaN, denormals (tensor.cpp:114-121)
    special = np.array([0.0, -0.0, 1.0, -1.5, 3.14159, 1e-3, 65504.0, 1e-30, 1e-40, np.inf, -np.inf, np.nan,
                        1.00390625, 1.01171875, -1.00390625, 3.4e38], np.float32)
    special = np.concatenate([special, rn(rng, 1000) * 100])
    out["bf16_in"], out["bf16_out"] = special, ref.to_bf16(special)
    np.savez(os.path.join(HERE, "layers.npz"), **out)

    # conv2d, test_ops.cpp:57-82 shapes
    for i, (N, Cin, Cout, H, W, k, stride) in enumerate(
        [(2, 3, 5, 9, 11, 3, 1), (1, 4, 6, 8, 8, 3, 2), (1, 7, 3, 5, 6, 1, 1), (2, 5, 6, 9, 11, 3, 2)]):
        x = rn(rng, N, Cin, H, W)
        w = rn(rng, Cout, Cin, k, k)
        b = rn(rng, Cout)
        pad = (k - 1) // 2
        y = ref.conv2d(x, w, b, stride, pad)
        np.savez(os.path.join(HERE, f"conv2d_{i}.npz"), x=x, w=w, b=b, y=y, dims=np.array([stride, pad]))
    # Z-Image transformer (zimage.cpp:138-228), small seeded config; the weights are
    # regenerated from the seed by the tests (sdb200.zimage.random_weights_numpy)
    from sdb200.zimage import ZConfig, random_weights_numpy

    for name, cfg, B_lat, L, t in [
        ("zimage_small", ZConfig(dim=256, heads=2, ffn=512, t_dim=256, t_hidden=512, cap_dim=128, layers=2,
                                 noise_refiners=1, context_refiners=1), (1, 16, 16, 16), 20, 0.6),
    ]:
        w, bf = random_weights_numpy(cfg, 0)
        zr = np.random.default_rng(1)
        x = zr.standard_normal(B_lat).astype(np.float32)
        cap = zr.standard_normal((1, L, cfg.cap_dim)).astype(np.float32)
        model = ref.zimage(w, bf, heads=cfg.heads)
        np.savez(os.path.join(HERE, f"{name}.npz"), x=x, cap=cap, t=np.float32(t), out=model(x, t, cap))
    flow(ref)
    print("golden vectors written to", HERE)


# Steps and shifts of the flow-matching schedule fixture (scheduler.cpp:117-127).
FLOW_STEPS = tuple(range(1, 41))
FLOW_SHIFTS = (0.5, 1.0, 2.0, 3.0, 6.0)


def flow(ref):
    """The reference's FlowMatchScheduler sigmas for every (steps, shift) pair, and one
    guided sampler update (pipeline.cpp:237-243) on seeded data."""
    sig = np.zeros((len(FLOW_STEPS), len(FLOW_SHIFTS), max(FLOW_STEPS) + 1), np.float32)
    for i, steps in enumerate(FLOW_STEPS):
        for j, shift in enumerate(FLOW_SHIFTS):
            sig[i, j, :steps + 1] = ref.flow_sigmas(steps, shift)
    rng = np.random.default_rng(77)
    x, o, neg = rn(rng, 4096), rn(rng, 4096), rn(rng, 4096)
    x_plain = ref.flow_step(x, o, None, 0.0, 2, 8, 3.0)
    x_cfg = ref.flow_step(x, o, neg, 2.5, 5, 8, 3.0)
    np.savez(os.path.join(HERE, "flow_sampler.npz"), sig=sig, steps=np.array(FLOW_STEPS), shifts=np.array(FLOW_SHIFTS),
             x=x, out=o, neg=neg, x_plain=x_plain, x_cfg=x_cfg)


if __name__ == "__main__":
    if sys.argv[1:] == ["flow"]:  # only the sampler fixture
        flow(RefCPU())
    else:
        main()
