"""TEST INFRASTRUCTURE ONLY: restatement of the reference's Z-Image transformer forward
(StableDiffusion-cpp src/zimage.cpp:71-228) composed from the C oracle kernels
(oracle.c: gemm_nt / gemm_nt_bf16, rms_norm, layer_norm, rms_norm_heads, rope,
attention, swiglu), used as the checker of the device DiT. It is pinned against the
reference ZImageTransformer compiled from its sources (tests/test_zimage_oracle.py).
"""
from __future__ import annotations

import numpy as np


class ZImageOracle:
    def __init__(self, orc, weights: dict, bf16_names: set, heads=30, patch=2, norm_eps=1e-5, rope_theta=256.0,
                 t_scale=1000.0, axes=(32, 48, 48)):
        self.o = orc
        self.w = weights
        self.bf16 = {n: orc.to_bf16(weights[n]) for n in bf16_names}
        self.heads, self.patch, self.eps = heads, patch, norm_eps
        self.theta, self.t_scale, self.axes = rope_theta, t_scale, axes
        self.D = weights["all_x_embedder.2-1.weight"].shape[0]
        self.hd = self.D // heads

    def has(self, n):
        return n in self.w

    # tensor.cpp:481-501 linear(); bf16 weights through gemm_nt_bf16, fp32 through gemm_nt
    def linear(self, x, prefix):
        W = self.w[prefix + ".weight"]
        b = self.w.get(prefix + ".bias")
        x2 = np.ascontiguousarray(x.reshape(-1, x.shape[-1]), np.float32)
        if prefix + ".weight" in self.bf16:
            y = self.o.gemm_nt_bf16(x2, self.bf16[prefix + ".weight"], b)
        else:
            y = self.o.gemm_nt(x2, W, b)
        return y.reshape(*x.shape[:-1], W.shape[0])

    # zimage.cpp:71-88 rope_tables(): double frequencies, float angle, float cos/sin
    def rope_tables(self, pos):
        S, d = len(pos), self.hd
        cs = np.zeros((S, d), np.float32)
        sn = np.zeros((S, d), np.float32)
        for s in range(S):
            off = 0
            for a in range(3):
                da = self.axes[a]
                k = np.arange(da // 2)
                freq = 1.0 / np.power(float(self.theta), (2.0 * k) / float(da))
                ang = (float(pos[s][a]) * freq).astype(np.float32)
                cs[s, off + 2 * k] = cs[s, off + 2 * k + 1] = np.cos(ang)
                sn[s, off + 2 * k] = sn[s, off + 2 * k + 1] = np.sin(ang)
                off += da
        return cs, sn

    # zimage.cpp:90-136 run_block()
    def run_block(self, p, x, cs, sn, adaln):
        D, o = self.D, self.o
        mod = None
        if self.has(p + ".adaLN_modulation.0.weight"):
            mod = self.linear(adaln, p + ".adaLN_modulation.0").reshape(4, D)
            scale_msa, gate_msa = mod[0] * 1.0 + 1.0, np.tanh(mod[1]).astype(np.float32)
            scale_mlp, gate_mlp = mod[2] * 1.0 + 1.0, np.tanh(mod[3]).astype(np.float32)
        h = o.rms_norm(x, self.w[p + ".attention_norm1.weight"], self.eps)
        if mod is not None:
            h = o.mul_rows(h, scale_msa.astype(np.float32))
        q = self.linear(h, p + ".attention.to_q")
        k = self.linear(h, p + ".attention.to_k")
        v = self.linear(h, p + ".attention.to_v")
        q = o.rms_norm_heads(q, self.hd, self.w[p + ".attention.norm_q.weight"], 1e-5)
        k = o.rms_norm_heads(k, self.hd, self.w[p + ".attention.norm_k.weight"], 1e-5)
        q = o.rope(q.reshape(1, -1, D), self.hd, cs, sn, True)
        k = o.rope(k.reshape(1, -1, D), self.hd, cs, sn, True)
        att = o.attention(q, k, v.reshape(1, -1, D), self.heads, self.heads, False)
        a = self.linear(att.reshape(-1, D), p + ".attention.to_out.0")
        a = o.rms_norm(a, self.w[p + ".attention_norm2.weight"], self.eps)
        x = o.add_rows_scaled(x, a, gate_msa) if mod is not None else (x + a).astype(np.float32)
        h = o.rms_norm(x, self.w[p + ".ffn_norm1.weight"], self.eps)
        if mod is not None:
            h = o.mul_rows(h, scale_mlp.astype(np.float32))
        f = self.linear(o.swiglu(self.linear(h, p + ".feed_forward.w1"), self.linear(h, p + ".feed_forward.w3")),
                        p + ".feed_forward.w2")
        f = o.rms_norm(f, self.w[p + ".ffn_norm2.weight"], self.eps)
        return o.add_rows_scaled(x, f, gate_mlp) if mod is not None else (x + f).astype(np.float32)

    # zimage.cpp:138-228 forward(): x [1, C, H, W], cap [1, L, capdim]
    def forward(self, x, t, cap):
        o, D, p = self.o, self.D, self.patch
        _, C, H, W = x.shape
        Ht, Wt = H // p, W // p
        n_img = Ht * Wt
        pad = lambda n: (n + 31) // 32 * 32  # noqa: E731
        n_img_pad, L = pad(n_img), cap.shape[1]
        n_cap_pad = pad(L)
        F = self.w["t_embedder.mlp.0.weight"].shape[1]
        half = F // 2
        tt = np.float32(t) * np.float32(self.t_scale)
        i = np.arange(half, dtype=np.float32)
        f = np.exp(-np.log(np.float32(10000.0)) * i / np.float32(half)).astype(np.float32)
        freq = np.concatenate([np.cos(tt * f), np.sin(tt * f)]).astype(np.float32)[None, :]
        adaln = self.linear(freq, "t_embedder.mlp.0")
        adaln = (adaln / (1.0 + np.exp(-adaln))).astype(np.float32)
        adaln = self.linear(adaln, "t_embedder.mlp.2")
        # patchify2d (tensor.cpp:936-951): token (h, w), features ordered (ph, pw, c)
        tok = x[0].reshape(C, Ht, p, Wt, p).transpose(1, 3, 2, 4, 0).reshape(n_img, p * p * C)
        img = self.linear(np.ascontiguousarray(tok), "all_x_embedder.2-1")
        img = np.concatenate([img, np.repeat(self.w["x_pad_token"], n_img_pad - n_img, 0)], 0)
        capt = self.linear(o.rms_norm(cap[0], self.w["cap_embedder.0.weight"], self.eps), "cap_embedder.1")
        capt = np.concatenate([capt, np.repeat(self.w["cap_pad_token"], n_cap_pad - L, 0)], 0)
        cap_pos = [(1 + i, 0, 0) for i in range(n_cap_pad)]
        img_pos = [(0, 0, 0)] * n_img_pad
        for hh in range(Ht):
            for ww in range(Wt):
                img_pos[hh * Wt + ww] = (n_cap_pad + 1, hh, ww)
        ics, isn = self.rope_tables(img_pos)
        ccs, csn = self.rope_tables(cap_pos)
        i = 0
        while self.has(f"noise_refiner.{i}.attention_norm1.weight"):
            img = self.run_block(f"noise_refiner.{i}", img, ics, isn, adaln)
            i += 1
        i = 0
        while self.has(f"context_refiner.{i}.attention_norm1.weight"):
            capt = self.run_block(f"context_refiner.{i}", capt, ccs, csn, None)
            i += 1
        uni = np.concatenate([img, capt], 0)
        ucs, usn = self.rope_tables(img_pos + cap_pos)
        i = 0
        while self.has(f"layers.{i}.attention_norm1.weight"):
            uni = self.run_block(f"layers.{i}", uni, ucs, usn, adaln)
            i += 1
        img_out = uni[:n_img]
        c = (adaln / (1.0 + np.exp(-adaln))).astype(np.float32)
        scale = self.linear(c, "all_final_layer.2-1.adaLN_modulation.1") * 1.0 + 1.0
        img_out = o.mul_rows(o.layer_norm(img_out, None, None, 1e-6), scale.reshape(-1).astype(np.float32))
        out_tok = self.linear(img_out, "all_final_layer.2-1.linear")
        out = out_tok.reshape(Ht, Wt, p, p, C).transpose(4, 0, 2, 1, 3).reshape(1, C, H, W)
        return np.ascontiguousarray(out, np.float32)
