"""Benchmark of StableDiffusion-cpp's dense-contraction hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload dit|dit_tp|gemm|attention|conv|vae|unet]

Workload `dit` (default): the full 30-layer Z-Image-shaped DiT (6.15 B
random-init bf16 parameters) at 1024x1024 (16-channel 128x128 latent, 128 text tokens of
width 2560 ~N(0,1)), one denoising step = one transformer forward over a global batch of
8 images. The 8 images are split across the N ranks (8/N per GPU, weights replicated,
no collective: image forwards are independent), so total work is fixed: "scaling":
"strong". Metric: ms per denoising step for the whole batch (lower is better), max over
ranks of CUDA-event time.

Workload `gemm`: Y[4096,11520] = X[4096,3840] W[11520,3840]^T + b,
one GEMM per GPU per step (replicas), TFLOP/s.

Workload `dit_tp`: the same DiT at batch 1, 2048x2048 (16512 tokens),
Megatron tensor parallelism over the N ranks; ms per step. The row-parallel outputs are
combined inside the kernels (--tp-mode 1, default: GEMM epilogue stores to the owner
rank over NVLink, sequence-sharded post-norm) or by an NCCL all-reduce (--tp-mode 0).

Workload `conv`: the VAE decoder's 3x3 convolutions at the four resolution stages of a
1024^2 decode (512@128^2, 512@256^2, 256@512^2, 128@1024^2), TFLOP/s through conv2d.

Workload `vae`: one FLUX / Z-Image VAE decode of a 1024x1024 image on the device
(sdb200_vae_decode), ms per decode.

Workload `unet`: the SD 1.5 UNet's contraction shapes at 512^2 - one
transformer block (self- and cross-attention projections, 8 heads of 40, 77 text tokens,
GEGLU feed-forward) and one 3x3 convolution 320 -> 320 on 64x64 - through the C ABI with
fp32 weights, ms per pass. The reference arm adds the full SD 1.5 UNet step through the
drop-in link (`reference_code_on_sdb200`).

Workload `attention`: the DiT's joint attention at 1024^2 alone (4224 tokens, 30 heads of
128), TFLOP/s of the tensor-core kernel (for profiling the second hot kernel).

Printed on rank 0 as one JSON line:
  value / ms_per_step  inputs resident in HBM
  e2e          the same metric through the C ABI with pinned HOST buffers: H2D of the
               step's latents and text states, D2H of the prediction, inside the timed
               region (weights resident, as after Weights::to_device)
  roofline     the dominant kernel (the tcgen05 GEMM) timed live with CUDA events on the
               library's stream across one profiled step: algorithmic FLOPs / kernel time,
               against MEASURED_PEAKS.json (sustained bf16 peak for a kernel inside a long
               step; burst for the isolated GEMM workload)
  cpu_baseline the reference's own CPU forward (oracle/_ref, compiled from its sources) on
               a bounded sample: one full-width block at 1024^2, scaled by FLOPs to the step
  gpu_launches kernels this library launched inside the timed region (counted by the library)
--impl reference times the reference's CPU implementation of the same workload (rank 0); its line
also reports the reference's own GPU backend (src/backend_cuda.cu + cuBLAS, built for sm_100a) on
the same seeded inputs as `reference_gpu` (--no-ref-gpu skips it).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "stablediffusion-cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

METRIC = "bf16 GEMM TFLOP/s (% tcgen05 peak); Z-Image DiT ms/step @1024² at 1/2/4/8 GPUs"
GLOBAL_BATCH = 8
LAT_H = LAT_W = 128        # 1024x1024 image / 8 (VAE)
TEXT_TOKENS = 128
THROTTLE_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
    0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"burst": d["bf16_tflops"], "sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "hbm": d["hbm_gbs"], "kind": "measured"}
    return {"burst": 1590.0, "sustained": 1400.0, "hbm": 6650.0, "kind": "fallback"}


def profile_value(fname, key):
    """A `key: value` line from a committed ncu summary under profiles/."""
    p = os.path.join(ROOT, "profiles", fname)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class ClockSampler:
    """Samples the SM clock and the clock-event (throttle) reasons through NVML every
    2 ms from a background thread while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception:
            self._ok = False
        return self

    def _run(self):
        nv, h = self._nv, self._h
        while not self._stop.is_set():
            try:
                self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                     nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
            except Exception:
                pass
            time.sleep(0.002)

    def __exit__(self, *a):
        self._stop.set()
        if self._ok:
            self._t.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        reasons = set()
        for _, bits in self.samples:
            for b, name in THROTTLE_BITS.items():
                if bits & b and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(c for c, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------------------
# FLOP model of one Z-Image forward (algorithmic: 2*M*N*K per GEMM, 4*S^2*D per attention)
# ---------------------------------------------------------------------------------------
def dit_forward_flops(cfg, H=LAT_H, W=LAT_W, L=TEXT_TOKENS):
    pad = lambda n: (n + 31) // 32 * 32  # noqa: E731
    D, F, T = cfg.dim, cfg.ffn, cfg.t_dim
    n_img = (H // cfg.patch) * (W // cfg.patch)
    s_img, s_cap = pad(n_img), pad(L)
    s_uni = s_img + s_cap
    pc = cfg.patch * cfg.patch * cfg.in_channels

    def block(S, modulated):
        lin = 2.0 * S * (4 * D * D + 3 * D * F)
        att = 4.0 * S * S * D
        mod = 2.0 * 4 * D * T if modulated else 0.0
        return lin, att, mod

    lin = att = small = 0.0
    for S, n, m in ((s_img, cfg.noise_refiners, True), (s_cap, cfg.context_refiners, False),
                    (s_uni, cfg.layers, True)):
        a, b, c = block(S, m)
        lin += n * a
        att += n * b
        small += n * c
    small += 2.0 * n_img * pc * D + 2.0 * L * cfg.cap_dim * D + 2.0 * n_img * D * pc
    small += 2.0 * (cfg.t_hidden * T * 2 + D * T)
    return {"total": lin + att + small, "linear": lin, "attention": att, "small": small}


def dist_setup():
    return int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), int(
        os.environ.get("LOCAL_RANK", "0"))


# ---------------------------------------------------------------------------------------
# Reference CPU path (oracle/_ref: the reference's own tensor.cpp / zimage.cpp)
# ---------------------------------------------------------------------------------------
def ref_dit_block_sample():
    """The reference ZImageTransformer with one full-width layer (no refiners) at 1024^2:
    returns (callable forward, sample FLOPs, threads, model keep-alive)."""
    import numpy as np

    from oracle import RefCPU
    from sdb200.zimage import ZConfig, random_weights_numpy

    ref = RefCPU()
    ref.set_num_threads(0)
    cfg = ZConfig(layers=1, noise_refiners=0, context_refiners=0)
    w, bf = random_weights_numpy(cfg, 11)
    model = ref.zimage(w, bf, heads=cfg.heads)
    rng = np.random.default_rng(12)
    x = rng.standard_normal((1, cfg.in_channels, LAT_H, LAT_W)).astype(np.float32)
    cap = rng.standard_normal((1, TEXT_TOKENS, cfg.cap_dim)).astype(np.float32)
    return (lambda: model(x, 0.5, cap)), dit_forward_flops(cfg)["total"], ref.num_threads(), model


def ref_gpu(world, local):
    """The reference's own GPU backend (src/backend_cuda.cu + cuBLAS, built from its sources
    into oracle/_ref/libsdref_cuda.so): a comparison column timed on the same B200, one
    process on device 0 only (the reference hard-wires device 0). Returns (RefCUDA or
    None, reason)."""
    if world != 1 or local != 0:
        return None, "single-GPU runs only (the reference backend uses device 0)"
    try:
        from oracle import RefCUDA

        if not RefCUDA.available():
            return None, "oracle/_ref/libsdref_cuda.so not built"
        r = RefCUDA()
        if not r.cuda_available():
            return None, "the reference backend found no CUDA device"
        return r, None
    except Exception as e:  # reported, never required
        return None, f"failed: {e}"


REF_GPU_KIND = "reference src/backend_cuda.cu + cuBLAS (its own GPU path), built for sm_100a, same B200"


def ref_gemm_sample(rows=512):
    import numpy as np

    from oracle import RefCPU
    from sdb200.workloads import cfg1_inputs

    ref = RefCPU()
    ref.set_num_threads(0)
    X, W, b = cfg1_inputs()
    Xs = np.ascontiguousarray(X[:rows])
    Wh = ref.to_bf16(W)
    return (lambda: ref.gemm_nt_bf16(Xs, Wh, b)), 2.0 * rows * W.shape[0] * W.shape[1], ref.num_threads(), None


def cpu_baseline(workload, reps=1):
    try:
        from oracle import RefCPU

        if not RefCPU.available():
            return {"value": None, "unit": None, "cores": None, "kind": "reference",
                    "sample": "oracle/_ref/libsdref.so not built"}
        if workload == "dit":
            from sdb200.zimage import Z_IMAGE

            fn, sample_flop, cores, _keep = ref_dit_block_sample()
            fn()  # warm-up (thread pool, page-in)
            t0 = time.perf_counter()
            for _ in range(reps):
                fn()
            dt = (time.perf_counter() - t0) / reps
            step_flop = GLOBAL_BATCH * dit_forward_flops(Z_IMAGE)["total"]
            return {"value": dt * 1e3 * step_flop / sample_flop, "unit": "ms/step", "cores": cores,
                    "kind": "reference",
                    "sample": f"reference ZImageTransformer forward with one full-width block at 1024^2 "
                              f"({sample_flop / 1e12:.2f} TFLOP, {dt:.2f} s), scaled by FLOPs to a step of "
                              f"{GLOBAL_BATCH} full 30-layer forwards ({step_flop / 1e12:.0f} TFLOP)"}
        fn, flop, cores, _ = ref_gemm_sample()
        fn()
        t0 = time.perf_counter()
        for _ in range(max(reps, 3)):
            fn()
        dt = (time.perf_counter() - t0) / max(reps, 3)
        return {"value": flop / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                "sample": "512 of 4096 rows of the cfg1 GEMM, reference gemm_nt_bf16 (tensor.cpp:412)"}
    except Exception as e:  # reported, never required
        return {"value": None, "unit": None, "cores": None, "kind": "reference", "sample": f"failed: {e}"}


def reference_gpu_line(args, world, local):
    """The reference's own GPU path (oracle/_ref/libsdref_cuda.so: src/backend_cuda.cu +
    cuBLAS) on this run's workload and the same seeded inputs as this library's arm,
    reported beside the reference arm's CPU value. Returns the JSON object, or a note
    saying why it was not measured."""
    if args.no_ref_gpu:
        return {"value": None, "unavailable": "--no-ref-gpu"}
    try:
        import torch

        if not torch.cuda.is_available():
            return {"value": None, "unavailable": "no CUDA device"}
        r, why = ref_gpu(world, local)
        if r is None:
            return {"value": None, "unavailable": why}
        torch.cuda.set_device(0)
        dev = torch.device("cuda", 0)
        stream = torch.cuda.current_stream()
        if args.workload == "gemm":
            from sdb200.workloads import cfg1_inputs, f32_to_bf16_bits

            M, N, K = 4096, 11520, 3840
            X, W, b = cfg1_inputs()
            Xd = torch.from_numpy(X).to(dev)
            Wd = torch.from_numpy(f32_to_bf16_bits(W).view("int16")).to(dev)
            bd = torch.from_numpy(b).to(dev)
            Yr = torch.empty((M, N), device=dev)
            fn = lambda: r.gemm_nt_bf16_dev(M, N, K, Xd.data_ptr(), K, Wd.data_ptr(), K, Yr.data_ptr(), N,  # noqa
                                            bd.data_ptr())
            for _ in range(3):
                fn()
            ms = timed_loop(fn, args.steps, stream, None, dev) / args.steps
            return {"value": 2.0 * M * N * K / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "kind": REF_GPU_KIND,
                    "sample": "cfg1 GEMM on device buffers: pack A to bf16, cublasGemmEx, bias kernel"}
        if args.workload == "attention":
            S, H, d = 4224, 30, 128
            g = torch.Generator(device=dev)
            g.manual_seed(77)
            q = torch.randn((1, S, H * d), generator=g, device=dev)
            k, v, o = torch.randn_like(q), torch.randn_like(q), torch.empty_like(q)
            fn = lambda: r.attention_dev(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), 1, S, S, H, H, d)  # noqa
            for _ in range(2):
                fn()
            ms = timed_loop(fn, args.steps, stream, None, dev) / args.steps
            return {"value": 4.0 * S * S * d * H / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "kind": REF_GPU_KIND,
                    "sample": "attention() on fp32 q/k/v device buffers (strided-batched SGEMM, softmax, SGEMM)"}
        if args.workload == "conv":
            g = torch.Generator(device=dev)
            g.manual_seed(31)
            bufs = []
            for c, s in CONV_STAGES:
                x = torch.randn((1, c, s, s), generator=g, device=dev)
                w = 0.02 * torch.randn((c, c, 3, 3), generator=g, device=dev)
                b = 0.02 * torch.randn((c,), generator=g, device=dev)
                bufs.append((c, s, x, w, b, torch.empty_like(x)))

            def fn():
                for c, s, x, w, b, y in bufs:
                    r.conv2d_dev(x.data_ptr(), 1, c, s, s, w.data_ptr(), c, 3, 3, b.data_ptr(), 1, 1, y.data_ptr(), s, s)

            fn()
            ms = timed_loop(fn, 1, stream, None, dev)
            return {"value": sum(conv_flops()) / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "kind": REF_GPU_KIND,
                    "ms_per_step": ms, "sample": "conv2d() of the four stages (im2col + fp32 SGEMM)"}
        if args.workload == "unet":
            t = cfg2_tensors(dev)
            ops = cfg2_ops_refgpu(r, t)
            flush_buf = torch.empty(64 << 20, device=dev)
            step = lambda: [o[3]() for o in ops]  # noqa: E731
            step()
            ms = timed_steps_flushed(step, args.steps, stream, None, dev, flush_buf.zero_) / args.steps
            return {"value": ms, "unit": "ms/step", "kind": REF_GPU_KIND,
                    "sample": "the config-2 op set on device buffers (cublasSgemm, batched SGEMM attention, "
                              "im2col conv), L2 flushed before each step"}
        if args.workload == "vae":
            import numpy as np

            from sdb200.vae import FLUX_VAE, random_weights

            rv = r.vae_cuda(random_weights(FLUX_VAE, 7), FLUX_VAE.scaling_factor, FLUX_VAE.shift_factor)
            z = np.random.default_rng(9).standard_normal((1, FLUX_VAE.latent_channels, LAT_H, LAT_W)).astype(np.float32)
            rv(z)
            t0 = time.perf_counter()
            rv(z)
            return {"value": (time.perf_counter() - t0) * 1e3, "unit": "ms/decode", "kind": REF_GPU_KIND,
                    "sample": "VAEDecoder::decode of a 1024^2 image on the GPU backend (wall clock, latent in and "
                              "image out included)"}
        if args.workload == "dit":
            from sdb200.zimage import Z_IMAGE, random_weights_torch

            wts = random_weights_torch(Z_IMAGE, 0, dev)
            rm = r.zimage_cuda(wts, heads=Z_IMAGE.heads)
            del wts
            g = torch.Generator(device=dev)
            g.manual_seed(1000)
            x = torch.randn((1, Z_IMAGE.in_channels, LAT_H, LAT_W), generator=g, device=dev).cpu().numpy()
            cap = torch.randn((1, TEXT_TOKENS, Z_IMAGE.cap_dim), generator=g, device=dev).cpu().numpy()
            rm(x, 0.5, cap)
            t0 = time.perf_counter()
            rm(x, 0.5, cap)
            dt = time.perf_counter() - t0
            return {"value": dt * 1e3 * GLOBAL_BATCH, "unit": "ms/step", "kind": REF_GPU_KIND,
                    "sample": f"one batch-1 forward of the full 30-layer model on the GPU backend ({dt * 1e3:.1f} ms, "
                              f"wall clock with latent in and prediction out) x {GLOBAL_BATCH} images per step"}
        return {"value": None, "unavailable": f"not measured for workload {args.workload}"}
    except Exception as e:  # reported, never required
        return {"value": None, "unavailable": f"failed: {e}"}


# ---------------------------------------------------------------------------------------
# the SD 1.5 UNet's contraction shapes at 512^2 (64x64 latent = 4096
# tokens of 320 channels), fp32 weights ~N(0, 0.02), activations ~N(0, 1): one transformer
# block's self-attention (q/k/v/out projections, 8 heads of 40), cross-attention (77 text
# tokens of width 768), GEGLU feed-forward (320 -> 2560 -> GEGLU -> 1280 -> 320), and one
# 3x3 convolution 320 -> 320 on 64x64 (modules.cpp:55-80, unet.cpp; shapes from the SD 1.5
# layout). One step = one pass over these ops.
# ---------------------------------------------------------------------------------------
CFG2 = dict(T=4096, C=320, heads=8, L=77, E=768, F=1280, side=64)


def cfg2_tensors(dev, seed=55):
    import torch

    c = CFG2
    T, C, L, E, F, side = c["T"], c["C"], c["L"], c["E"], c["F"], c["side"]
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rn = lambda *shape, s=1.0: s * torch.randn(shape, generator=g, device=dev)  # noqa: E731
    t = {"x": rn(T, C), "ctx": rn(L, E), "img": rn(1, C, side, side)}
    for n in ("q1", "k1", "v1", "o1", "q2", "o2"):
        t["W" + n] = rn(C, C, s=0.02)
    t["Wk2"], t["Wv2"] = rn(C, E, s=0.02), rn(C, E, s=0.02)
    t["Wf1"], t["Wf2"] = rn(2 * F, C, s=0.02), rn(C, F, s=0.02)
    t["Wc"] = rn(C, C, 3, 3, s=0.02)
    for n in ("bo1", "bo2", "bf2", "bc"):
        t[n] = rn(C, s=0.02)
    t["bf1"] = rn(2 * F, s=0.02)
    for n, shape in (("q1", (T, C)), ("k1", (T, C)), ("v1", (T, C)), ("a1", (T, C)), ("o1", (T, C)), ("q2", (T, C)),
                     ("k2", (L, C)), ("v2", (L, C)), ("a2", (T, C)), ("o2", (T, C)), ("f1", (T, 2 * F)),
                     ("g", (T, F)), ("f2", (T, C)), ("y", (1, C, side, side))):
        t[n] = torch.empty(shape, device=dev)
    return t


def cfg2_ops(t, gemm, attention, geglu, conv):
    """[(name, FLOP, minimum bytes, call)] of one cfg2 pass over tensors t, with the four
    backend entry points given as callables taking device pointers:
    gemm(M, N, K, A, B, C, bias), attention(q, k, v, out, Sq, Skv), geglu(x, y, rows, D),
    conv(x, w, bias, out)."""
    c = CFG2
    T, C, L, E, F, side, H = c["T"], c["C"], c["L"], c["E"], c["F"], c["side"], c["heads"]
    p = lambda n: t[n].data_ptr() if n else None  # noqa: E731

    def lin(name, M, N, K, a, w, out, bias=None):
        return (name, 2.0 * M * N * K, 4.0 * (M * K + N * K + M * N), lambda: gemm(M, N, K, p(a), p(w), p(out), p(bias)))

    def att(name, q, k, v, o, Sq, Skv):
        return (name, 4.0 * Sq * Skv * C, 4.0 * (2 * Sq * C + 2 * Skv * C),
                lambda: attention(p(q), p(k), p(v), p(o), Sq, Skv))

    return [
        lin("self_q", T, C, C, "x", "Wq1", "q1"), lin("self_k", T, C, C, "x", "Wk1", "k1"),
        lin("self_v", T, C, C, "x", "Wv1", "v1"), att("self_attention", "q1", "k1", "v1", "a1", T, T),
        lin("self_out", T, C, C, "a1", "Wo1", "o1", "bo1"),
        lin("cross_q", T, C, C, "x", "Wq2", "q2"), lin("cross_k", L, C, E, "ctx", "Wk2", "k2"),
        lin("cross_v", L, C, E, "ctx", "Wv2", "v2"), att("cross_attention", "q2", "k2", "v2", "a2", T, L),
        lin("cross_out", T, C, C, "a2", "Wo2", "o2", "bo2"),
        lin("ffn_proj", T, 2 * F, C, "x", "Wf1", "f1", "bf1"),
        ("ffn_geglu", 0.0, 4.0 * (T * 2 * F + T * F), lambda: geglu(p("f1"), p("g"), T, F)),
        lin("ffn_out", T, C, F, "g", "Wf2", "f2", "bf2"),
        ("conv3x3", 2.0 * C * C * 9 * side * side, 4.0 * (2 * C * side * side + 9 * C * C),
         lambda: conv(p("img"), p("Wc"), p("bc"), p("y"))),
    ]


def cfg2_ops_sdb(t):
    import sdb200

    L = sdb200.lib()
    c = CFG2
    C, H, side = c["C"], c["heads"], c["side"]
    ck = sdb200.check
    return cfg2_ops(
        t,
        lambda M, N, K, a, w, o, b: ck(L.sdb200_gemm_nt_f32(M, N, K, a, K, w, K, o, N, b, 0)),
        lambda q, k, v, o, Sq, Skv: ck(L.sdb200_attention(q, k, v, o, 1, Sq, Skv, H, H, C // H, 0)),
        lambda x, y, rows, D: ck(L.sdb200_geglu(x, y, rows, D)),
        lambda x, w, b, o: ck(L.sdb200_conv2d(x, 1, C, side, side, w, C, 3, 3, b, 1, 1, o, side, side)))


def cfg2_ops_refgpu(r, t):
    c = CFG2
    C, H, side = c["C"], c["heads"], c["side"]
    return cfg2_ops(
        t,
        lambda M, N, K, a, w, o, b: r.gemm_nt_f32_dev(M, N, K, a, K, w, K, o, N, b),
        lambda q, k, v, o, Sq, Skv: r.attention_dev(q, k, v, o, 1, Sq, Skv, H, H, C // H),
        lambda x, y, rows, D: r.geglu_dev(x, y, rows, D),
        lambda x, w, b, o: r.conv2d_dev(x, 1, C, side, side, w, C, 3, 3, b, 1, 1, o, side, side))


def cfg2_flop():
    return sum(f for _, f, _, _ in cfg2_ops({}, *(lambda *a: None,) * 4))


def timed_steps_flushed(fn, steps, stream, pg, dev, flush):
    """Sum over `steps` calls of the CUDA-event time of each, with `flush` (a write of a
    buffer larger than L2) run untimed before every call; barrier + synchronize on both
    sides, max over ranks."""
    import torch

    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    total = 0.0
    evs = []
    for _ in range(steps):
        flush()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    total = sum(a.elapsed_time(b) for a, b in evs)
    if pg:
        pg.barrier()
    t = torch.tensor([total], device=dev)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def run_unet(args, world, rank, local, pg, dev):
    """BASELINE config 2 on this library through the C ABI (sdb200_gemm_nt_f32 on tf32
    tensor cores, sdb200_attention, sdb200_geglu, sdb200_conv2d), L2 flushed before each
    step. value = ms per pass over the config-2 ops; every rank runs its own replica."""
    import torch

    import sdb200
    from sdb200 import backend as be

    L = sdb200.lib()
    t = cfg2_tensors(dev)
    ops = cfg2_ops_sdb(t)
    flop = sum(o[1] for o in ops)
    flush_buf = torch.empty(64 << 20, device=dev)  # 256 MB > L2
    flush = flush_buf.zero_
    step = lambda: [o[3]() for o in ops]  # noqa: E731
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_steps_flushed(step, args.steps, stream, pg, dev, flush)
    launches = L.sdb200_launch_count() - n0
    ms_step = ms / args.steps
    # per-op CUDA-event times (one flushed pass per op)
    per_op = {}
    pk = peaks()
    for name, f, nbytes, call in ops:
        opms = timed_steps_flushed(call, 3, stream, None, dev, flush) / 3
        per_op[name] = {"us": opms * 1e3, "tflops": f / (opms * 1e-3) / 1e12 if f else None,
                        "gb_s_min_bytes": nbytes / (opms * 1e-3) / 1e9}
    top = max(per_op, key=lambda n: per_op[n]["us"])
    # end to end: the step's inputs (latent tokens, text states, conv input) from pinned
    # host memory and its outputs (self, cross and FFN outputs, conv output) back
    ins = [t[n] for n in ("x", "ctx", "img")]
    outs = [t[n] for n in ("o1", "o2", "f2", "y")]
    hin = [x.cpu().pin_memory() for x in ins]
    hout = [torch.empty_like(x, device="cpu").pin_memory() for x in outs]

    def e2e_step():
        for h, d in zip(hin, ins):
            sdb200.check(L.sdb200_upload(d.data_ptr(), h.data_ptr(), h.numel() * 4))
        step()
        for h, d in zip(hout, outs):
            sdb200.check(L.sdb200_download(h.data_ptr(), d.data_ptr(), h.numel() * 4))

    e2e_step()
    e2e_ms = timed_steps_flushed(e2e_step, args.steps, stream, pg, dev, flush) / args.steps
    # The same op set with the opt-in packed-operand cache (constant weights packed once).
    sdb200.check(L.sdb200_set_operand_cache(1))
    step()
    cached_ms = timed_steps_flushed(step, args.steps, stream, pg, dev, flush) / args.steps
    sdb200.check(L.sdb200_set_operand_cache(0))
    if rank == 0:
        top_f = next(o for o in ops if o[0] == top)
        top_tf = per_op[top]["tflops"]
        print(json.dumps({
            "metric": "SD 1.5 UNet config-2 op set ms per pass (512^2: 4096 tokens x 320 ch)", "value": ms_step,
            "unit": "ms/step", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp32 weights/activations; tf32 tensor-core GEMM and conv operands, fp16 attention operands",
            "data": "synthetic (N(0,0.02) fp32 weights, N(0,1) activations)",
            "config": {"workload": "cfg2: SD 1.5 transformer block at 512^2 (self-attn q/k/v/out 4096x320x320, "
                                   "8 heads of 40; cross-attn 77 tokens of 768; GEGLU FFN 320->2560->1280->320) "
                                   "+ 3x3 conv 320->320 on 64x64",
                       "parallelism": f"replicas x{world}", "l2": "256 MB buffer written before every step (untimed)",
                       "gflop_per_step": flop / 1e9},
            "step_tflops": flop / (ms_step * 1e-3) / 1e12, "gpu_launches": int(launches),
            "ms_per_step_operand_cache": cached_ms,
            "roofline": {"bound": "tensor", "kernel": f"{top} (the op with the largest time)",
                         "achieved": top_tf, "peak": pk["burst"], "unit": "TFLOP/s",
                         "frac": top_tf / pk["burst"] if top_tf else None,
                         "peak_kind": f"{pk['kind']} bf16 burst (the tf32 rate is half of it)",
                         "traffic": None, "ops": per_op, "top_op_flop": top_f[1]},
            "e2e": {"value": e2e_ms, "unit": "ms/step", "h2d_bytes_per_step": int(sum(h.numel() * 4 for h in hin)),
                    "d2h_bytes_per_step": int(sum(h.numel() * 4 for h in hout))},
            "cpu_baseline": None, "clocks": clk.summary(), "device_error_word": be.device_error_word()}), flush=True)


def ref_unet_ops_cpu():
    """The config-2 op set on the reference's CPU path (oracle/_ref: gemm_nt, attention,
    geglu, conv2d on host arrays): returns (call, FLOP, threads)."""
    import numpy as np

    from oracle import RefCPU

    ref = RefCPU()
    ref.set_num_threads(0)
    c = CFG2
    T, C, L, E, F, side, H = c["T"], c["C"], c["L"], c["E"], c["F"], c["side"], c["heads"]
    rng = np.random.default_rng(55)
    rn = lambda *shape, s=1.0: (s * rng.standard_normal(shape)).astype(np.float32)  # noqa: E731
    x, ctx, img = rn(T, C), rn(L, E), rn(1, C, side, side)
    W = {n: rn(C, C, s=0.02) for n in ("q1", "k1", "v1", "o1", "q2", "o2")}
    Wk2, Wv2, Wf1, Wf2, Wc = rn(C, E, s=0.02), rn(C, E, s=0.02), rn(2 * F, C, s=0.02), rn(C, F, s=0.02), rn(
        C, C, 3, 3, s=0.02)
    b = rn(C, s=0.02)
    bf1 = rn(2 * F, s=0.02)

    def fn():
        q1, k1, v1 = (ref.gemm_nt(x, W[n]) for n in ("q1", "k1", "v1"))
        a1 = ref.attention(q1[None], k1[None], v1[None], H)[0]
        ref.gemm_nt(a1, W["o1"], b)
        q2 = ref.gemm_nt(x, W["q2"])
        k2, v2 = ref.gemm_nt(ctx, Wk2), ref.gemm_nt(ctx, Wv2)
        a2 = ref.attention(q2[None], k2[None], v2[None], H)[0]
        ref.gemm_nt(a2, W["o2"], b)
        g = ref.geglu(ref.gemm_nt(x, Wf1, bf1))
        ref.gemm_nt(g, Wf2, b)
        ref.conv2d(img, Wc, b, 1, 1)

    return fn, cfg2_flop(), ref.num_threads()


def dropin_line(args, world, local):
    """The maintainer's link: the reference's own model code (zimage.cpp,
    unet.cpp over tensor.cpp / modules.cpp) linked against libsdb200.so in place of its
    backend (oracle/_ref/libsdref_b200.so), timed on this run's model workload beside the
    same code on its own GPU backend. Returns the JSON object or a note."""
    if args.no_ref_gpu:
        return {"value": None, "unavailable": "--no-ref-gpu"}
    try:
        import torch

        if world != 1 or local != 0:
            return {"value": None, "unavailable": "single-GPU runs only"}
        if not torch.cuda.is_available():
            return {"value": None, "unavailable": "no CUDA device"}
        from oracle import RefOnB200

        if not RefOnB200.available():
            return {"value": None, "unavailable": "oracle/_ref/libsdref_b200.so not built"}
        r = RefOnB200()
        dev = torch.device("cuda", 0)
        kind = ("the reference's own model code (tensor.cpp, modules.cpp, zimage.cpp / unet.cpp) linked against "
                "libsdb200.so in place of its backend: every sd::cuda call lands in this library")
        if args.workload == "dit":
            from sdb200.zimage import Z_IMAGE, random_weights_torch

            wts = random_weights_torch(Z_IMAGE, 0, dev)
            rm = r.zimage_cuda(wts, heads=Z_IMAGE.heads)
            del wts
            g = torch.Generator(device=dev)
            g.manual_seed(1000)
            x = torch.randn((1, Z_IMAGE.in_channels, LAT_H, LAT_W), generator=g, device=dev).cpu().numpy()
            cap = torch.randn((1, TEXT_TOKENS, Z_IMAGE.cap_dim), generator=g, device=dev).cpu().numpy()
            rm(x, 0.5, cap)
            reps = 3
            t0 = time.perf_counter()
            for _ in range(reps):
                rm(x, 0.5, cap)
            dt = (time.perf_counter() - t0) / reps
            del rm
            torch.cuda.empty_cache()
            return {"value": dt * 1e3 * GLOBAL_BATCH, "unit": "ms/step", "kind": kind,
                    "ms_per_image": dt * 1e3,
                    "sample": f"batch-1 forwards of the full 30-layer model at 1024^2 (mean of {reps}, wall clock "
                              f"with latent in and prediction out) x {GLOBAL_BATCH} images per step"}
        if args.workload == "unet":
            import numpy as np

            from oracle import RefCUDA
            from sdb200.unet import SD15, unet_weights

            w = unet_weights(seed=3, device="cuda", **SD15)
            rng = np.random.default_rng(4)
            x = rng.standard_normal((2, 4, 64, 64)).astype(np.float32)
            ctx = rng.standard_normal((2, 77, 768)).astype(np.float32)
            import sdb200

            times, outs = {}, {}
            for name, lib in (("reference_backend", RefCUDA() if RefCUDA.available() else None), ("sdb200", r),
                              ("sdb200_operand_cache", r)):
                if lib is None:
                    continue
                if name == "sdb200_operand_cache":
                    sdb200.check(sdb200.lib().sdb200_set_operand_cache(1))
                m = lib.unet(w, heads=8, on_device=True)
                m(x, 500.0, ctx)
                t0 = time.perf_counter()
                for _ in range(3):
                    outs[name] = m(x, 500.0, ctx)
                times[name] = (time.perf_counter() - t0) / 3 * 1e3
                del m
                sdb200.check(sdb200.lib().sdb200_set_operand_cache(0))
            agree = None
            if "sdb200" in outs and "reference_backend" in outs:
                a, b2 = outs["sdb200"].astype(np.float64), outs["reference_backend"].astype(np.float64)
                agree = float(np.linalg.norm(a - b2) / np.linalg.norm(b2))
            cache_agree = None
            if "sdb200_operand_cache" in outs:
                a, b2 = outs["sdb200_operand_cache"].astype(np.float64), outs["sdb200"].astype(np.float64)
                cache_agree = float(np.linalg.norm(a - b2) / np.linalg.norm(b2))
            return {"value": times["sdb200"], "unit": "ms/UNet step", "kind": kind,
                    "with_operand_cache_ms": times.get("sdb200_operand_cache"),
                    "operand_cache_rel_diff": cache_agree,
                    "reference_backend_ms": times.get("reference_backend"), "rel_diff_vs_reference_backend": agree,
                    "sample": "the full SD 1.5 UNet (unet.cpp, 860 M fp32 parameters) at 512^2 with a CFG batch of 2, "
                              "mean of 3 steps, wall clock with latent in and prediction out"}
        return {"value": None, "unavailable": f"not measured for workload {args.workload}"}
    except Exception as e:  # reported, never required
        return {"value": None, "unavailable": f"failed: {e}"}


def run_reference(args, world, rank, local=0):
    """--impl reference: the reference's CPU implementation, rank 0 only. Beside it,
    `reference_gpu` reports the reference's own GPU backend on the same workload."""
    if rank != 0:
        return
    if args.workload == "dit":
        from sdb200.zimage import Z_IMAGE

        fn, sample_flop, cores, _keep = ref_dit_block_sample()
        step_flop = GLOBAL_BATCH * dit_forward_flops(Z_IMAGE)["total"]
        for _ in range(args.warmup):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        dt = (time.perf_counter() - t0) / args.steps
        ms = dt * 1e3 * step_flop / sample_flop
        line = {"impl": "reference", "metric": METRIC, "value": ms, "unit": "ms/step", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32 activations x bf16 weights (CPU)",
                "data": "synthetic (random-init weights, N(0,1) latents and text states)",
                "config": {"workload": "cfg4: 30-layer Z-Image DiT @1024^2, batch of 8 images, one denoising step",
                           "parallelism": "reference CPU thread pool"},
                "cpu_baseline": {"value": ms, "unit": "ms/step", "cores": cores, "kind": "reference",
                                 "sample": f"one full-width block forward per step ({dt:.2f} s), scaled by FLOPs "
                                           f"({sample_flop / 1e12:.2f} -> {step_flop / 1e12:.0f} TFLOP)"},
                "e2e": {"value": ms, "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    elif args.workload == "vae":
        from sdb200.vae import FLUX_VAE, decode_flops

        fn, f0, cores, _keep = ref_vae_sample()
        FLOP = decode_flops(FLUX_VAE, LAT_H, LAT_W)
        for _ in range(min(args.warmup, 1)):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        dt = (time.perf_counter() - t0) / args.steps
        ms = dt * 1e3 * FLOP / f0
        line = {"impl": "reference", "metric": "VAE decode ms (1024^2 image, FLUX / Z-Image VAE)", "value": ms,
                "unit": "ms/decode", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (CPU)",
                "data": "synthetic (random-init weights, N(0,1) latent)",
                "config": {"workload": "AutoencoderKL decoder, latent 16x128x128 -> 3x1024x1024",
                           "sample": "a 256^2 decode per step, scaled by FLOPs"},
                "cpu_baseline": {"value": ms, "unit": "ms/decode", "cores": cores, "kind": "reference",
                                 "sample": f"VAEDecoder::decode of a 256^2 image per step ({dt:.2f} s), FLOP-scaled"},
                "e2e": {"value": ms, "unit": "ms/decode", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    elif args.workload == "unet":
        fn, flop, cores = ref_unet_ops_cpu()
        fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        ms = (time.perf_counter() - t0) / args.steps * 1e3
        line = {"impl": "reference", "metric": "SD 1.5 UNet config-2 op set ms per pass (512^2: 4096 tokens x 320 ch)",
                "value": ms, "unit": "ms/step", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms, "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 (CPU)", "data": "synthetic (N(0,0.02) fp32 weights, N(0,1) activations)",
                "config": {"workload": "cfg2 op set (see --workload unet)", "parallelism": "reference CPU thread pool"},
                "cpu_baseline": {"value": ms, "unit": "ms/step", "cores": cores, "kind": "reference",
                                 "sample": f"the whole config-2 op set per step ({flop / 1e9:.1f} GFLOP)"},
                "e2e": {"value": ms, "unit": "ms/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    elif args.workload == "conv":
        fn, flop, cores = ref_conv_sample()
        for _ in range(min(args.warmup, 1)):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        dt = (time.perf_counter() - t0) / args.steps
        v = flop / dt / 1e12
        line = {"impl": "reference", "metric": "VAE-decoder conv2d TFLOP/s (3x3, 4 stages of a 1024^2 decode)",
                "value": v, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": dt * 1e3 * sum(conv_flops()) / flop, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32 (CPU)", "data": "synthetic N(0,1) activations, N(0,0.02) weights",
                "config": {"workload": "conv2d 3x3 pad 1, C->C: " + ", ".join(f"{c}@{s}^2" for c, s in CONV_STAGES),
                           "sample": "the 512-channel 128^2 stage per step"},
                "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                                 "sample": "reference conv2d of the 512-channel 128^2 stage per step"},
                "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    else:
        fn, flop, cores, _ = ref_gemm_sample()
        for _ in range(args.warmup):
            fn()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            fn()
        dt = (time.perf_counter() - t0) / args.steps
        v = flop / dt / 1e12
        line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TFLOP/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3 * 8, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32 x bf16 -> f32 (CPU)",
                "data": "synthetic (seeded N(0,1) activations, N(0,0.02) bf16 weights)",
                "config": {"workload": "cfg1 fused-QKV GEMM 4096x11520x3840", "sample_rows": 512},
                "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                                 "sample": "512 of 4096 rows per step"},
                "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    line["reference_gpu"] = reference_gpu_line(args, world, local)
    if args.workload in ("dit", "unet"):
        line["reference_code_on_sdb200"] = dropin_line(args, world, local)
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
def timed_loop(fn, steps, stream, pg, dev):
    """CUDA-event time of `steps` calls on `stream`, barrier + synchronize on both sides,
    max over ranks."""
    import torch

    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        fn()
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b)
    if pg:
        pg.barrier()
    t = torch.tensor([ms], device=dev)
    if pg:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


# The skinny and epilogue-bound GEMM shapes of the DiT (HBM-bound: arithmetic intensity
# below the bf16 ridge of about 250 FLOP/byte), called the way the reference calls them
# (fp32 A, bf16 weights, fp32 out, bias): zimage.cpp:97-112 (adaLN), :171 (cap_embed),
# :198 (context refiner at M = 128 text tokens).
SKINNY_SHAPES = [
    ("adaln_gemv", 1, 15360, 256),
    ("cap_embed", 128, 3840, 2560),
    ("context_refiner_qkv", 128, 11520, 3840),
    ("context_refiner_w13", 128, 20480, 3840),
    ("context_refiner_w2", 128, 3840, 10240),
]


def skinny_shapes(dev, stream, hbm_peak, launches=40):
    """Device time per call of sdb200_gemm_nt_bf16 on each SKINNY_SHAPES entry. Each shape
    cycles through enough distinct weight matrices to hold more than 2x the 126 MB L2, so
    every call streams its weights from HBM. The calls are recorded once into a CUDA graph
    and replayed, so that the CUDA-event time is the kernels' (back to back on the device)
    and not the host's per-call launch cost; `host_us_per_call` is the same loop launched
    directly. Algorithmic bytes per call: weights 2NK + A 4MK + C 4MN + bias 4N."""
    import torch

    import sdb200
    from sdb200 import backend as be

    L = sdb200.lib()
    out = {}
    for name, M, N, K in SKINNY_SHAPES:
        wbytes = 2 * N * K
        copies = max(2, -(-(256 << 20) // wbytes))
        g = torch.Generator(device=dev)
        g.manual_seed(N + K)
        Ws = [(0.02 * torch.randn((N, K), generator=g, device=dev)).to(torch.bfloat16) for _ in range(copies)]
        A = torch.randn((M, K), generator=g, device=dev)
        bias = 0.01 * torch.randn((N,), generator=g, device=dev)
        C = torch.empty((M, N), device=dev)

        def call(i):
            sdb200.check(L.sdb200_gemm_nt_bf16(M, N, K, A.data_ptr(), K, Ws[i % copies].data_ptr(), K, C.data_ptr(),
                                               N, bias.data_ptr(), 0))

        for i in range(copies):
            call(i)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for i in range(launches):
            call(i)
        b.record(stream)
        torch.cuda.synchronize()
        host_ms = a.elapsed_time(b) / launches
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.graph(graph, stream=side):
            be.bind_stream()  # the library issues on the capturing stream
            for i in range(launches):
                call(i)
        be.bind_stream()
        graph.replay()
        torch.cuda.synchronize()
        a.record(stream)
        graph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / launches
        del graph
        nbytes = wbytes + 4 * M * K + 4 * M * N + 4 * N
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"M": M, "N": N, "K": K, "us_per_call": ms * 1e3, "host_us_per_call": host_ms * 1e3,
                     "bytes_per_call": nbytes, "gb_s": gbs, "frac_hbm": gbs / hbm_peak,
                     "tflops": 2.0 * M * N * K / (ms * 1e-3) / 1e12,
                     "path": "k_gemv_rows (exact fp32 A)" if M <= 16 else "bf16 pack + k_gemm_tc (split-K)",
                     "weights_cycled": copies}
        del Ws, A, bias, C
    torch.cuda.empty_cache()
    return out


def run_skinny(args, world, rank, local, pg, dev):
    """The skinny and epilogue-bound DiT GEMM shapes alone (SKINNY_SHAPES), through
    sdb200_gemm_nt_bf16 with fp32 A, each cycling through more than 2x L2 of weights.
    value = achieved HBM GB/s of the adaLN GEMV (M = 1, the first shape); the line lists
    every shape."""
    import torch

    from sdb200 import backend as be

    pk = peaks()
    stream = torch.cuda.current_stream()
    with ClockSampler(local) as clk:
        shapes = skinny_shapes(dev, stream, pk["hbm"], launches=max(args.steps, 8))
    first = shapes[SKINNY_SHAPES[0][0]]
    if rank == 0:
        print(json.dumps({
            "metric": "HBM GB/s of the DiT's skinny GEMMs (adaLN GEMV M=1 x 15360 x 256)", "value": first["gb_s"],
            "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": first["us_per_call"] * 1e-3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32 A, bf16 weights, fp32 accumulate",
            "data": "synthetic N(0,1) activations, N(0,0.02) weights",
            "config": {"workload": "skinny DiT GEMM shapes through gemm_nt_bf16", "parallelism": f"replicas x{world}",
                       "l2": "each shape cycles through > 256 MB of distinct weights"},
            "roofline": {"bound": "hbm", "kernel": "k_gemv_rows (adaLN GEMV)", "achieved": first["gb_s"],
                         "peak": pk["hbm"], "unit": "GB/s", "frac": first["gb_s"] / pk["hbm"],
                         "traffic": profile_value("skinny_gemm_shapes.md", "traffic_bytes_per_launch")},
            "shapes": shapes, "cpu_baseline": None, "clocks": clk.summary(),
            "device_error_word": be.device_error_word()}), flush=True)


def hbm_in_step(prof, hbm_peak):
    """GB/s of the memory-bound kernels timed live inside one profiled step (CUDA events
    around every launch on the library's stream), against the measured copy bandwidth."""
    out = {"peak_gb_s": hbm_peak, "peak_kind": "MEASURED_PEAKS.json hbm_gbs (copy)"}
    for key, kern in (("post_norm", "k_post_norm_mod_bcast_v4 (post-norm + gated residual + next RMSNorm x mod)"),
                      ("adaln", "k_gemv_rows (adaLN GEMV, M = 1, N = 15360, K = 256)")):
        ms, nbytes, n = prof.get(key + "_ms", 0.0), prof.get(key + "_bytes", 0.0), prof.get(key + "_launches", 0.0)
        if not ms:
            continue
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[key] = {"kernel": kern, "ms_per_step": ms, "launches_per_step": n, "bytes_per_launch": nbytes / n,
                    "gb_s": gbs, "frac_hbm": gbs / hbm_peak}
    if "post_norm" in out:
        out["post_norm"]["traffic_ncu_4096_rows"] = profile_value("post_norm_dit.md", "traffic_bytes_per_launch")
        out["post_norm"]["traffic_note"] = ("ncu DRAM read + write of one 4096-row launch "
                                            "(profiles/post_norm_dit.md; algorithmic 220 MB)")
    return out


def run_dit(args, world, rank, local, pg, dev):
    import numpy as np
    import torch

    import sdb200
    from sdb200 import backend as be
    from sdb200.zimage import Z_IMAGE, ZImageB200, random_weights_torch

    L = sdb200.lib()
    if GLOBAL_BATCH % world:
        raise SystemExit(f"global batch {GLOBAL_BATCH} does not split over {world} GPUs")
    B = args.dit_batch or GLOBAL_BATCH // world
    cfg = Z_IMAGE
    if args.dit_layers:
        import dataclasses

        cfg = dataclasses.replace(Z_IMAGE, layers=args.dit_layers)
    profiling_size = bool(args.dit_layers or args.dit_batch)
    wts = random_weights_torch(cfg, 0, dev)
    model = ZImageB200(wts, cfg)
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    x = torch.randn((B, cfg.in_channels, LAT_H, LAT_W), generator=g, device=dev)
    cap = torch.randn((B, TEXT_TOKENS, cfg.cap_dim), generator=g, device=dev)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    step = lambda: model.forward(x, 0.5, cap, out)  # noqa: E731
    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_loop(step, args.steps, stream, pg, dev)
    launches = L.sdb200_launch_count() - n0
    ms_step = ms / args.steps
    fl = dit_forward_flops(cfg)
    step_flop = B * world * fl["total"]

    # one profiled step: GEMM and attention kernels timed live with CUDA events
    model.profile(True)
    step()
    prof = model.profile_read()
    model.profile(False)
    pk = peaks()
    gemm_tf = prof["gemm_flop"] / (prof["gemm_ms"] * 1e-3) / 1e12 if prof["gemm_ms"] else None
    attn_tf = prof["attn_flop"] / (prof["attn_ms"] * 1e-3) / 1e12 if prof["attn_ms"] else None
    hbm = hbm_in_step(prof, pk["hbm"])

    # end to end through the C ABI: latents + text states in from pinned host memory,
    # prediction back out, every step
    xh = x.cpu().pin_memory()
    caph = cap.cpu().pin_memory()
    outh = torch.empty_like(out, device="cpu").pin_memory()
    xd, capd = torch.empty_like(x), torch.empty_like(cap)

    def e2e_step():
        sdb200.check(L.sdb200_upload(xd.data_ptr(), xh.data_ptr(), xh.numel() * 4))
        sdb200.check(L.sdb200_upload(capd.data_ptr(), caph.data_ptr(), caph.numel() * 4))
        model.forward(xd, 0.5, capd, out)
        sdb200.check(L.sdb200_download(outh.data_ptr(), out.data_ptr(), outh.numel() * 4))

    e2e_step()
    e2e_ms = timed_loop(e2e_step, args.steps, stream, pg, dev) / args.steps
    # The whole sampler of BASELINE config 4 (8 flow-matching Euler steps, shift 3,
    # scheduler.cpp:117-135) on the device, once, after the per-step timing.
    sampler_ms = timed_loop(lambda: model.sample(x, cap, steps=8, shift=3.0), 1, stream, pg, dev)
    if rank == 0 and not profiling_size:
        hbm["skinny_shapes_standalone"] = skinny_shapes(dev, stream, pk["hbm"])
    err = be.device_error_word()
    # At N > 1 the same run also times BASELINE config 5 (tensor parallelism over the N
    # ranks), so a scaling run records both multi-GPU modes.
    tp = None
    if world > 1:
        del model, wts
        torch.cuda.empty_cache()
        tp = measure_tp(args, world, rank, local, pg, dev, check_vs_single=True)
        err |= be.device_error_word()
    cpu = cpu_baseline("dit") if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": ms_step, "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 GEMM operands, fp16 attention operands, fp32 accumulate/activations",
            "data": "synthetic (random-init Z-Image-shaped weights, N(0,1) latents and text states)",
            "config": {"workload": "cfg4: 30-layer Z-Image DiT (dim 3840, 30 heads, FFN 10240, 2+2 refiners) "
                                   "@1024^2, 128 text tokens, global batch 8 images per denoising step",
                       "global_batch": GLOBAL_BATCH, "images_per_gpu": B, "seq_len": 4224,
                       "parallelism": f"image-parallel x{world} (no collective)",
                       "l2": "weights 12.3 GB + activations > 126 MB L2 per step, no flush needed"},
            "images_per_s": B * world / (ms_step * 1e-3),
            "step_tflops": step_flop / (ms_step * 1e-3) / 1e12,
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc_pair / k_gemm_tc (all GEMMs of one step, rank 0)",
                         "achieved": gemm_tf, "peak": pk["sustained"], "unit": "TFLOP/s",
                         "frac": (gemm_tf / pk["sustained"]) if gemm_tf else None,
                         "peak_kind": f"{pk['kind']} bf16 sustained",
                         "traffic": profile_value("gemm_tc_cfg1.md", "traffic_bytes_per_launch"),
                         "traffic_note": "ncu DRAM bytes of the cfg1 GEMM launch (profiles/gemm_tc_cfg1.md)",
                         "gemm_ms_per_step": prof["gemm_ms"], "gemm_launches_per_step": prof["gemm_launches"],
                         "attention_tflops": attn_tf, "attention_ms_per_step": prof["attn_ms"],
                         "forward_ms_profiled": prof["forward_ms"]},
            "e2e": {"value": e2e_ms, "unit": "ms/step", "h2d_bytes_per_step": int((xh.numel() + caph.numel()) * 4),
                    "d2h_bytes_per_step": int(outh.numel() * 4)},
            "sampler_8_steps": {"ms": sampler_ms, "ms_per_step": sampler_ms / 8,
                                "note": "sdb200_zimage_sample: 8 flow-matching Euler steps, shift 3, on the device"},
            "hbm_kernels": hbm,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "device_error_word": err,
        }
        if tp is not None:
            line["cfg5_tp"] = tp
        if profiling_size:
            line["config"]["workload"] = (f"PROFILING SIZE, not config 4: {cfg.layers}-layer Z-Image DiT @1024^2, "
                                          f"{B} image(s) per GPU")
            line["config"]["global_batch"] = B * world
        print(json.dumps(line), flush=True)


def measure_tp(args, world, rank, local, pg, dev, check_vs_single=False):
    """BASELINE config 5 on the N ranks: the 30-layer DiT at batch 1, 2048x2048 (256x256
    latent: 16384 image + 128 text tokens), Megatron tensor parallelism (column-parallel
    QKV by heads and w1/w3, row-parallel to_out and w2; --tp-mode 1 combines the
    row-parallel outputs inside the kernels over NVLink, 0 with an NCCL all-reduce).
    Returns the measurements (every rank); with check_vs_single, rank 0 also runs the
    unsharded model on its GPU and reports the relative error of the TP output."""
    import torch

    import sdb200
    from sdb200 import backend as be
    from sdb200.tp import Comm, shard_weights
    from sdb200.zimage import Z_IMAGE, ZImageB200, random_weights_torch

    L = sdb200.lib()
    cfg = Z_IMAGE
    H = W = 256
    full = random_weights_torch(cfg, 0, dev)
    shards = shard_weights(full, cfg.heads, cfg.dim // cfg.heads, rank, world)
    del full
    torch.cuda.empty_cache()
    model = ZImageB200(shards, cfg)
    comm = Comm(rank, world, None)
    comm.set_barrier(args.tp_barrier == "flags")
    model.set_tp(comm, mode=args.tp_mode)
    g = torch.Generator(device=dev)
    g.manual_seed(2000)  # every rank holds the same image and text states
    x = torch.randn((1, cfg.in_channels, H, W), generator=g, device=dev)
    cap = torch.randn((1, TEXT_TOKENS, cfg.cap_dim), generator=g, device=dev)
    out = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    step = lambda: model.forward(x, 0.5, cap, out)  # noqa: E731
    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_loop(step, args.steps, stream, pg, dev)
    launches = L.sdb200_launch_count() - n0
    ms_step = ms / args.steps
    model.profile(True)
    step()
    prof = model.profile_read()
    model.profile(False)
    fl = dit_forward_flops(cfg, H, W)
    pk = peaks()
    gemm_tf = prof["gemm_flop"] / (prof["gemm_ms"] * 1e-3) / 1e12 if prof["gemm_ms"] else None
    attn_tf = prof["attn_flop"] / (prof["attn_ms"] * 1e-3) / 1e12 if prof["attn_ms"] else None
    xh, caph = x.cpu().pin_memory(), cap.cpu().pin_memory()
    outh = torch.empty_like(out, device="cpu").pin_memory()
    xd, capd = torch.empty_like(x), torch.empty_like(cap)

    def e2e_step():
        sdb200.check(L.sdb200_upload(xd.data_ptr(), xh.data_ptr(), xh.numel() * 4))
        sdb200.check(L.sdb200_upload(capd.data_ptr(), caph.data_ptr(), caph.numel() * 4))
        model.forward(xd, 0.5, capd, out)
        sdb200.check(L.sdb200_download(outh.data_ptr(), out.data_ptr(), outh.numel() * 4))

    e2e_step()
    e2e_ms = timed_loop(e2e_step, args.steps, stream, pg, dev) / args.steps
    # every rank holds the whole output: the largest difference from rank 0's copy
    y0 = out.clone()
    if pg:
        pg.broadcast(y0, src=0)
    rank_diff = torch.tensor([float((out - y0).abs().max().item())], device=dev)
    if pg:
        pg.all_reduce(rank_diff, op=pg.ReduceOp.MAX)
    hbm = hbm_in_step(prof, pk["hbm"])
    model.set_tp(None)
    comm.close()
    del model, shards
    torch.cuda.empty_cache()
    rel = None
    if check_vs_single and rank == 0:
        single = ZImageB200(random_weights_torch(cfg, 0, dev), cfg)
        ys = single.forward(x, 0.5, cap)
        torch.cuda.synchronize()
        rel = float((out.double() - ys.double()).norm() / ys.double().norm())
        del single, ys
        torch.cuda.empty_cache()
    if pg:
        pg.barrier()
    comm_ms = prof["allreduce_ms"]
    return {
        "workload": "cfg5: 30-layer Z-Image DiT @2048^2 (16512 tokens), batch 1, one denoising step",
        "ms_per_step": ms_step, "e2e_ms_per_step": e2e_ms, "tp_ranks": world, "steps": args.steps,
        "parallelism": f"tensor-parallel x{world} (column QKV/w1/w3, row to_out/w2; " + (
            "partial rows scattered to their owner rank from the GEMM epilogue over NVLink, "
            "sequence-sharded post-norm broadcasting the next bf16 input)" if args.tp_mode == 1 else
            "NCCL all-reduce fp32)"),
        "tp_mode": args.tp_mode, "tp_barrier": args.tp_barrier if args.tp_mode == 1 else None,
        "communicator_ranks": world, "step_tflops": fl["total"] / (ms_step * 1e-3) / 1e12,
        "gemm_ms_per_step": prof["gemm_ms"], "gemm_tflops": gemm_tf, "attention_ms_per_step": prof["attn_ms"],
        "attention_tflops": attn_tf, "comm_ms_per_step": comm_ms, "comm_calls_per_step": prof["allreduces"],
        "comm_share": comm_ms / prof["forward_ms"] if prof["forward_ms"] else None,
        "forward_ms_profiled": prof["forward_ms"], "hbm_kernels": hbm, "gpu_launches": int(launches),
        "max_rank_diff": float(rank_diff.item()), "rel_err_vs_single_gpu": rel,
        "e2e": {"value": e2e_ms, "unit": "ms/step", "h2d_bytes_per_step": int((xh.numel() + caph.numel()) * 4),
                "d2h_bytes_per_step": int(outh.numel() * 4)},
        "gemm_peak": pk["sustained"], "clocks": clk.summary(),
    }


def run_dit_tp(args, world, rank, local, pg, dev):
    """BASELINE config 5 as the line's own workload (see measure_tp). Total work fixed:
    "scaling": "strong"."""
    from sdb200 import backend as be

    tp = measure_tp(args, world, rank, local, pg, dev)
    err = be.device_error_word()
    if rank == 0:
        gemm_tf, peak = tp["gemm_tflops"], tp["gemm_peak"]
        print(json.dumps({
            "metric": METRIC, "value": tp["ms_per_step"], "unit": "ms/step", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tp["ms_per_step"], "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 GEMM operands, fp16 attention operands, fp32 accumulate/activations",
            "data": "synthetic (random-init Z-Image-shaped weights, N(0,1) latent and text states)",
            "config": {"workload": tp["workload"], "global_batch": 1, "seq_len": 16512,
                       "parallelism": tp["parallelism"], "tp_barrier": tp["tp_barrier"]},
            "step_tflops": tp["step_tflops"], "gpu_launches": tp["gpu_launches"],
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc_pair / k_gemm_tc (all GEMMs of one step, rank 0)",
                         "achieved": gemm_tf, "peak": peak, "unit": "TFLOP/s",
                         "frac": (gemm_tf / peak) if gemm_tf else None, "peak_kind": "bf16 sustained",
                         "traffic": None, "gemm_ms_per_step": tp["gemm_ms_per_step"],
                         "attention_tflops": tp["attention_tflops"],
                         "attention_ms_per_step": tp["attention_ms_per_step"],
                         "comm_ms_per_step": tp["comm_ms_per_step"], "comm_calls_per_step": tp["comm_calls_per_step"],
                         "forward_ms_profiled": tp["forward_ms_profiled"]},
            "hbm_kernels": tp["hbm_kernels"], "e2e": tp["e2e"], "max_rank_diff": tp["max_rank_diff"],
            "cpu_baseline": None, "clocks": tp["clocks"], "device_error_word": err}), flush=True)


def run_gemm(args, world, rank, local, pg, dev):
    import torch

    import sdb200
    from sdb200 import backend as be
    from sdb200.workloads import cfg1_inputs, f32_to_bf16_bits

    L = sdb200.lib()
    M, N, K = 4096, 11520, 3840
    FLOP = 2.0 * M * N * K
    X, W, b = cfg1_inputs()
    Wbits = f32_to_bf16_bits(W)
    Xd = torch.from_numpy(X).to(dev)
    Wd = torch.from_numpy(Wbits.view("int16")).to(dev).view(torch.bfloat16)
    bd = torch.from_numpy(b).to(dev)
    Yd = torch.empty((M, N), device=dev)
    stream = torch.cuda.current_stream()

    def step():
        sdb200.check(L.sdb200_gemm_nt_bf16(M, N, K, Xd.data_ptr(), K, Wd.data_ptr(), K, Yd.data_ptr(), N,
                                           bd.data_ptr(), 0))

    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_loop(step, args.steps, stream, pg, dev)
    launches = L.sdb200_launch_count() - n0
    value = FLOP * args.steps * world / (ms * 1e-3) / 1e12
    # the tensor-core kernel alone (A pre-packed to bf16)
    Xbf = Xd.to(torch.bfloat16)
    kstep = lambda: sdb200.check(L.sdb200_gemm_nt_bf16a(M, N, K, Xbf.data_ptr(), K, Wd.data_ptr(), K,  # noqa: E731
                                                         Yd.data_ptr(), N, bd.data_ptr(), 0))
    for _ in range(3):
        kstep()
    reps = max(args.steps, 10)
    kms = timed_loop(kstep, reps, stream, None, dev) / reps
    pk = peaks()
    achieved = FLOP / (kms * 1e-3) / 1e12
    Xh = torch.from_numpy(X).pin_memory()
    Yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
    Xs = torch.empty_like(Xd)

    def e2e_step():
        sdb200.check(L.sdb200_upload(Xs.data_ptr(), Xh.data_ptr(), Xh.numel() * 4))
        sdb200.check(L.sdb200_gemm_nt_bf16(M, N, K, Xs.data_ptr(), K, Wd.data_ptr(), K, Yd.data_ptr(), N,
                                           bd.data_ptr(), 0))
        sdb200.check(L.sdb200_download(Yh.data_ptr(), Yd.data_ptr(), Yh.numel() * 4))

    e2e_step()
    e2e_ms = timed_loop(e2e_step, args.steps, stream, pg, dev)
    e2e_value = FLOP * args.steps * world / (e2e_ms * 1e-3) / 1e12
    err = be.device_error_word()
    cpu = cpu_baseline("gemm") if (rank == 0 and world == 1 and not args.no_cpu_baseline) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 x bf16 -> f32 (A rounded from f32)",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02) bf16 weights, N(0,0.01) bias)",
            "config": {"workload": "cfg1 fused-QKV GEMM Y[4096,11520] = X[4096,3840] W[11520,3840]^T + b",
                       "global_batch": world, "parallelism": f"replicas x{world} (no collective)",
                       "l2": "inputs 340 MB/step > 126 MB L2, no flush"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc_pair (tcgen05 kind::f16, cta_group::2, 256x256 tiles on SM pairs)",
                         "achieved": achieved, "peak": pk["burst"], "unit": "TFLOP/s", "frac": achieved / pk["burst"],
                         "peak_kind": f"{pk['kind']} bf16 burst",
                         "traffic": profile_value("gemm_tc_cfg1.md", "traffic_bytes_per_launch"), "kernel_ms": kms},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": int(Xh.numel() * 4),
                    "d2h_bytes_per_step": int(Yh.numel() * 4)},
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "device_error_word": err,
        }
        print(json.dumps(line), flush=True)


def run_attention(args, world, rank, local, pg, dev):
    """The Z-Image joint-sequence attention at 1024^2 (one image): 4224 tokens, 30 heads
    of 128, non-causal. value = TFLOP/s of the tensor-core kernel on fp16 operands
    resident in HBM (4*S^2*d*heads per launch); e2e = the drop-in fp32 API with host
    buffers."""
    import torch

    import sdb200
    from sdb200 import backend as be

    L = sdb200.lib()
    S, H, d, dp = 4224, 30, 128, 128
    FLOP = 4.0 * S * S * d * H
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    q = torch.randn((1, S, H * d), generator=g, device=dev)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    o = torch.empty_like(q)
    q16, k16, v16 = (torch.empty(S * H * dp, dtype=torch.float16, device=dev) for _ in range(3))
    for x, y in ((q, q16), (k, k16), (v, v16)):
        sdb200.check(L.sdb200_pack_heads_f16(x.data_ptr(), y.data_ptr(), S, H, d, dp))
    stream = torch.cuda.current_stream()
    step = lambda: sdb200.check(L.sdb200_attention_f16(q16.data_ptr(), k16.data_ptr(), v16.data_ptr(),  # noqa: E731
                                                       o.data_ptr(), 0, 1, S, S, H, H, d, dp, 0))
    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_loop(step, args.steps, stream, pg, dev)
    launches = L.sdb200_launch_count() - n0
    value = FLOP * args.steps * world / (ms * 1e-3) / 1e12
    qh, kh, vh = (t.cpu().pin_memory() for t in (q, k, v))
    oh = torch.empty_like(qh).pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(q), torch.empty_like(q)

    def e2e_step():
        for hsrc, ddst in ((qh, qd), (kh, kd), (vh, vd)):
            sdb200.check(L.sdb200_upload(ddst.data_ptr(), hsrc.data_ptr(), hsrc.numel() * 4))
        sdb200.check(L.sdb200_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), 1, S, S, H, H, d, 0))
        sdb200.check(L.sdb200_download(oh.data_ptr(), o.data_ptr(), oh.numel() * 4))

    e2e_step()
    e2e_ms = timed_loop(e2e_step, args.steps, stream, pg, dev)
    pk = peaks()
    if rank == 0:
        achieved = FLOP / (ms / args.steps * 1e-3) / 1e12
        print(json.dumps({
            "metric": "attention TFLOP/s (Z-Image joint attention @1024^2)", "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 operands, fp32 accumulate and softmax", "data": "synthetic N(0,1) q/k/v",
            "config": {"workload": "attention S=4224 heads=30 d=128 non-causal, fp16 packed operands",
                       "parallelism": f"replicas x{world}"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "k_attention_tc<128>", "achieved": achieved,
                         "peak": pk["burst"], "unit": "TFLOP/s", "frac": achieved / pk["burst"],
                         "peak_kind": f"{pk['kind']} bf16 burst (dense fp16 = bf16 rate)", "traffic": None},
            "e2e": {"value": FLOP * args.steps * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(3 * qh.numel() * 4), "d2h_bytes_per_step": int(oh.numel() * 4)},
            "cpu_baseline": None, "clocks": clk.summary(),
            "device_error_word": be.device_error_word()}), flush=True)


# The VAE decoder's 3x3 convolution at each resolution stage of a 1024^2 decode (channels,
# side): 512 @ 128^2, 512 @ 256^2, 256 @ 512^2, 128 @ 1024^2 (AutoencoderKL decoder, vae.cpp).
CONV_STAGES = [(512, 128), (512, 256), (256, 512), (128, 1024)]


def conv_flops():
    return [2.0 * c * c * 9 * s * s for c, s in CONV_STAGES]


def ref_conv_sample():
    """The reference's CPU conv2d (tensor.cpp:529-586) on the smallest stage."""
    import numpy as np

    from oracle import RefCPU

    ref = RefCPU()
    ref.set_num_threads(0)
    c, s = CONV_STAGES[0]
    rng = np.random.default_rng(5)
    x = rng.standard_normal((1, c, s, s)).astype(np.float32)
    w = (0.02 * rng.standard_normal((c, c, 3, 3))).astype(np.float32)
    b = (0.02 * rng.standard_normal(c)).astype(np.float32)
    return (lambda: ref.conv2d(x, w, b, 1, 1)), conv_flops()[0], ref.num_threads()


def run_conv(args, world, rank, local, pg, dev):
    """One step = the four VAE-decoder stage convolutions (3x3, pad 1, C -> C, batch 1)
    through the reference API (sdb200_conv2d: NHWC repack + implicit GEMM). value =
    TFLOP/s over the step; roofline = the implicit-GEMM kernel alone on packed operands
    (sdb200_conv2d_nhwc), against a cuBLAS tf32 GEMM measured in the same run."""
    import torch

    import sdb200
    from sdb200 import backend as be

    global CONV_STAGES
    if args.conv_stage >= 0:
        CONV_STAGES = [CONV_STAGES[args.conv_stage]]
    L = sdb200.lib()
    g = torch.Generator(device=dev)
    g.manual_seed(31 + rank)
    bufs = []
    for c, s in CONV_STAGES:
        x = torch.randn((1, c, s, s), generator=g, device=dev)
        w = 0.02 * torch.randn((c, c, 3, 3), generator=g, device=dev)
        b = 0.02 * torch.randn((c,), generator=g, device=dev)
        bufs.append((c, s, x, w, b, torch.empty_like(x)))
    flops = conv_flops()
    FLOP = sum(flops)
    stream = torch.cuda.current_stream()

    def step():
        for c, s, x, w, b, y in bufs:
            sdb200.check(L.sdb200_conv2d(x.data_ptr(), 1, c, s, s, w.data_ptr(), c, 3, 3, b.data_ptr(), 1, 1,
                                         y.data_ptr(), s, s))

    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_loop(step, args.steps, stream, pg, dev)
    launches = L.sdb200_launch_count() - n0
    value = FLOP * args.steps * world / (ms * 1e-3) / 1e12
    # the implicit-GEMM kernel alone, operands packed once
    packed = []
    for c, s, x, w, b, y in bufs:
        xh = torch.empty(s * s * c, device=dev)
        wp = torch.empty(c * 9 * c, device=dev)
        sdb200.check(L.sdb200_conv_pack_input(x.data_ptr(), xh.data_ptr(), 1, c, s * s, c))
        sdb200.check(L.sdb200_conv_pack_weight(w.data_ptr(), wp.data_ptr(), c, c, 9, c))
        packed.append((c, s, xh, wp, b, y))
    kstep = lambda: [sdb200.check(L.sdb200_conv2d_nhwc(xh.data_ptr(), 1, c, c, s, s, wp.data_ptr(), c, c, 3, 3, 1,  # noqa: E731
                                                       b.data_ptr(), None, y.data_ptr(), s, s))
                     for c, s, xh, wp, b, y in packed]
    for _ in range(3):
        kstep()
    reps = max(args.steps, 5)
    kms = timed_loop(kstep, reps, stream, None, dev) / reps
    achieved = FLOP / (kms * 1e-3) / 1e12
    # cuBLAS tf32 reference rate on the same stream (8192^3, as the bf16 peak is measured)
    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    A = torch.randn((8192, 8192), device=dev)
    B = torch.randn((8192, 8192), device=dev)
    for _ in range(3):
        torch.matmul(A, B)
    tms = min(timed_loop(lambda: torch.matmul(A, B), 5, stream, None, dev) / 5 for _ in range(2))
    torch.backends.cuda.matmul.allow_tf32 = allow
    tf32_peak = 2.0 * 8192 ** 3 / (tms * 1e-3) / 1e12
    del A, B
    # end to end: host NCHW activations in, host outputs back, per stage
    hosts = [(c, s, x.cpu().pin_memory(), torch.empty(x.shape).pin_memory(), x, w, b, y) for c, s, x, w, b, y in bufs]

    def e2e_step():
        for c, s, xh_, yh, x, w, b, y in hosts:
            sdb200.check(L.sdb200_upload(x.data_ptr(), xh_.data_ptr(), xh_.numel() * 4))
            sdb200.check(L.sdb200_conv2d(x.data_ptr(), 1, c, s, s, w.data_ptr(), c, 3, 3, b.data_ptr(), 1, 1,
                                         y.data_ptr(), s, s))
            sdb200.check(L.sdb200_download(yh.data_ptr(), y.data_ptr(), yh.numel() * 4))

    e2e_step()
    e2e_ms = timed_loop(e2e_step, args.steps, stream, pg, dev)
    io = sum(h[2].numel() * 4 for h in hosts)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            fn, f0, cores = ref_conv_sample()
            fn()
            t0 = time.perf_counter()
            fn()
            dt = time.perf_counter() - t0
            cpu = {"value": f0 / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "reference",
                   "sample": f"reference conv2d (im2col + CPU GEMM) of the 512-channel 128^2 stage ({dt:.2f} s)"}
        except Exception as e:  # reported, never required
            cpu = {"value": None, "unit": None, "cores": None, "kind": "reference", "sample": f"failed: {e}"}
    if rank == 0:
        print(json.dumps({
            "metric": "VAE-decoder conv2d TFLOP/s (3x3, 4 stages of a 1024^2 decode)", "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32 activations and weights, tf32 tensor cores, f32 accumulate",
            "data": "synthetic N(0,1) activations, N(0,0.02) weights and bias",
            "config": {"workload": "conv2d 3x3 pad 1, C->C: " + ", ".join(f"{c}@{s}^2" for c, s in CONV_STAGES),
                       "parallelism": f"replicas x{world}", "l2": "inputs 1 GB/step > 126 MB L2, no flush"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "k_gemm_tc<256, tf32, conv> (implicit GEMM, NHWC TMA boxes)",
                         "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s", "frac": achieved / tf32_peak,
                         "peak_kind": "cuBLAS tf32 8192^3 measured live in this run (burst)", "kernel_ms": kms,
                         "traffic": profile_value("conv_tc_vae.md", "traffic_bytes_per_step")},
            "e2e": {"value": FLOP * args.steps * world / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": int(io), "d2h_bytes_per_step": int(io)},
            "cpu_baseline": cpu, "clocks": clk.summary(),
            "device_error_word": be.device_error_word()}), flush=True)


def ref_vae_sample(side=32):
    """The reference's VAEDecoder::decode (vae.cpp:35-51) with the FLUX / Z-Image VAE's
    widths on a side x side latent (a 8*side image), random-init weights."""
    import numpy as np

    from oracle import RefCPU
    from sdb200.vae import FLUX_VAE, decode_flops, random_weights

    ref = RefCPU()
    ref.set_num_threads(0)
    m = ref.vae(random_weights(FLUX_VAE, 7), FLUX_VAE.scaling_factor, FLUX_VAE.shift_factor)
    z = np.random.default_rng(8).standard_normal((1, FLUX_VAE.latent_channels, side, side)).astype(np.float32)
    return (lambda: m(z)), decode_flops(FLUX_VAE, side, side), ref.num_threads(), m


def run_vae(args, world, rank, local, pg, dev):
    """One step = one VAE decode of a 1024^2 image (latent [1, 16, 128, 128] -> [1, 3, 1024,
    1024]) through sdb200_vae_decode, per GPU (replicas). value = ms per decode."""
    import ctypes as C

    import numpy as np
    import torch

    import sdb200
    from sdb200 import backend as be
    from sdb200.vae import FLUX_VAE, VAE, decode_flops, random_weights

    L = sdb200.lib()
    cfg = FLUX_VAE
    side = LAT_H
    FLOP = decode_flops(cfg, side, side)
    v = VAE(cfg, random_weights(cfg, 7))
    g = torch.Generator(device=dev)
    g.manual_seed(9 + rank)
    z = torch.randn((1, cfg.latent_channels, side, side), generator=g, device=dev)
    out = torch.empty((1, 3, side * v.upscale, side * v.upscale), device=dev)
    stream = torch.cuda.current_stream()
    step = lambda: v.decode(z, out)  # noqa: E731
    for _ in range(args.warmup):
        step()
    n0 = L.sdb200_launch_count()
    with ClockSampler(local) as clk:
        ms = timed_loop(step, args.steps, stream, pg, dev)
    launches = L.sdb200_launch_count() - n0
    # one profiled decode: convolution kernels alone (CUDA events around each launch)
    sdb200.check(L.sdb200_vae_profile(v.h, 1))
    step()
    prof = (C.c_double * 5)()
    sdb200.check(L.sdb200_vae_profile_read(v.h, prof))
    sdb200.check(L.sdb200_vae_profile(v.h, 0))
    conv_ms, conv_flop, conv_n, att_ms, att_flop = list(prof)
    # cuBLAS tf32 rate measured on the same stream as the denominator
    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    A = torch.randn((8192, 8192), device=dev)
    B = torch.randn((8192, 8192), device=dev)
    for _ in range(3):
        torch.matmul(A, B)
    tms = min(timed_loop(lambda: torch.matmul(A, B), 5, stream, None, dev) / 5 for _ in range(2))
    torch.backends.cuda.matmul.allow_tf32 = allow
    tf32_peak = 2.0 * 8192 ** 3 / (tms * 1e-3) / 1e12
    del A, B
    zh = z.cpu().pin_memory()
    oh = torch.empty(out.shape).pin_memory()
    zd = torch.empty_like(z)

    def e2e_step():
        sdb200.check(L.sdb200_upload(zd.data_ptr(), zh.data_ptr(), zh.numel() * 4))
        v.decode(zd, out)
        sdb200.check(L.sdb200_download(oh.data_ptr(), out.data_ptr(), oh.numel() * 4))

    e2e_step()
    e2e_ms = timed_loop(e2e_step, args.steps, stream, pg, dev)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            fn, f0, cores, _keep = ref_vae_sample()
            t0 = time.perf_counter()
            fn()
            dt = time.perf_counter() - t0
            cpu = {"value": dt * 1e3 * FLOP / f0, "unit": "ms/decode", "cores": cores, "kind": "reference",
                   "sample": f"reference VAEDecoder::decode of a 256^2 image ({f0 / 1e12:.2f} TFLOP, {dt:.2f} s), "
                             f"scaled by FLOPs to 1024^2 ({FLOP / 1e12:.2f} TFLOP)"}
        except Exception as e:  # reported, never required
            cpu = {"value": None, "unit": None, "cores": None, "kind": "reference", "sample": f"failed: {e}"}
    if rank == 0:
        achieved = conv_flop / (conv_ms * 1e-3) / 1e12
        per = ms / args.steps
        print(json.dumps({
            "metric": "VAE decode ms (1024^2 image, FLUX / Z-Image VAE)", "value": per, "unit": "ms/decode",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": per,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None,
            "tflops": FLOP / (per * 1e-3) / 1e12,
            "dtype": "f32 activations and weights, tf32 tensor cores, f32 accumulate",
            "data": "synthetic (random-init weights, N(0,1) latent)",
            "config": {"workload": "AutoencoderKL decoder (16 latent ch, widths 128/256/512/512, 3 resnets per up "
                                   "block, 1-head mid attention), latent 16x128x128 -> 3x1024x1024",
                       "parallelism": f"replicas x{world}", "l2": "activations up to 1 GB per layer > 126 MB L2"},
            "gpu_launches": int(launches),
            "roofline": {"bound": "tensor", "kernel": "implicit-GEMM conv (k_gemm_tc_pair<conv>, k_gemm_tc<256,tf32,conv>)",
                         "achieved": achieved, "peak": tf32_peak, "unit": "TFLOP/s", "frac": achieved / tf32_peak,
                         "peak_kind": "cuBLAS tf32 8192^3 measured live in this run (burst)",
                         "conv_ms": conv_ms, "conv_launches": int(conv_n), "attention_ms": att_ms,
                         "attention_tflops": att_flop / (att_ms * 1e-3) / 1e12 if att_ms else None,
                         "traffic": None},
            "e2e": {"value": e2e_ms / args.steps, "unit": "ms/decode", "h2d_bytes_per_step": int(zh.numel() * 4),
                    "d2h_bytes_per_step": int(oh.numel() * 4)},
            "cpu_baseline": cpu, "clocks": clk.summary(),
            "device_error_word": be.device_error_word()}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="dit",
                    choices=["dit", "dit_tp", "gemm", "attention", "conv", "vae", "unet", "skinny"])
    ap.add_argument("--dit-layers", type=int, default=0,
                    help="dit: profiling size - this many main layers instead of 30 (the line then says so)")
    ap.add_argument("--dit-batch", type=int, default=0,
                    help="dit: profiling size - this many images per GPU instead of 8 / N")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="skip the reference GPU backend comparison (oracle/_ref/libsdref_cuda.so)")
    ap.add_argument("--conv-stage", type=int, default=-1, choices=[-1, 0, 1, 2, 3],
                    help="conv: run only this stage of the VAE-decoder stack (-1: all four)")
    ap.add_argument("--tp-mode", type=int, default=1, choices=[0, 1],
                    help="dit_tp: 1 = exchange fused into the GEMM epilogue and post-norm over NVLink, "
                         "0 = NCCL all-reduce")
    ap.add_argument("--tp-barrier", default="flags", choices=["flags", "nccl"],
                    help="dit_tp --tp-mode 1: barrier between the fused kernels, a flag exchange over "
                         "NVLink or a 4-byte NCCL all-reduce")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, world, rank, local)

    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist
    import sdb200
    from sdb200 import backend as be

    if not sdb200.available():
        raise SystemExit("libsdb200: no usable sm_100 device: " + sdb200.lib().sdb200_last_error().decode())
    be.bind_stream()
    if args.workload == "dit":
        run_dit(args, world, rank, local, pg, dev)
    elif args.workload == "attention":
        run_attention(args, world, rank, local, pg, dev)
    elif args.workload == "dit_tp":
        run_dit_tp(args, world, rank, local, pg, dev)
    elif args.workload == "conv":
        run_conv(args, world, rank, local, pg, dev)
    elif args.workload == "vae":
        run_vae(args, world, rank, local, pg, dev)
    elif args.workload == "unet":
        run_unet(args, world, rank, local, pg, dev)
    elif args.workload == "skinny":
        run_skinny(args, world, rank, local, pg, dev)
    else:
        run_gemm(args, world, rank, local, pg, dev)
    if pg:
        pg.barrier()
        pg.destroy_process_group()


if __name__ == "__main__":
    main()
