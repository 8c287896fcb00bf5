"""Z-Image DiT on libsdb200 (sdb200_zimage_* C ABI) plus random-init weights under the
checkpoint names the reference binds (src/zimage.cpp:38-67).

No checkpoint exists here, so weights are random (seeded): linear weights ~N(0, 0.02),
biases ~N(0, 0.01), norm gammas ~N(1, 0.02), pad tokens ~N(0, 1). Storage follows the
reference loader (safetensors.cpp:119 keeps tensors of >= 2^20 elements in bf16): every
block linear and cap_embedder.1 are bf16, the small layers fp32. `Z_IMAGE` holds the
published model's hyper-parameters (zimage.h:40-47; dim 3840, 30 heads, FFN 10240,
30 layers + 2 noise and 2 context refiners, 16 latent channels, text width 2560).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import check, lib
from .workloads import f32_to_bf16_bits


@dataclass(frozen=True)
class ZConfig:
    dim: int = 3840
    heads: int = 30
    ffn: int = 10240
    t_dim: int = 256          # sinusoid width = adaLN input width
    t_hidden: int = 1024      # t_embedder.mlp.0 output
    cap_dim: int = 2560       # text hidden width (Qwen3-4B)
    in_channels: int = 16
    patch: int = 2
    layers: int = 30
    noise_refiners: int = 2
    context_refiners: int = 2
    norm_eps: float = 1e-5
    rope_theta: float = 256.0
    t_scale: float = 1000.0
    axes: tuple = (32, 48, 48)


Z_IMAGE = ZConfig()


def weight_specs(cfg: ZConfig):
    """[(name, shape, kind, bf16)] with kind in {"w", "b", "g", "tok"}."""
    D, F, T, TH, CD = cfg.dim, cfg.ffn, cfg.t_dim, cfg.t_hidden, cfg.cap_dim
    pc = cfg.patch * cfg.patch * cfg.in_channels
    hd = D // cfg.heads
    s = [
        ("all_x_embedder.2-1.weight", (D, pc), "w", False), ("all_x_embedder.2-1.bias", (D,), "b", False),
        ("cap_embedder.0.weight", (CD,), "g", False),
        ("cap_embedder.1.weight", (D, CD), "w", True), ("cap_embedder.1.bias", (D,), "b", False),
        ("t_embedder.mlp.0.weight", (TH, T), "w", False), ("t_embedder.mlp.0.bias", (TH,), "b", False),
        ("t_embedder.mlp.2.weight", (T, TH), "w", False), ("t_embedder.mlp.2.bias", (T,), "b", False),
        ("all_final_layer.2-1.linear.weight", (pc, D), "w", False),
        ("all_final_layer.2-1.linear.bias", (pc,), "b", False),
        ("all_final_layer.2-1.adaLN_modulation.1.weight", (D, T), "w", False),
        ("all_final_layer.2-1.adaLN_modulation.1.bias", (D,), "b", False),
        ("x_pad_token", (1, D), "tok", False), ("cap_pad_token", (1, D), "tok", False),
    ]

    def block(p, modulated):
        out = [(p + ".attention_norm1.weight", (D,), "g", False), (p + ".attention_norm2.weight", (D,), "g", False),
               (p + ".ffn_norm1.weight", (D,), "g", False), (p + ".ffn_norm2.weight", (D,), "g", False),
               (p + ".attention.norm_q.weight", (hd,), "g", False), (p + ".attention.norm_k.weight", (hd,), "g", False)]
        for n in ("to_q", "to_k", "to_v", "to_out.0"):
            out.append((p + ".attention." + n + ".weight", (D, D), "w", True))
        out += [(p + ".feed_forward.w1.weight", (F, D), "w", True), (p + ".feed_forward.w2.weight", (D, F), "w", True),
                (p + ".feed_forward.w3.weight", (F, D), "w", True)]
        if modulated:
            out += [(p + ".adaLN_modulation.0.weight", (4 * D, T), "w", True),
                    (p + ".adaLN_modulation.0.bias", (4 * D,), "b", False)]
        return out

    for i in range(cfg.noise_refiners):
        s += block(f"noise_refiner.{i}", True)
    for i in range(cfg.context_refiners):
        s += block(f"context_refiner.{i}", False)
    for i in range(cfg.layers):
        s += block(f"layers.{i}", True)
    return s


def _scale(kind):
    return {"w": (0.0, 0.02), "b": (0.0, 0.01), "g": (1.0, 0.02), "tok": (0.0, 1.0)}[kind]


def random_weights_numpy(cfg: ZConfig, seed: int = 0):
    """name -> fp32 numpy array (bf16-stored weights are returned already rounded to
    their bf16 values), and the set of bf16-stored names."""
    rng = np.random.default_rng(seed)
    out, bf = {}, set()
    for name, shape, kind, is_bf16 in weight_specs(cfg):
        mu, sd = _scale(kind)
        a = (mu + sd * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        if is_bf16:
            a = (f32_to_bf16_bits(a).astype(np.uint32) << 16).view(np.float32)
            bf.add(name)
        out[name] = a
    return out, bf


def random_weights_torch(cfg: ZConfig, seed: int, device):
    """name -> CUDA tensor (torch.bfloat16 for bf16-stored names, else float32),
    generated on the device (6B parameters in seconds)."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = {}
    for name, shape, kind, is_bf16 in weight_specs(cfg):
        mu, sd = _scale(kind)
        t = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(sd).add_(mu)
        out[name] = t.to(torch.bfloat16) if is_bf16 else t
    return out


class ZImageB200:
    """The Z-Image transformer on the device (ZImageTransformer, zimage.h:56)."""

    def __init__(self, weights, cfg: ZConfig = Z_IMAGE, bf16_names=None, device="cuda"):
        import torch

        from . import backend

        backend.bind_stream()
        self.cfg = cfg
        self._bufs = {}
        L = lib()
        self._m = L.sdb200_zimage_create(cfg.heads, cfg.patch, cfg.norm_eps, cfg.rope_theta, cfg.t_scale, *cfg.axes)
        if not self._m:
            raise RuntimeError(L.sdb200_last_error().decode())
        for name, arr in weights.items():
            if isinstance(arr, np.ndarray):
                if bf16_names is not None and name in bf16_names:
                    t = torch.from_numpy(f32_to_bf16_bits(arr).view(np.int16)).to(device).view(torch.bfloat16)
                else:
                    t = torch.from_numpy(np.ascontiguousarray(arr, np.float32)).to(device)
            else:
                t = arr.contiguous()
            is_bf16 = t.dtype == torch.bfloat16
            shape = (C.c_int64 * t.dim())(*t.shape)
            self._bufs[name] = t
            check(L.sdb200_zimage_set_weight(self._m, name.encode(), t.data_ptr(), int(is_bf16), shape, t.dim()))
        check(L.sdb200_zimage_finalize(self._m))

    @classmethod
    def from_checkpoint(cls, dir_: str, base: str = "diffusion_pytorch_model", cfg: ZConfig = Z_IMAGE, rank: int = 0,
                        world: int = 1, bf16_min_numel: int = 0):
        """A model over the checkpoint <dir>/<base> (.safetensors, sharded .index.json or
        .fp16), read by the library as the reference reads it (sdb200_zimage_load); with
        world > 1 only rank's tensor-parallel shard is read (then call set_tp)."""
        from . import backend

        backend.bind_stream()
        self = cls.__new__(cls)
        self.cfg = cfg
        self._bufs = {}
        L = lib()
        self._m = L.sdb200_zimage_create(cfg.heads, cfg.patch, cfg.norm_eps, cfg.rope_theta, cfg.t_scale, *cfg.axes)
        if not self._m:
            raise RuntimeError(L.sdb200_last_error().decode())
        check(L.sdb200_zimage_load(self._m, dir_.encode(), base.encode(), int(rank), int(world), int(bf16_min_numel)))
        check(L.sdb200_zimage_finalize(self._m))
        return self

    def get_weight(self, name: str):
        """The registered weight `name` copied back to the host: numpy uint16 (BF16 bits)
        or float32 (sdb200_zimage_get_weight)."""
        from . import _read_tensor

        return _read_tensor(lambda d, nb, s, n, b: lib().sdb200_zimage_get_weight(self._m, name.encode(), d, nb, s,
                                                                                   n, b))

    def forward(self, x, t: float, cap, out=None):
        """x [B, C, H, W], cap [B, L, cap_dim] (CUDA fp32) -> [B, C, H, W]."""
        import torch

        B, Cc, H, W = x.shape
        out = torch.empty_like(x) if out is None else out
        check(lib().sdb200_zimage_forward(self._m, x.data_ptr(), B, Cc, H, W, float(t), cap.data_ptr(), cap.shape[1],
                                          cap.shape[2], out.data_ptr()))
        return out

    def sample(self, x, cap, steps: int = 8, shift: float = 3.0, cap_neg=None, cfg: float = 0.0):
        """The pipeline's flow-matching Euler sampler (pipeline.cpp:229-244) with every step
        on the device: returns the denoised latent for the noise x [B, C, H, W] and the
        text states cap (cap_neg and cfg > 0 add classifier-free guidance)."""
        B, Cc, H, W = x.shape
        y = x.clone()
        check(lib().sdb200_zimage_sample(self._m, y.data_ptr(), B, Cc, H, W, cap.data_ptr(),
                                         cap_neg.data_ptr() if cap_neg is not None else None, cap.shape[1],
                                         cap.shape[2], float(cfg), int(steps), float(shift)))
        return y

    def profile(self, enable: bool = True):
        """Times later forwards' GEMM and attention kernels with CUDA events."""
        check(lib().sdb200_zimage_profile(self._m, int(enable)))

    def profile_read(self) -> dict:
        """Kernel times since the last read (ms), algorithmic FLOP or bytes, launches."""
        out = (C.c_double * 16)()
        check(lib().sdb200_zimage_profile_read_ex(self._m, out, 16))
        keys = ("gemm_ms", "gemm_flop", "gemm_launches", "attn_ms", "attn_flop", "attn_launches", "forward_ms",
                "forwards", "allreduce_ms", "allreduces", "post_norm_ms", "post_norm_bytes", "post_norm_launches",
                "adaln_ms", "adaln_bytes", "adaln_launches")
        return dict(zip(keys, list(out)))

    def set_tp(self, comm, mode: int = 1):
        """Attaches a tensor-parallel communicator (sdb200.tp.Comm); the registered weights
        must be this rank's shards (sdb200.tp.shard_weights). mode 1 combines the
        row-parallel outputs inside the kernels over NVLink, mode 0 with an NCCL
        all-reduce (sdb200_zimage_set_tp_mode)."""
        self._comm = comm
        check(lib().sdb200_zimage_set_tp(self._m, comm.handle if comm is not None else None))
        check(lib().sdb200_zimage_set_tp_mode(self._m, int(mode)))

    def __del__(self):
        try:
            if self._m:
                lib().sdb200_zimage_destroy(self._m)
                self._m = None
        except Exception:
            pass
