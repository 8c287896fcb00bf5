"""AutoencoderKL decoder on libsdb200 (sdb200_vae_* C ABI) plus random-init weights under
the checkpoint names the reference binds (src/vae.cpp:15-32, src/modules.cpp:27-31,
:119-131; the diffusers AutoencoderKL decoder layout).

No checkpoint exists here, so weights are random (seeded): convolution and linear weights
~N(0, 1/fan_in) so activations keep their scale through the residual stack, biases
~N(0, 0.02), GroupNorm gammas ~N(1, 0.1) and betas ~N(0, 0.1). `FLUX_VAE` holds the
published Z-Image / FLUX VAE's hyper-parameters (16 latent channels, block widths
128/256/512/512, 2 layers per block, scaling 0.3611, shift 0.1159, no post-quant conv).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import check, lib


@dataclass(frozen=True)
class VConfig:
    latent_channels: int = 16
    block_out_channels: tuple = (128, 256, 512, 512)
    layers_per_block: int = 2
    out_channels: int = 3
    post_quant_conv: bool = False
    scaling_factor: float = 0.3611
    shift_factor: float = 0.1159


FLUX_VAE = VConfig()


def weight_specs(cfg: VConfig):
    """[(name, shape, kind)] with kind in {"conv", "lin", "b", "g", "beta"}."""
    s = []

    def conv(p, co, ci, k):
        s.append((p + ".weight", (co, ci, k, k), "conv"))
        s.append((p + ".bias", (co,), "b"))

    def norm(p, c):
        s.append((p + ".weight", (c,), "g"))
        s.append((p + ".bias", (c,), "beta"))

    def resnet(p, ci, co):
        norm(p + ".norm1", ci)
        conv(p + ".conv1", co, ci, 3)
        norm(p + ".norm2", co)
        conv(p + ".conv2", co, co, 3)
        if ci != co:
            conv(p + ".conv_shortcut", co, ci, 1)

    L = cfg.latent_channels
    chans = list(reversed(cfg.block_out_channels))
    top = chans[0]
    if cfg.post_quant_conv:
        conv("post_quant_conv", L, L, 1)
    conv("decoder.conv_in", top, L, 3)
    resnet("decoder.mid_block.resnets.0", top, top)
    a = "decoder.mid_block.attentions.0"
    norm(a + ".group_norm", top)
    for n in ("to_q", "to_k", "to_v", "to_out.0"):
        s.append((f"{a}.{n}.weight", (top, top), "lin"))
        s.append((f"{a}.{n}.bias", (top,), "b"))
    resnet("decoder.mid_block.resnets.1", top, top)
    prev = top
    for i, ch in enumerate(chans):
        for j in range(cfg.layers_per_block + 1):
            resnet(f"decoder.up_blocks.{i}.resnets.{j}", prev if j == 0 else ch, ch)
        if i + 1 < len(chans):
            conv(f"decoder.up_blocks.{i}.upsamplers.0.conv", ch, ch, 3)
        prev = ch
    norm("decoder.conv_norm_out", chans[-1])
    conv("decoder.conv_out", cfg.out_channels, chans[-1], 3)
    return s


def random_weights(cfg: VConfig, seed: int = 0) -> dict:
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape, kind in weight_specs(cfg):
        if kind in ("conv", "lin"):
            fan_in = int(np.prod(shape[1:]))
            a = rng.standard_normal(shape) / np.sqrt(fan_in)
        elif kind == "b":
            a = 0.02 * rng.standard_normal(shape)
        elif kind == "g":
            a = 1.0 + 0.1 * rng.standard_normal(shape)
        else:
            a = 0.1 * rng.standard_normal(shape)
        out[name] = a.astype(np.float32)
    return out


def decode_flops(cfg: VConfig, h: int, w: int, n: int = 1) -> float:
    """Algorithmic FLOPs of one decode: 2*Cout*Cin*k*k*H*W per convolution, 2*S*C*C per
    attention projection, 4*S^2*C for the attention itself."""
    f = 0.0
    H, W = h, w
    L = cfg.latent_channels
    chans = list(reversed(cfg.block_out_channels))
    top = chans[0]

    def conv(co, ci, k, H, W):
        return 2.0 * co * ci * k * k * H * W

    def resnet(ci, co, H, W):
        x = conv(co, ci, 3, H, W) + conv(co, co, 3, H, W)
        return x + (conv(co, ci, 1, H, W) if ci != co else 0.0)

    if cfg.post_quant_conv:
        f += conv(L, L, 1, H, W)
    f += conv(top, L, 3, H, W)
    f += 2 * resnet(top, top, H, W)
    S = H * W
    f += 4 * 2.0 * S * top * top + 4.0 * S * S * top
    prev = top
    for i, ch in enumerate(chans):
        for j in range(cfg.layers_per_block + 1):
            f += resnet(prev if j == 0 else ch, ch, H, W)
        if i + 1 < len(chans):
            H, W = 2 * H, 2 * W
            f += conv(ch, ch, 3, H, W)
        prev = ch
    f += conv(cfg.out_channels, chans[-1], 3, H, W)
    return n * f


class VAE:
    """Device decoder. `weights` maps names to numpy fp32 arrays (uploaded and kept alive
    here), or use from_checkpoint()."""

    def __init__(self, cfg: VConfig, weights: dict | None = None, device="cuda"):
        import torch

        self.cfg = cfg
        self._lib = lib()
        self.h = self._lib.sdb200_vae_create(cfg.scaling_factor, cfg.shift_factor)
        if not self.h:
            raise RuntimeError(self._lib.sdb200_last_error().decode())
        self._keep = []
        if weights is not None:
            for name, a in weights.items():
                t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)
                self._keep.append(t)
                shp = (C.c_int64 * a.ndim)(*a.shape)
                check(self._lib.sdb200_vae_set_weight(self.h, name.encode(), t.data_ptr(), shp, a.ndim))
            self.finalize()

    @classmethod
    def from_checkpoint(cls, cfg: VConfig, directory: str, base: str = "diffusion_pytorch_model"):
        v = cls(cfg)
        check(v._lib.sdb200_vae_load(v.h, directory.encode(), base.encode()))
        v.finalize()
        return v

    def finalize(self):
        check(self._lib.sdb200_vae_finalize(self.h))
        lc, oc, up = C.c_int64(), C.c_int64(), C.c_int64()
        check(self._lib.sdb200_vae_info(self.h, C.byref(lc), C.byref(oc), C.byref(up)))
        self.latent_channels, self.out_channels, self.upscale = lc.value, oc.value, up.value

    def decode(self, z, out=None):
        """z: torch fp32 CUDA tensor [N, C, h, w] -> [N, 3, h * up, w * up]."""
        import torch

        from .backend import bind_stream

        N, Cc, h, w = z.shape
        if out is None:
            out = torch.empty((N, self.out_channels, h * self.upscale, w * self.upscale), device=z.device)
        bind_stream()
        check(self._lib.sdb200_vae_decode(self.h, z.data_ptr(), N, Cc, h, w, out.data_ptr()))
        return out

    def __del__(self):
        try:
            if self.h:
                self._lib.sdb200_vae_destroy(self.h)
                self.h = None
        except Exception:
            pass
