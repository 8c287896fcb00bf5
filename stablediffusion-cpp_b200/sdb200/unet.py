"""Random-init weights for an SD 1.x UNet under the diffusers UNet2DConditionModel names
that the reference binds (src/unet.cpp:18-56, src/modules.cpp:11-31, :86-131): conv_in, a
time MLP, down blocks of (resnet [+ transformer]) with downsamplers, a mid block, up
blocks of (layers + 1) resnets over concatenated skips with upsamplers, conv_out. No
checkpoint exists here, so the UNet tests and benchmarks run on these.

Convolution and linear weights ~N(0, 1/fan_in) so activations keep their scale, biases
~N(0, 0.02), norm gammas ~N(1, 0.1) and betas ~N(0, 0.1). `SD15` holds the SD 1.5 layout
(channels 320 / 640 / 1280 / 1280, 2 layers per block, attention in the first three
stages, text width 768).
"""
import numpy as np

SD15 = dict(channels=(320, 640, 1280, 1280), layers=2, in_ch=4, ctx_dim=768, attn=(True, True, True, False))


def unet_specs(channels=(64, 128), layers=1, in_ch=4, ctx_dim=96, attn=(True, False)):
    s = []

    def conv(p, co, ci, k):
        s.append((p + ".weight", (co, ci, k, k)))
        s.append((p + ".bias", (co,)))

    def lin(p, o, i, bias=True):
        s.append((p + ".weight", (o, i)))
        if bias:
            s.append((p + ".bias", (o,)))

    def norm(p, c):
        s.append((p + ".weight", (c,)))
        s.append((p + ".bias", (c,)))

    temb = 4 * channels[0]

    def resnet(p, ci, co):
        norm(p + ".norm1", ci)
        conv(p + ".conv1", co, ci, 3)
        lin(p + ".time_emb_proj", co, temb)
        norm(p + ".norm2", co)
        conv(p + ".conv2", co, co, 3)
        if ci != co:
            conv(p + ".conv_shortcut", co, ci, 1)

    def transformer(p, c):
        norm(p + ".norm", c)
        lin(p + ".proj_in", c, c)
        b = p + ".transformer_blocks.0"
        for n in ("norm1", "norm2", "norm3"):
            norm(f"{b}.{n}", c)
        for a, kv in (("attn1", c), ("attn2", ctx_dim)):
            lin(f"{b}.{a}.to_q", c, c, bias=False)
            lin(f"{b}.{a}.to_k", c, kv, bias=False)
            lin(f"{b}.{a}.to_v", c, kv, bias=False)
            lin(f"{b}.{a}.to_out.0", c, c)
        lin(f"{b}.ff.net.0.proj", 8 * c, c)
        lin(f"{b}.ff.net.2", c, 4 * c)
        lin(p + ".proj_out", c, c)

    conv("conv_in", channels[0], in_ch, 3)
    lin("time_embedding.linear_1", temb, channels[0])
    lin("time_embedding.linear_2", temb, temb)
    ch = channels[0]
    skips = [ch]
    for i, c in enumerate(channels):
        for j in range(layers):
            resnet(f"down_blocks.{i}.resnets.{j}", ch, c)
            ch = c
            if attn[i]:
                transformer(f"down_blocks.{i}.attentions.{j}", c)
            skips.append(c)
        if i + 1 < len(channels):
            conv(f"down_blocks.{i}.downsamplers.0.conv", c, c, 3)
            skips.append(c)
    resnet("mid_block.resnets.0", ch, ch)
    transformer("mid_block.attentions.0", ch)
    resnet("mid_block.resnets.1", ch, ch)
    for i, c in enumerate(reversed(channels)):
        for j in range(layers + 1):
            sk = skips.pop()
            resnet(f"up_blocks.{i}.resnets.{j}", ch + sk, c)
            ch = c
            if attn[len(channels) - 1 - i]:
                transformer(f"up_blocks.{i}.attentions.{j}", c)
        if i + 1 < len(channels):
            conv(f"up_blocks.{i}.upsamplers.0.conv", c, c, 3)
    norm("conv_norm_out", channels[0])
    conv("conv_out", in_ch, channels[0], 3)
    return s


def unet_weights(seed=0, device=None, **cfg):
    """name -> fp32 numpy array. With device (a torch CUDA device) the numbers are drawn
    there (a full-size UNet's 860 M parameters in a second) and copied to the host."""
    if device is not None:
        import torch

        g = torch.Generator(device=device)
        g.manual_seed(seed)
        out = {}
        for name, shape in unet_specs(**cfg):
            leaf = name.rsplit(".", 1)[0]
            t = torch.randn(shape, generator=g, device=device)
            if name.endswith(".weight") and len(shape) >= 2:
                t *= 1.0 / float(np.sqrt(np.prod(shape[1:])))
            elif name.endswith(".bias"):
                t *= 0.1 if "norm" in leaf.rsplit(".", 1)[-1] else 0.02
            else:
                t = 1.0 + 0.1 * t
            out[name] = t.cpu().numpy()
        return out
    rng = np.random.default_rng(seed)
    out = {}
    for name, shape in unet_specs(**cfg):
        leaf = name.rsplit(".", 1)[0]
        a = rng.standard_normal(shape, dtype=np.float32)
        if name.endswith(".weight") and len(shape) >= 2:
            a *= np.float32(1.0 / np.sqrt(np.prod(shape[1:])))
        elif name.endswith(".bias"):
            a *= np.float32(0.1 if "norm" in leaf.rsplit(".", 1)[-1] else 0.02)
        else:  # norm gamma
            a = np.float32(1.0) + np.float32(0.1) * a
        out[name] = a
    return out
