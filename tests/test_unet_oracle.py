"""Host-side check of the miniature UNet weight layout (no GPU): the reference's own UNet
(unet.cpp:18-56, compiled from its sources) binds the generated names, pairs every up-path
resnet with a skip of the right width, and predicts a latent of the input's shape."""
import numpy as np
import pytest

from sdb200.unet import unet_specs, unet_weights


@pytest.mark.parametrize("cfg,heads", [
    (dict(channels=(64, 128), layers=1, in_ch=4, ctx_dim=96, attn=(True, False)), 2),
    (dict(channels=(64, 128, 128), layers=2, in_ch=4, ctx_dim=32, attn=(True, True, False)), 4),
])
def test_reference_unet_binds_generated_weights(ref, cfg, heads):
    m = ref.unet(unet_weights(seed=0, **cfg), heads=heads)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 4, 16, 16)).astype(np.float32)
    ctx = rng.standard_normal((2, 7, cfg["ctx_dim"])).astype(np.float32)
    y = m(x, 250.0, ctx)
    assert y.shape == x.shape and np.isfinite(y).all()


def test_skip_widths_balance():
    names = {n for n, _ in unet_specs(channels=(320, 640, 1280, 1280), layers=2, ctx_dim=768,
                                      attn=(True, True, True, False))}
    # SD 1.5 layout: 4 down blocks of 2 resnets, 3 downsamplers, 4 up blocks of 3 resnets
    assert "down_blocks.3.resnets.1.conv2.weight" in names
    assert "down_blocks.3.downsamplers.0.conv.weight" not in names
    assert "up_blocks.3.resnets.2.conv2.weight" in names
    assert "up_blocks.0.attentions.0.norm.weight" not in names
    assert "up_blocks.1.attentions.2.transformer_blocks.0.attn2.to_k.weight" in names
