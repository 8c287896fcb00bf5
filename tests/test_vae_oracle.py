"""Host-side checks of the VAE weight layout (no GPU): the reference's own VAEDecoder
(vae.cpp:15-32, compiled from its sources) binds the generated names for every test
configuration and decodes to the expected shape."""
import numpy as np
import pytest

from sdb200.vae import FLUX_VAE, VConfig, decode_flops, random_weights, weight_specs


@pytest.mark.parametrize("cfg,N,h,w,up", [
    (VConfig(latent_channels=4, block_out_channels=(32, 64), layers_per_block=1, post_quant_conv=True,
             scaling_factor=0.18215, shift_factor=0.0), 2, 4, 6, 2),
    (VConfig(latent_channels=16, block_out_channels=(32, 64, 64), layers_per_block=2), 1, 5, 4, 4),
])
def test_reference_binds_generated_weights(ref, cfg, N, h, w, up):
    m = ref.vae(random_weights(cfg, 0), cfg.scaling_factor, cfg.shift_factor)
    z = np.random.default_rng(1).standard_normal((N, cfg.latent_channels, h, w)).astype(np.float32)
    y = m(z)
    assert y.shape == (N, 3, h * up, w * up)
    assert np.isfinite(y).all()


def test_flux_vae_layout():
    names = {n for n, _, _ in weight_specs(FLUX_VAE)}
    # 4 up blocks of 3 resnets, upsamplers on the first three, shortcuts where widths change
    assert "decoder.up_blocks.3.resnets.2.conv2.weight" in names
    assert "decoder.up_blocks.2.upsamplers.0.conv.weight" in names
    assert "decoder.up_blocks.3.upsamplers.0.conv.weight" not in names
    assert "decoder.up_blocks.2.resnets.0.conv_shortcut.weight" in names     # 512 -> 256
    assert "decoder.up_blocks.1.resnets.0.conv_shortcut.weight" not in names  # 512 -> 512
    assert "post_quant_conv.weight" not in names
    # about 10.5 TFLOP for a 1024^2 decode, 3x3 convolutions dominating
    assert 10.0e12 < decode_flops(FLUX_VAE, 128, 128) < 11.0e12
