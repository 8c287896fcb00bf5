"""The VAE decoder on the device (sdb200_vae_*) against the reference's own
VAEDecoder::decode (vae.cpp:35-51) compiled from its sources (oracle/_ref), on the same
random-init weights and latents.

Gate: relative Frobenius error <= 1e-2 on the decoded image, the final-output gate. Every
convolution runs on tf32 tensor cores (about 3e-4 each) and the attention on tf32 GEMMs.
"""
import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL_IMAGE = 1e-2


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


CONFIGS = {
    # SD 1.x layout in miniature: 4 latent channels, post-quant 1x1 conv, scaling 0.18215
    "sd": dict(latent_channels=4, block_out_channels=(32, 64), layers_per_block=1, post_quant_conv=True,
               scaling_factor=0.18215, shift_factor=0.0),
    # FLUX / Z-Image layout: 16 latent channels with a shift, three up stages, 3 resnets each
    "flux": dict(latent_channels=16, block_out_channels=(32, 64, 64), layers_per_block=2, post_quant_conv=False,
                 scaling_factor=0.3611, shift_factor=0.1159),
    # the real widths of the last two stages (128 / 256 channels) at a small size
    "wide": dict(latent_channels=16, block_out_channels=(128, 256), layers_per_block=1, post_quant_conv=False,
                 scaling_factor=0.3611, shift_factor=0.1159),
}


@pytest.mark.parametrize("name,N,h,w", [("sd", 2, 8, 8), ("flux", 1, 12, 10), ("wide", 1, 16, 16)])
def test_vae_decode_vs_reference(sdb, ref, name, N, h, w):
    from sdb200.vae import VAE, VConfig, random_weights

    cfg = VConfig(**CONFIGS[name])
    weights = random_weights(cfg, seed=3)
    z = np.random.default_rng(4).standard_normal((N, cfg.latent_channels, h, w)).astype(np.float32)
    want = ref.vae(weights, cfg.scaling_factor, cfg.shift_factor)(z)
    v = VAE(cfg, weights)
    got = _np(v.decode(_t(z)))
    assert got.shape == want.shape
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= TOL_IMAGE, name
    assert sdb.backend.device_error_word() == 0


def test_vae_load_checkpoint(sdb, tmp_path):
    """sdb200_vae_load on a two-file checkpoint (index.json) decodes bit-identically to
    the same weights registered one by one."""
    from safetensors_writer import write_checkpoint
    from sdb200.vae import VAE, VConfig, random_weights

    cfg = VConfig(**CONFIGS["sd"])
    weights = random_weights(cfg, seed=5)
    write_checkpoint(str(tmp_path), "diffusion_pytorch_model", {n: ("F32", a) for n, a in weights.items()}, shards=2)
    loaded = VAE.from_checkpoint(cfg, str(tmp_path))
    same = VAE(cfg, weights)
    z = _t(np.random.default_rng(6).standard_normal((1, 4, 8, 8)).astype(np.float32))
    assert np.array_equal(_np(loaded.decode(z)), _np(same.decode(z)))


def test_vae_rejects_wrong_latent_channels(sdb):
    from sdb200 import SdbError
    from sdb200.vae import VAE, VConfig, random_weights

    cfg = VConfig(**CONFIGS["sd"])
    v = VAE(cfg, random_weights(cfg, seed=1))
    import torch

    with pytest.raises(SdbError):
        v.decode(torch.zeros((1, 16, 8, 8), device="cuda"))
