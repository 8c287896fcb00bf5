"""The drop-in boundary exercised end to end: the reference's own model code
(src/unet.cpp, src/zimage.cpp, src/vae.cpp over src/tensor.cpp and src/modules.cpp)
linked against libsdb200.so in place of its backend (oracle/_ref/libsdref_b200.so, the
maintainer's link), running on the GPU, against the same code on its CPU path.

Every sd::cuda call of those models lands in this library. Gate: 1e-2 relative Frobenius
on the model output (the final-output gate). It covers the SD 1.x UNet, whose output the
north-star gate names.
"""
import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL_OUT = 1e-2


@pytest.fixture(scope="module")
def dropin():
    from oracle import RefOnB200

    if not RefOnB200.available():
        pytest.skip("oracle/_ref/libsdref_b200.so not built here")
    return RefOnB200()


@pytest.mark.parametrize("cfg,heads,N,HW,L", [
    # miniature layout: 64 / 128 channels, attention in the first stage, head dims 32 and 64
    (dict(channels=(64, 128), layers=1, in_ch=4, ctx_dim=96, attn=(True, False)), 2, 2, 32, 12),
    # SD 1.5 widths and heads (320 / 640 channels, 8 heads of 40 / 80, text width 768, 77 tokens)
    (dict(channels=(320, 640), layers=1, in_ch=4, ctx_dim=768, attn=(True, True)), 8, 2, 16, 77),
])
def test_unet_on_this_library(sdb, ref, dropin, cfg, heads, N, HW, L):
    from sdb200.unet import unet_weights

    w = unet_weights(seed=1, **cfg)
    rng = np.random.default_rng(2)
    x = rng.standard_normal((N, cfg["in_ch"], HW, HW)).astype(np.float32)
    ctx = rng.standard_normal((N, L, cfg["ctx_dim"])).astype(np.float32)
    want = ref.unet(w, heads=heads)(x, 421.0, ctx)
    got = dropin.unet(w, heads=heads, on_device=True)(x, 421.0, ctx)
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= TOL_OUT
    assert sdb.backend.device_error_word() == 0


def test_zimage_on_this_library(sdb, ref, dropin):
    import torch

    from sdb200.zimage import ZConfig, random_weights_torch

    cfg = ZConfig(dim=512, heads=4, ffn=1024, t_dim=256, t_hidden=512, cap_dim=256, layers=2, noise_refiners=1,
                  context_refiners=1)
    wts = random_weights_torch(cfg, 5, "cuda")
    host = {n: t.float().cpu().numpy() for n, t in wts.items()}
    bf = {n for n, t in wts.items() if t.dtype == torch.bfloat16}
    rng = np.random.default_rng(6)
    x = rng.standard_normal((1, 16, 32, 32)).astype(np.float32)
    cap = rng.standard_normal((1, 40, 256)).astype(np.float32)
    want = ref.zimage(host, bf, heads=cfg.heads)(x, 0.6, cap)
    got = dropin.zimage_cuda(wts, heads=cfg.heads)(x, 0.6, cap)
    assert rel_fro(got, want) <= TOL_OUT


def test_vae_on_this_library(sdb, ref, dropin):
    from sdb200.vae import VConfig, random_weights

    cfg = VConfig(latent_channels=16, block_out_channels=(32, 64, 64), layers_per_block=1)
    w = random_weights(cfg, seed=8)
    z = np.random.default_rng(9).standard_normal((1, 16, 12, 12)).astype(np.float32)
    want = ref.vae(w, cfg.scaling_factor, cfg.shift_factor)(z)
    got = dropin.vae_cuda(w, cfg.scaling_factor, cfg.shift_factor)(z)
    assert rel_fro(got, want) <= TOL_OUT


def test_sd15_unet_step_through_both_backends(sdb, dropin, capsys):
    """BASELINE config 2 in full: the reference's own UNet (SD 1.5 widths 320/640/1280/1280, 2
    layers per block, 8 heads, 77 x 768 text states) at 512^2 with a batch of 2, as its CFG
    pipeline runs it, once through its own GPU backend (backend_cuda.cu + cuBLAS) and once
    through this library (the drop-in link), same weights and inputs. The outputs agree at
    the output gate; the step times are printed (-s) as the relink speed-up."""
    import time

    from oracle import RefCUDA
    from sdb200.unet import unet_weights

    if not RefCUDA.available():
        pytest.skip("oracle/_ref/libsdref_cuda.so not built here")
    cfg = dict(channels=(320, 640, 1280, 1280), layers=2, in_ch=4, ctx_dim=768, attn=(True, True, True, False))
    w = unet_weights(seed=3, device="cuda", **cfg)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 4, 64, 64)).astype(np.float32)
    ctx = rng.standard_normal((2, 77, 768)).astype(np.float32)
    times, outs = {}, {}
    for name, lib in (("reference backend", RefCUDA()), ("this library", dropin)):
        m = lib.unet(w, heads=8, on_device=True)
        m(x, 500.0, ctx)  # warm-up: allocator caches, cuBLAS / tensor maps
        t0 = time.perf_counter()
        for _ in range(3):
            outs[name] = m(x, 500.0, ctx)
        times[name] = (time.perf_counter() - t0) / 3 * 1e3
        del m
    err = rel_fro(outs["this library"], outs["reference backend"])
    with capsys.disabled():
        print(f"\nSD 1.5 UNet step @512^2, batch 2 (ms, wall clock incl. latent in / out): "
              f"reference backend {times['reference backend']:.1f}, this library {times['this library']:.1f}, "
              f"outputs agree to {err:.2e}")
    assert err <= TOL_OUT
