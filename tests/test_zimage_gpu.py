"""GPU parity of the device Z-Image transformer (sdb200_zimage_*) against the reference.

Gate (north star): relative Frobenius error <= 1e-2 on the final DiT output latent
against the reference CPU forward on the same seeded weights and inputs. The device
path rounds every GEMM's activation operand to bf16 (as the reference GPU backend does)
and runs attention on fp16 operands; the CPU reference keeps fp32 activations.
"""
import numpy as np
import pytest

from conftest import load_golden, rel_fro

pytestmark = pytest.mark.gpu

TOL_LATENT = 1e-2


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _np(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


def _model(cfg, seed):
    from sdb200.zimage import ZImageB200, random_weights_numpy

    w, bf = random_weights_numpy(cfg, seed)
    return w, bf, ZImageB200(w, cfg, bf16_names=bf)


def test_zimage_small_vs_golden_and_oracle(sdb, orc):
    from sdb200.zimage import ZConfig
    from zimage_oracle import ZImageOracle

    cfg = ZConfig(dim=256, heads=2, ffn=512, t_dim=256, t_hidden=512, cap_dim=128, layers=2, noise_refiners=1,
                  context_refiners=1)
    w, bf, m = _model(cfg, 0)
    g = load_golden("zimage_small")
    got = _np(m.forward(_t(g["x"]), float(g["t"]), _t(g["cap"])))
    assert np.isfinite(got).all()
    assert rel_fro(got, g["out"]) <= TOL_LATENT
    want = ZImageOracle(orc, w, bf, heads=cfg.heads).forward(g["x"], float(g["t"]), g["cap"])
    assert rel_fro(got, want) <= TOL_LATENT


def test_zimage_batch_equals_single(sdb):
    """B images in one forward give exactly the per-image results (rows of the batched
    GEMMs and attention samples are independent)."""
    import torch

    from sdb200.zimage import ZConfig

    cfg = ZConfig(dim=256, heads=2, ffn=512, t_dim=256, t_hidden=512, cap_dim=128, layers=2, noise_refiners=1,
                  context_refiners=1)
    _, _, m = _model(cfg, 5)
    rng = np.random.default_rng(6)
    x = _t(rng.standard_normal((3, 16, 12, 20)).astype(np.float32))
    cap = _t(rng.standard_normal((3, 9, 128)).astype(np.float32))
    yb = m.forward(x, 0.4, cap)
    ys = torch.cat([m.forward(x[i:i + 1].contiguous(), 0.4, cap[i:i + 1].contiguous()) for i in range(3)])
    assert torch.equal(yb, ys)


def test_zimage_full_width_block(sdb, orc):
    """One full-width Z-Image block (dim 3840, 30 heads, FFN 10240, adaLN from a 256-d
    embedding) inside the forward, at a reduced sequence (256 image + 32 text tokens)."""
    from sdb200.zimage import ZConfig
    from zimage_oracle import ZImageOracle

    cfg = ZConfig(layers=1, noise_refiners=0, context_refiners=0)
    w, bf, m = _model(cfg, 7)
    rng = np.random.default_rng(8)
    x = rng.standard_normal((1, 16, 32, 32)).astype(np.float32)
    cap = rng.standard_normal((1, 32, 2560)).astype(np.float32)
    got = _np(m.forward(_t(x), 0.7, _t(cap)))
    want = ZImageOracle(orc, w, bf, heads=30).forward(x, 0.7, cap)
    assert rel_fro(got, want) <= TOL_LATENT


def test_zimage_cfg3_block_1024(sdb, ref):
    """one single-stream block at 1024^2 (4096 image + 128 text tokens,
    hidden 3840, 30 heads, SwiGLU 10240, adaLN), random-init bf16 weights, against the
    reference CPU forward compiled from its sources."""
    from sdb200.zimage import ZConfig

    cfg = ZConfig(layers=1, noise_refiners=0, context_refiners=0)
    w, bf, m = _model(cfg, 9)
    rng = np.random.default_rng(10)
    x = rng.standard_normal((1, 16, 128, 128)).astype(np.float32)
    cap = rng.standard_normal((1, 128, 2560)).astype(np.float32)
    got = _np(m.forward(_t(x), 0.5, _t(cap)))
    want = ref.zimage(w, bf, heads=30)(x, 0.5, cap)
    assert rel_fro(got, want) <= TOL_LATENT


def test_zimage_cfg5_block_2048(sdb, ref):
    """BASELINE config 5's sequence on one GPU: one full-width single-stream block at 2048^2
    (16384 image + 128 text tokens = 16512), random-init bf16 weights, against the
    reference CPU forward compiled from its sources (zimage.cpp:90-136 at S = 16512)."""
    from sdb200.zimage import ZConfig

    cfg = ZConfig(layers=1, noise_refiners=0, context_refiners=0)
    w, bf, m = _model(cfg, 21)
    rng = np.random.default_rng(22)
    x = rng.standard_normal((1, 16, 256, 256)).astype(np.float32)
    cap = rng.standard_normal((1, 128, 2560)).astype(np.float32)
    got = _np(m.forward(_t(x), 0.35, _t(cap)))
    want = ref.zimage(w, bf, heads=30)(x, 0.35, cap)
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= TOL_LATENT


class _HostFloat32(dict):
    """name -> torch CUDA tensor, handed out one tensor at a time as a float32 numpy array
    (the reference model keeps its own bf16 copy; 6 B parameters never sit in fp32 on the
    host at once)."""

    def items(self):
        for n, t in super().items():
            yield n, t.float().cpu().numpy()


def test_dit_full_model_vs_reference_cpu(sdb, ref):
    """BASELINE config 4's model at full size (30 layers + 2 + 2 refiners, 6.15 B
    parameters) for one image at 1024^2 (4224 tokens), against the reference's CPU
    ZImageTransformer::forward (zimage.cpp:138-228) over the same weights: the full-depth
    check against the CPU path, whose activations stay fp32 (the device rounds every GEMM
    operand to bf16 and runs attention on fp16)."""
    import torch

    from sdb200.zimage import Z_IMAGE, ZImageB200, random_weights_torch

    wts = random_weights_torch(Z_IMAGE, 5, "cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(2025)
    x = torch.randn((1, 16, 128, 128), generator=g, device="cuda")
    cap = torch.randn((1, 128, Z_IMAGE.cap_dim), generator=g, device="cuda")
    model = ZImageB200(wts, Z_IMAGE)
    got = _np(model.forward(x, 0.6, cap))
    del model
    bf = {n for n, t in wts.items() if t.dtype == torch.bfloat16}
    rm = ref.zimage(_HostFloat32(wts), bf, heads=Z_IMAGE.heads)
    del wts
    torch.cuda.empty_cache()
    want = rm(x.cpu().numpy(), 0.6, cap.cpu().numpy())
    del rm
    assert np.isfinite(got).all()
    assert rel_fro(got, want) <= TOL_LATENT


@pytest.mark.parametrize("cfg_scale", [0.0, 2.0])
def test_zimage_sampler_on_device(sdb, orc, ref, cfg_scale):
    """sdb200_zimage_sample (the pipeline's flow-matching Euler loop run on the device)
    against the same loop on the host over the device forward (identical up to the
    update's rounding), and against the reference's CPU forward + FlowMatchScheduler per
    image at the DiT latent gate."""
    from sdb200.zimage import ZConfig

    cfg = ZConfig(dim=256, heads=2, ffn=512, t_dim=256, t_hidden=512, cap_dim=128, layers=2, noise_refiners=1,
                  context_refiners=1)
    w, bf, m = _model(cfg, 0)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 16, 16, 16)).astype(np.float32)
    cap = rng.standard_normal((2, 20, 128)).astype(np.float32)
    neg = rng.standard_normal((2, 20, 128)).astype(np.float32)
    steps, shift = 3, 3.0
    got = _np(m.sample(_t(x), _t(cap), steps=steps, shift=shift, cap_neg=_t(neg) if cfg_scale else None,
                       cfg=cfg_scale))
    assert np.isfinite(got).all()
    sig = orc.flow_sigmas(steps, shift)
    y = x.copy()
    for i in range(steps):
        o = _np(m.forward(_t(y), 1.0 - sig[i], _t(cap)))
        n = _np(m.forward(_t(y), 1.0 - sig[i], _t(neg))) if cfg_scale else None
        y = orc.flow_step(y, o, n, cfg_scale, sig[i] - sig[i + 1])
    assert rel_fro(got, y) <= 1e-5
    model = ref.zimage(w, bf, heads=cfg.heads)
    for b in range(2):
        yr = x[b:b + 1].copy()
        for i in range(steps):
            o = model(yr, 1.0 - sig[i], cap[b:b + 1])
            n = model(yr, 1.0 - sig[i], neg[b:b + 1]) if cfg_scale else None
            yr = ref.flow_step(yr, o, n, cfg_scale, i, steps, shift)
        assert rel_fro(got[b:b + 1], yr) <= TOL_LATENT


def _as_read(w, bf, min_numel):
    """The weights as the checkpoint reader returns them from a file that holds the bf16
    names as BF16 and the rest as F32: BF16 from min_numel elements up, F32 below."""
    from sdb200.workloads import f32_to_bf16_bits

    out, names = {}, set()
    for n, a in w.items():
        if a.size >= min_numel:
            out[n] = (f32_to_bf16_bits(a).astype(np.uint32) << 16).view(np.float32)
            names.add(n)
        else:
            out[n] = a
    return out, names


def test_zimage_load_checkpoint(sdb, ref, tmp_path):
    """sdb200_zimage_load on a two-file checkpoint (index.json) against the same weights
    registered one by one (bit-identical output), and against the reference loading the
    same directory with its own reader (latent gate)."""
    from safetensors_writer import write_checkpoint
    from sdb200.workloads import f32_to_bf16_bits
    from sdb200.zimage import ZConfig, ZImageB200, random_weights_numpy

    cfg = ZConfig(dim=256, heads=2, ffn=512, t_dim=256, t_hidden=512, cap_dim=128, layers=2, noise_refiners=1,
                  context_refiners=1)
    w, bf = random_weights_numpy(cfg, 0)
    tensors = {n: ("BF16", f32_to_bf16_bits(a)) if n in bf else ("F32", a) for n, a in w.items()}
    base = "diffusion_pytorch_model"
    write_checkpoint(str(tmp_path), base, tensors, shards=2)
    mn = 32768  # every block matrix is at least this large
    loaded = ZImageB200.from_checkpoint(str(tmp_path), base, cfg, bf16_min_numel=mn)
    w2, bf2 = _as_read(w, bf, mn)
    same = ZImageB200(w2, cfg, bf16_names=bf2)
    rng = np.random.default_rng(9)
    x = rng.standard_normal((2, 16, 16, 16)).astype(np.float32)
    cap = rng.standard_normal((2, 20, 128)).astype(np.float32)
    got = _np(loaded.forward(_t(x), 0.4, _t(cap)))
    assert np.array_equal(got, _np(same.forward(_t(x), 0.4, _t(cap))))
    rm = ref.zimage_load(str(tmp_path), base, heads=cfg.heads)
    for b in range(2):
        assert rel_fro(got[b:b + 1], rm(x[b:b + 1], 0.4, cap[b:b + 1])) <= TOL_LATENT
