"""CPU: pins the Z-Image restatement (oracle/zimage_oracle.py) against the reference's
own ZImageTransformer: the committed golden output, and the compiled reference."""
import numpy as np

from conftest import load_golden, rel_fro

SMALL = dict(dim=256, heads=2, ffn=512, t_dim=256, t_hidden=512, cap_dim=128, layers=2, noise_refiners=1,
             context_refiners=1)


def _small():
    from sdb200.zimage import ZConfig, random_weights_numpy

    cfg = ZConfig(**SMALL)
    w, bf = random_weights_numpy(cfg, 0)
    return cfg, w, bf


def test_zimage_oracle_vs_golden(orc):
    from zimage_oracle import ZImageOracle

    cfg, w, bf = _small()
    g = load_golden("zimage_small")
    out = ZImageOracle(orc, w, bf, heads=cfg.heads).forward(g["x"], float(g["t"]), g["cap"])
    assert np.isfinite(out).all()
    assert rel_fro(out, g["out"]) <= 1e-5


def test_zimage_oracle_vs_reference_library(orc, ref):
    from sdb200.zimage import ZConfig, random_weights_numpy
    from zimage_oracle import ZImageOracle

    cfg = ZConfig(dim=256, heads=2, ffn=256, t_dim=256, t_hidden=256, cap_dim=64, layers=1, noise_refiners=2,
                  context_refiners=0)
    w, bf = random_weights_numpy(cfg, 3)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 16, 10, 14)).astype(np.float32)  # 35 image tokens -> padded to 64
    cap = rng.standard_normal((1, 7, 64)).astype(np.float32)
    a = ZImageOracle(orc, w, bf, heads=2).forward(x, 0.25, cap)
    b = ref.zimage(w, bf, heads=2)(x, 0.25, cap)
    assert rel_fro(a, b) <= 1e-5
