"""GPU: the DiT block's post-norm step through sdb200_dit_post_norm (the kernel the device
program runs after every row-parallel projection) against a numpy restatement of the
reference's sequence (zimage.cpp:122-126 / :131-135, then the next block's rms_norm and
modulation, :113-115): x += gate * rms_norm(sum of the partial rows) * gamma2, then
h = bf16(rms_norm(x) * gamma_next * scale_next) into every destination.

The multi-rank forms (several partial slots, h stored into several buffers, four rows per
block under one system-scope fence) otherwise run only in the 2-GPU tensor-parallel test;
here the "peer" destinations are buffers on the same device."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


def _bf16_to_f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _reference(partials, world, slot_rows, rows, x, row0, gamma2, gate, gamma_n, scale_n, eps):
    a = partials[0:rows].astype(np.float32).copy()
    for s in range(1, world):
        a = a + partials[s * slot_rows:s * slot_rows + rows]
    rstd = (1.0 / np.sqrt(np.mean(a.astype(np.float64) ** 2, axis=1) + eps)).astype(np.float32)
    v = a * rstd[:, None] * (gamma2 if gamma2 is not None else 1.0)
    xn = x[row0:row0 + rows] + (gate * v if gate is not None else v)
    rstd2 = (1.0 / np.sqrt(np.mean(xn.astype(np.float64) ** 2, axis=1) + eps)).astype(np.float32)
    h = xn * rstd2[:, None] * (gamma_n if gamma_n is not None else 1.0)
    if scale_n is not None:
        h = h * scale_n
    return xn.astype(np.float32), h.astype(np.float32)


@pytest.mark.parametrize("world,n_dst,D,affine", [
    (2, 2, 3840, True),    # two ranks' partial slots, h to both: four rows per block, one fence
    (1, 1, 3840, True),    # one rank
    (3, 0, 3840, True),    # no next block: x only
    (4, 4, 1000, False),   # narrow rows, no gammas / gate / scale
    (2, 2, 1002, True),    # D % 4 != 0: the shared-memory form
])
def test_dit_post_norm_vs_reference(sdb, world, n_dst, D, affine):
    import torch

    L = sdb.lib()
    rng = np.random.default_rng(world * 10 + n_dst + D)
    rows, slot_rows, row0, xrows = 37, 40, 5, 50
    eps = 1e-6
    partials = rng.standard_normal((world * slot_rows, D)).astype(np.float32)
    x = rng.standard_normal((xrows, D)).astype(np.float32)
    vec = lambda: (1.0 + 0.3 * rng.standard_normal(D)).astype(np.float32)  # noqa: E731
    gamma2, gate, gamma_n, scale_n = (vec(), np.tanh(vec()).astype(np.float32), vec(), vec()) if affine else \
        (None, None, None, None)
    t = lambda a: None if a is None else torch.from_numpy(a).cuda()  # noqa: E731
    pd, xd = t(partials), t(x)
    g2, gt, gn, sn = t(gamma2), t(gate), t(gamma_n), t(scale_n)
    hs = [torch.zeros((xrows, D), dtype=torch.int16, device="cuda") for _ in range(n_dst)]
    hptr = (C.c_void_p * max(1, n_dst))(*[h.data_ptr() for h in hs]) if n_dst else None
    p = lambda a: None if a is None else a.data_ptr()  # noqa: E731
    sdb.backend.bind_stream()
    sdb.check(L.sdb200_dit_post_norm(pd.data_ptr(), slot_rows, world, row0, rows, xd.data_ptr(), D, p(g2), p(gt),
                                     p(gn), p(sn), C.cast(hptr, C.c_void_p) if hptr is not None else None, n_dst,
                                     eps))
    torch.cuda.synchronize()
    want_x, want_h = _reference(partials, world, slot_rows, rows, x, row0, gamma2, gate, gamma_n, scale_n, eps)
    got_x = xd.cpu().numpy()
    assert rel_fro(got_x[row0:row0 + rows], want_x) <= 1e-5
    assert np.array_equal(got_x[:row0], x[:row0]) and np.array_equal(got_x[row0 + rows:], x[row0 + rows:])
    for h in hs:
        hb = h.cpu().numpy().view(np.uint16)
        assert np.array_equal(hb, hs[0].cpu().numpy().view(np.uint16))
        assert rel_fro(_bf16_to_f32(hb[row0:row0 + rows]), want_h) <= 4e-3
        assert not hb[:row0].any() and not hb[row0 + rows:].any()
    assert sdb.backend.device_error_word() == 0
