"""This library against the reference's own GPU backend (src/backend_cuda.cu + cuBLAS,
built from its sources into oracle/_ref/libsdref_cuda.so) on the same device buffers.

The reference packs A to bf16 with the same rounding and accumulates in fp32, so the bf16
GEMM agrees to within fp32 summation order. Attention and convolution run in fp32 there
(SGEMM) and on fp16 / tf32 tensor cores here: the per-contraction gate applies. The DiT
forward is compared on a small model under the latent gate.
"""
import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def rgpu():
    from oracle import RefCUDA

    if not RefCUDA.available():
        pytest.skip("oracle/_ref/libsdref_cuda.so not built here")
    r = RefCUDA()
    if not r.cuda_available():
        pytest.fail("the reference GPU backend sees no device")
    return r


def _np(t):
    import torch

    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("M,N,K", [(4096, 11520, 3840), (300, 520, 136), (8, 3840, 256)])
def test_gemm_bf16_vs_reference_gpu(sdb, rgpu, M, N, K):
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    rng = np.random.default_rng(M + N)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    Wb = torch.from_numpy(f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32)).view(np.int16)).cuda()
    b = torch.from_numpy((0.01 * rng.standard_normal(N)).astype(np.float32)).cuda()
    ours, ref = torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")
    sdb.check(sdb.lib().sdb200_gemm_nt_bf16(M, N, K, A.data_ptr(), K, Wb.data_ptr(), K, ours.data_ptr(), N,
                                            b.data_ptr(), 0))
    rgpu.gemm_nt_bf16_dev(M, N, K, A.data_ptr(), K, Wb.data_ptr(), K, ref.data_ptr(), N, b.data_ptr())
    # M <= 16 runs the exact-fp32 skinny kernel here (A not rounded to bf16), so it differs
    # from the reference by the reference's own A rounding: the GEMM gate applies there.
    assert rel_fro(_np(ours), _np(ref)) <= (1e-5 if M > 16 else 2e-3)


@pytest.mark.parametrize("N,S,H,KVH,d,causal", [(1, 4224, 30, 30, 128, False), (2, 300, 32, 8, 128, True),
                                                (1, 1024, 1, 1, 512, False)])
def test_attention_vs_reference_gpu(sdb, rgpu, N, S, H, KVH, d, causal):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(S + H)
    q = torch.randn((N, S, H * d), generator=g, device="cuda")
    k = torch.randn((N, S, KVH * d), generator=g, device="cuda")
    v = torch.randn((N, S, KVH * d), generator=g, device="cuda")
    ours = sdb.backend.attention(q, k, v, H, causal=causal, kv_heads=KVH)
    ref = torch.empty_like(q)
    rgpu.attention_dev(q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), N, S, S, H, KVH, d, causal)
    assert rel_fro(_np(ours), _np(ref)) <= 2e-3


@pytest.mark.parametrize("N,Cin,H,W,Cout,k,pad", [(1, 128, 96, 96, 128, 3, 1), (2, 64, 33, 47, 256, 3, 1),
                                                  (1, 256, 40, 40, 128, 1, 0)])
def test_conv2d_vs_reference_gpu(sdb, rgpu, N, Cin, H, W, Cout, k, pad):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(Cin + H)
    x = torch.randn((N, Cin, H, W), generator=g, device="cuda")
    w = 0.05 * torch.randn((Cout, Cin, k, k), generator=g, device="cuda")
    b = 0.05 * torch.randn((Cout,), generator=g, device="cuda")
    Ho, Wo = H + 2 * pad - k + 1, W + 2 * pad - k + 1
    ours = sdb.backend.conv2d(x, w, b, 1, pad)
    ref = torch.empty_like(ours)
    rgpu.conv2d_dev(x.data_ptr(), N, Cin, H, W, w.data_ptr(), Cout, k, k, b.data_ptr(), 1, pad, ref.data_ptr(), Ho,
                    Wo)
    assert rel_fro(_np(ours), _np(ref)) <= 2e-3


def test_dit_forward_vs_reference_gpu(sdb, rgpu):
    """The whole Z-Image forward (small model) against the reference's ZImageTransformer on
    its GPU backend, with the same device weights copied into the reference's storage."""
    import torch

    from sdb200.zimage import ZConfig, ZImageB200, random_weights_torch

    cfg = ZConfig(dim=512, heads=4, ffn=1024, t_dim=256, t_hidden=512, cap_dim=256, layers=2, noise_refiners=1,
                  context_refiners=1)
    wts = random_weights_torch(cfg, 3, "cuda")
    model = ZImageB200(wts, cfg)
    ref = rgpu.zimage_cuda(wts, heads=cfg.heads)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((1, 16, 32, 32)).astype(np.float32)
    cap = rng.standard_normal((1, 40, 256)).astype(np.float32)
    want = ref(x, 0.3, cap)
    got = _np(model.forward(torch.from_numpy(x).cuda(), 0.3, torch.from_numpy(cap).cuda()))
    assert rel_fro(got, want) <= 1e-2


def test_dit_full_model_vs_reference_gpu(sdb, rgpu):
    """BASELINE config 4's model at full size (30 layers + 2 + 2 refiners, 6.15 B parameters)
    at 1024^2 for one image, against the reference's GPU forward over the same weights
    (the CPU forward is the other full-depth check, tests/test_zimage_gpu.py)."""
    import torch

    from sdb200.zimage import Z_IMAGE, ZImageB200, random_weights_torch

    wts = random_weights_torch(Z_IMAGE, 0, "cuda")
    model = ZImageB200(wts, Z_IMAGE)
    g = torch.Generator(device="cuda")
    g.manual_seed(1000)
    x = torch.randn((1, 16, 128, 128), generator=g, device="cuda")
    cap = torch.randn((1, 128, Z_IMAGE.cap_dim), generator=g, device="cuda")
    got = _np(model.forward(x, 0.5, cap))
    ref = rgpu.zimage_cuda(wts, heads=Z_IMAGE.heads)
    want = ref(x.cpu().numpy(), 0.5, cap.cpu().numpy())
    del ref, model, wts
    torch.cuda.empty_cache()
    assert rel_fro(got, want) <= 1e-2
