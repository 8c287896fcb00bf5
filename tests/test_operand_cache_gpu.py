"""GPU: the opt-in packed-operand cache (sdb200_set_operand_cache).

With the cache on, gemm_nt_f32 keeps the tf32-rounded copy of its B (the weights of the
reference's linear layers, tensor.cpp:481-501) and conv2d the [Cout, tap, Cin] slab of its
weights (tensor.cpp:529-586) across calls instead of repacking them every time. The results
must be bit-identical to the uncached path, each weight must be packed once, and an entry
must be dropped when its source buffer is overwritten through the library (upload, copy,
zero) or freed, so that a later call sees the new contents. A strided convolution, whose
internal GEMM takes the im2col scratch as B, must not use the cache.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture
def cache(sdb):
    L = sdb.lib()
    sdb.check(L.sdb200_set_operand_cache(0))
    yield L
    sdb.check(L.sdb200_set_operand_cache(0))
    assert L.sdb200_operand_cache_entries() == 0


def _dev_buffer(sdb, host):
    """A library-allocated device copy of a float32 numpy array."""
    L = sdb.lib()
    p = L.sdb200_malloc(host.nbytes)
    assert p
    sdb.check(L.sdb200_upload(p, host.ctypes.data_as(ctypes.c_void_p), host.nbytes))
    return p


def _run_gemm(sdb, A, Bp, M, N, K):
    import torch

    C = torch.empty((M, N), device="cuda")
    sdb.check(sdb.lib().sdb200_gemm_nt_f32(M, N, K, A.data_ptr(), K, Bp, K, C.data_ptr(), N, None, 0))
    torch.cuda.synchronize()
    return C.cpu().numpy()


def test_gemm_f32_weights_packed_once(sdb, cache):
    import torch

    L = cache
    M, N, K = 300, 640, 1000
    rng = np.random.default_rng(4)
    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    W = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    W2 = (0.02 * rng.standard_normal((N, K))).astype(np.float32)
    Bp = _dev_buffer(sdb, W)
    try:
        want = _run_gemm(sdb, A, Bp, M, N, K)  # cache off
        sdb.check(L.sdb200_set_operand_cache(1))
        first = _run_gemm(sdb, A, Bp, M, N, K)
        assert L.sdb200_operand_cache_entries() == 1
        second = _run_gemm(sdb, A, Bp, M, N, K)
        assert L.sdb200_operand_cache_entries() == 1
        assert np.array_equal(first, want) and np.array_equal(second, want)
        # new weights through the library: the stale pack is dropped, the result follows
        sdb.check(L.sdb200_upload(Bp, W2.ctypes.data_as(ctypes.c_void_p), W2.nbytes))
        assert L.sdb200_operand_cache_entries() == 0
        got2 = _run_gemm(sdb, A, Bp, M, N, K)
        sdb.check(L.sdb200_set_operand_cache(0))
        assert np.array_equal(got2, _run_gemm(sdb, A, Bp, M, N, K))
        sdb.check(L.sdb200_set_operand_cache(1))
        _run_gemm(sdb, A, Bp, M, N, K)
        sdb.check(L.sdb200_zero(Bp, 64))  # a partial overwrite drops it too
        assert L.sdb200_operand_cache_entries() == 0
        _run_gemm(sdb, A, Bp, M, N, K)
        assert L.sdb200_operand_cache_entries() == 1
    finally:
        sdb.check(L.sdb200_free(Bp))
    assert L.sdb200_operand_cache_entries() == 0  # freeing the weights drops their pack


def test_conv2d_weights_packed_once(sdb, cache):
    import torch

    L = cache
    N, Cin, H, W_, Cout = 2, 96, 24, 40, 128
    rng = np.random.default_rng(5)
    x = torch.from_numpy(rng.standard_normal((N, Cin, H, W_)).astype(np.float32)).cuda()
    w = (0.05 * rng.standard_normal((Cout, Cin, 3, 3))).astype(np.float32)
    w2 = (0.05 * rng.standard_normal((Cout, Cin, 3, 3))).astype(np.float32)
    b = torch.from_numpy((0.05 * rng.standard_normal(Cout)).astype(np.float32)).cuda()
    wp = _dev_buffer(sdb, w)
    src2 = _dev_buffer(sdb, w2)

    def conv(stride=1):
        Ho, Wo = (H + 2 - 3) // stride + 1, (W_ + 2 - 3) // stride + 1
        y = torch.empty((N, Cout, Ho, Wo), device="cuda")
        sdb.check(L.sdb200_conv2d(x.data_ptr(), N, Cin, H, W_, wp, Cout, 3, 3, b.data_ptr(), stride, 1,
                                  y.data_ptr(), Ho, Wo))
        torch.cuda.synchronize()
        return y.cpu().numpy()

    try:
        want, want_s2 = conv(), conv(2)
        sdb.check(L.sdb200_set_operand_cache(1))
        assert np.array_equal(conv(), want)
        assert L.sdb200_operand_cache_entries() == 1
        assert np.array_equal(conv(), want)
        assert L.sdb200_operand_cache_entries() == 1
        # stride 2 (im2col + GEMM over a scratch buffer, one image after another): not cached
        assert np.array_equal(conv(2), want_s2)
        assert L.sdb200_operand_cache_entries() == 1
        sdb.check(L.sdb200_copy(wp, src2, w2.nbytes))  # device-to-device overwrite
        assert L.sdb200_operand_cache_entries() == 0
        got2 = conv()
        sdb.check(L.sdb200_set_operand_cache(0))
        assert np.array_equal(got2, conv())
        assert not np.array_equal(got2, want)
    finally:
        sdb.check(L.sdb200_free(wp))
        sdb.check(L.sdb200_free(src2))
