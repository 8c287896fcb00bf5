"""GPU: sdb200_gemm_nt_bf16_noalloc, the GEMM entry point for callers that cannot
allocate device memory (inside another party's graph capture, under a framework that
owns all device allocations, in loops that must not hit a synchronising cudaMalloc).

It must give the results of sdb200_gemm_nt_bf16 (same kernels) on consecutive calls
that share its fixed scratch array, leave device free memory unchanged, and reject
problems larger than the scratch. No sdb200 call precedes the first no-alloc call here,
so in a fresh process it also runs without a library device context.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-3  # the bf16-weight GEMM tolerance of tests/test_gemm_gpu.py


def _inputs(rng, M, N, K):
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    A = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    Wb = f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32))
    B = torch.from_numpy(Wb.view(np.int16)).cuda().view(torch.bfloat16)
    bias = torch.from_numpy((0.01 * rng.standard_normal(N)).astype(np.float32)).cuda()
    return A, B, bias


def test_noalloc_matches_gemm_nt_bf16_on_consecutive_calls():
    import torch

    import sdb200

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but torch sees no CUDA device")
    L = sdb200.lib()
    rng = np.random.default_rng(2024)
    shapes = [(1000, 1536, 640), (4096, 2304, 3840)]  # second: M * K = 15.7 Mi, near the 16 Mi limit
    cases = []
    for M, N, K in shapes:
        A, B, bias = _inputs(rng, M, N, K)
        cases.append((M, N, K, A, B, bias, torch.empty((M, N), device="cuda"), torch.empty((M, N), device="cuda")))
    torch.cuda.synchronize()

    # first call on this device: resolves the scratch address (set-up), then runs
    M, N, K, A, B, bias, Y, _ = cases[0]
    sdb200.check(L.sdb200_gemm_nt_bf16_noalloc(M, N, K, A.data_ptr(), K, B.data_ptr(), K, Y.data_ptr(), N,
                                               bias.data_ptr(), 0))
    torch.cuda.synchronize()

    # second call, larger shape, measured: device free memory must not move
    M2, N2, K2, A2, B2, bias2, Y2, _ = cases[1]
    free_before, _ = torch.cuda.mem_get_info()
    sdb200.check(L.sdb200_gemm_nt_bf16_noalloc(M2, N2, K2, A2.data_ptr(), K2, B2.data_ptr(), K2, Y2.data_ptr(), N2,
                                               bias2.data_ptr(), 0))
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, "the no-alloc entry point changed device free memory"

    # the existing entry point on the same inputs
    for M, N, K, A, B, bias, Y, Yref in cases:
        sdb200.check(L.sdb200_gemm_nt_bf16(M, N, K, A.data_ptr(), K, B.data_ptr(), K, Yref.data_ptr(), N,
                                           bias.data_ptr(), 0))
    torch.cuda.synchronize()
    for M, N, K, A, B, bias, Y, Yref in cases:
        got, want = Y.cpu().numpy(), Yref.cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_fro(got, want) <= TOL_BF16, (M, N, K)

    # repeat the first shape after the larger one: stale scratch contents do not leak in
    M, N, K, A, B, bias, Y, Yref = cases[0]
    Y.zero_()
    sdb200.check(L.sdb200_gemm_nt_bf16_noalloc(M, N, K, A.data_ptr(), K, B.data_ptr(), K, Y.data_ptr(), N,
                                               bias.data_ptr(), 0))
    torch.cuda.synchronize()
    assert rel_fro(Y.cpu().numpy(), Yref.cpu().numpy()) <= TOL_BF16
    w = ctypes.c_int(0)
    sdb200.check(L.sdb200_device_error_word(ctypes.byref(w)))
    assert w.value == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    import sdb200

    L = sdb200.lib()
    # 4097 x 4096 > 16 Mi elements: rejected on the host with a clear message
    rc = L.sdb200_gemm_nt_bf16_noalloc(4097, 64, 4096, 16, 4096, 16, 4096, 16, 64, None, 0)
    assert rc == sdb200.ERR_INVALID_ARG
    assert b"exceeds the fixed scratch" in L.sdb200_last_error()
    # B whose row pitch breaks TMA's 16-byte rule cannot be repacked without scratch
    rc = L.sdb200_gemm_nt_bf16_noalloc(64, 64, 100, 16, 100, 16, 100, 16, 64, None, 0)
    assert rc == sdb200.ERR_INVALID_ARG
