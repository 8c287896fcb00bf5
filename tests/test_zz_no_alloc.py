"""GPU: sdb200_gemm_nt_bf16_noalloc, the GEMM entry point for callers that cannot
allocate device memory (a host framework that owns every device allocation through its
own pool, or a loop that must never reach a device-synchronising cudaMalloc / cudaFree).

It must give exactly the results of sdb200_gemm_nt_bf16 (the same kernels and the same
bf16 rounding of A) on consecutive calls that share its fixed scratch array, stay within
the bf16-weight GEMM gate of the CPU oracle, leave device free memory unchanged, report a
clean status word, and reject problems larger than the scratch. No sdb200 call precedes
the first no-alloc call here, so in a fresh process the first two calls also run without
a library device context. This file is collected last so that a failure here comes after
every other test has run.
"""
import ctypes

import numpy as np
import pytest

from conftest import rel_fro

pytestmark = pytest.mark.gpu

TOL_BF16 = 2e-3  # the bf16-weight GEMM gate of tests/test_gemm_gpu.py


def _inputs(rng, M, N, K):
    import torch

    from sdb200.workloads import f32_to_bf16_bits

    A = rng.standard_normal((M, K)).astype(np.float32)
    Wb = f32_to_bf16_bits((0.02 * rng.standard_normal((N, K))).astype(np.float32))
    bias = (0.01 * rng.standard_normal(N)).astype(np.float32)
    dev = (torch.from_numpy(A).cuda(), torch.from_numpy(Wb.view(np.int16)).cuda(), torch.from_numpy(bias).cuda())
    return (A, Wb, bias), dev


def _noalloc(L, sdb200, M, N, K, A, B, bias, Y):
    sdb200.check(L.sdb200_gemm_nt_bf16_noalloc(M, N, K, A.data_ptr(), K, B.data_ptr(), K, Y.data_ptr(), N,
                                               bias.data_ptr(), 0))


def _error_word(L, sdb200):
    w = ctypes.c_int(-1)
    sdb200.check(L.sdb200_device_error_word(ctypes.byref(w)))
    return w.value


def test_noalloc_matches_gemm_nt_bf16_on_consecutive_calls(orc):
    import torch

    import sdb200

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but torch sees no CUDA device")
    L = sdb200.lib()
    rng = np.random.default_rng(2024)
    # (1000, 1536, 640): ragged M; (4096, 2304, 3840): M * K = 15.7 Mi, near the 16 Mi
    # limit; (8, 3840, 256): M <= 16, the exact fp32-A kernel, no scratch used.
    shapes = [(1000, 1536, 640), (4096, 2304, 3840), (8, 3840, 256)]
    cases = []
    for M, N, K in shapes:
        host, (A, B, bias) = _inputs(rng, M, N, K)
        cases.append((M, N, K, host, A, B, bias, torch.empty((M, N), device="cuda"),
                      torch.empty((M, N), device="cuda")))
    torch.cuda.synchronize()

    # first call on this device: resolves the scratch address (set-up), then runs
    M, N, K, _, A, B, bias, Y, _ = cases[0]
    _noalloc(L, sdb200, M, N, K, A, B, bias, Y)
    torch.cuda.synchronize()

    # second call, larger shape, measured: device free memory must not move
    M, N, K, _, A, B, bias, Y, _ = cases[1]
    free_before, _ = torch.cuda.mem_get_info()
    _noalloc(L, sdb200, M, N, K, A, B, bias, Y)
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert free_after == free_before, "the no-alloc entry point changed device free memory"
    # the status of those two calls (no library context existed while they ran)
    assert _error_word(L, sdb200) == 0

    # third call: the small-M path
    M, N, K, _, A, B, bias, Y, _ = cases[2]
    _noalloc(L, sdb200, M, N, K, A, B, bias, Y)

    # the existing entry point on the same inputs: bit-identical outputs
    for M, N, K, _, A, B, bias, _, Yref in cases:
        sdb200.check(L.sdb200_gemm_nt_bf16(M, N, K, A.data_ptr(), K, B.data_ptr(), K, Yref.data_ptr(), N,
                                           bias.data_ptr(), 0))
    torch.cuda.synchronize()
    for M, N, K, (Ah, Wh, bh), _, _, _, Y, Yref in cases:
        got, want = Y.cpu().numpy(), Yref.cpu().numpy()
        assert np.isfinite(got).all()
        assert np.array_equal(got, want), (M, N, K, float(np.abs(got - want).max()))
        rows = np.arange(M) if M <= 1024 else np.random.default_rng(M).choice(M, 256, replace=False)
        assert rel_fro(got[rows], orc.gemm_nt_bf16(np.ascontiguousarray(Ah[rows]), Wh, bh)) <= TOL_BF16, (M, N, K)

    # repeat the first shape after the larger one: stale scratch contents do not leak in
    M, N, K, _, A, B, bias, Y, Yref = cases[0]
    Y.zero_()
    _noalloc(L, sdb200, M, N, K, A, B, bias, Y)
    torch.cuda.synchronize()
    assert torch.equal(Y, Yref)
    assert _error_word(L, sdb200) == 0
    sdb200.check(L.sdb200_synchronize())


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
