"""CPU: the C-ABI library loads, exports every entry point include/sdb200.h declares
and every sd::cuda symbol of the reference backend API (src/backend_cuda.h:24-80), and
rejects bad arguments on the host before touching a device. No compute call runs."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

HEADER = os.path.join(ROOT, "include", "sdb200.h")
LIB = os.path.join(PKG, "sdb200", "libsdb200.so")

# Every function of the reference's sd::cuda namespace (backend_cuda.h:24-80).
REFERENCE_API = [
    "available", "device_name", "device_memory", "malloc", "free", "upload", "download", "copy", "zero",
    "synchronize", "gemm_nt_f32", "gemm_nt_bf16", "conv2d", "group_norm", "layer_norm", "rms_norm",
    "rms_norm_heads", "rope", "softmax_rows", "attention", "geglu", "swiglu", "silu", "tanh", "gelu",
    "quick_gelu", "add", "scale", "affine", "mul_rows", "add_rows_scaled", "add_channel_bias",
    "upsample_nearest2x", "concat_channels", "nchw_to_nlc", "nlc_to_nchw", "patchify", "unpatchify",
]


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(sdb200_[a-z0-9_]+)\s*\(", text)))


def test_library_built():
    assert os.path.exists(LIB), "build with `make -C stablediffusion-cpp_b200`"


def test_exports_every_declared_symbol():
    lib = ctypes.CDLL(LIB)
    syms = declared_symbols()
    assert len(syms) >= 45
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing


def test_exports_reference_cpp_api():
    out = subprocess.run(["nm", "-DC", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    names = set(re.findall(r"sd::cuda::([a-z0-9_]+)\(", out))
    missing = [n for n in REFERENCE_API if n not in names]
    assert not missing, missing


def test_signature_of_drop_in_gemm():
    """The C++ symbols must carry the reference declarations exactly
    (backend_cuda.h:39-43, :58-59) for the Makefile link to resolve."""
    out = subprocess.run(["nm", "-DC", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    want = [
        "sd::cuda::gemm_nt_bf16(long, long, long, float const*, long, unsigned short const*, long, float*, long, "
        "float const*, bool)",
        "sd::cuda::gemm_nt_f32(long, long, long, float const*, long, float const*, long, float*, long, "
        "float const*, bool)",
        "sd::cuda::attention(float const*, float const*, float const*, float*, long, long, long, int, int, long, bool)",
        "sd::cuda::malloc(unsigned long)",
        "sd::cuda::download(void*, void const*, unsigned long)",
    ]
    for w in want:
        assert w in out, w


def test_host_validation_rejects_bad_args():
    import sdb200

    L = sdb200.lib()
    f = L.sdb200_gemm_nt_bf16
    # lda < K
    assert f(8, 8, 16, 1, 8, 1, 16, 1, 8, None, 0) == sdb200.ERR_INVALID_ARG
    assert b"lda < K" in L.sdb200_last_error()
    # ldc < N
    assert f(8, 8, 16, 1, 16, 1, 16, 1, 4, None, 0) == sdb200.ERR_INVALID_ARG
    # null C
    assert f(8, 8, 16, 1, 16, 1, 16, None, 8, None, 0) == sdb200.ERR_INVALID_ARG
    # K < 0
    assert L.sdb200_gemm_nt_f32(8, 8, -1, 1, 16, 1, 16, 1, 8, None, 0) == sdb200.ERR_INVALID_ARG
    # gated epilogue needs N % 32 == 0
    assert L.sdb200_gemm_bf16_epilogue(8, 48, 16, 1, 16, 0, 1, 16, 1, 24, 0, None, 1) == sdb200.ERR_INVALID_ARG
    # attention: heads not a multiple of kv_heads
    assert L.sdb200_attention(1, 1, 1, 1, 1, 4, 4, 3, 2, 8, 0) == sdb200.ERR_INVALID_ARG
    # M <= 0 is a no-op success, as in the reference (backend_cuda.cu:464)
    assert f(0, 8, 16, None, 16, None, 16, 1, 8, None, 0) == sdb200.OK
    # tensor-parallel barrier self-test: null flags, more than 8 ranks, rank outside the group,
    # and a misaligned flag array are refused before any device work
    assert L.sdb200_comm_barrier_selftest(None, 2, 0, 1) == sdb200.ERR_INVALID_ARG
    assert L.sdb200_comm_barrier_selftest(16, 9, 0, 1) == sdb200.ERR_INVALID_ARG
    assert L.sdb200_comm_barrier_selftest(16, 2, 2, 1) == sdb200.ERR_INVALID_ARG
    assert L.sdb200_comm_barrier_selftest(18, 2, 0, 1) == sdb200.ERR_INVALID_ARG
    # barrier choice on a null communicator
    assert L.sdb200_comm_set_barrier(None, 1) == sdb200.ERR_INVALID_ARG


def test_no_device_reports_unavailable():
    import torch

    import sdb200

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert sdb200.available() is False
    assert sdb200.lib().sdb200_device_name() == b""
