"""Torch-facing wrappers of the C ABI, named after the reference backend API
(src/backend_cuda.h, namespace sd::cuda) and the tensor ops that call it
(src/tensor.h: linear, attention, rms_norm, ...).

Tensors are CUDA torch tensors used as plain device buffers: fp32 activations
(torch.float32) and bf16 weights (torch.bfloat16, whose bit pattern is the
reference's uint16 bf16). Every call goes through libsdb200.so on the current
device's stream; the wrappers bind that stream to torch's current stream first so
CUDA events recorded by torch order correctly with the library's kernels.
"""
from __future__ import annotations

import torch

from . import check, lib


def _p(t):
    return None if t is None else t.data_ptr()


def bind_stream(device=None) -> None:
    """Issues the library's ops for `device` on torch's current stream."""
    if device is not None:
        check(lib().sdb200_set_device(torch.device(device).index or 0))
    s = torch.cuda.current_stream()
    check(lib().sdb200_set_stream(s.cuda_stream))


def _need(t, dtype, name):
    if not t.is_cuda or t.dtype != dtype:
        raise TypeError(f"{name}: expected a CUDA {dtype} tensor, got {t.dtype} on {t.device}")


# ---------------------------------------------------------------------------------
# GEMM (backend_cuda.h:39-43)
# ---------------------------------------------------------------------------------
def gemm_nt_bf16(A, B, bias=None, C=None, accumulate=False, M=None, N=None, K=None, lda=None, ldb=None, ldc=None):
    """C[M,N] = A[M,K] B[N,K]^T (+bias) (+C): A fp32, B bf16. Returns C."""
    _need(A, torch.float32, "A")
    _need(B, torch.bfloat16, "B")
    M = A.shape[0] if M is None else M
    N = B.shape[0] if N is None else N
    K = A.shape[1] if K is None else K
    lda = A.stride(0) if lda is None else lda
    ldb = B.stride(0) if ldb is None else ldb
    if C is None:
        C = torch.empty((M, N), device=A.device, dtype=torch.float32)
    ldc = C.stride(0) if ldc is None else ldc
    bind_stream()
    check(lib().sdb200_gemm_nt_bf16(M, N, K, _p(A), lda, _p(B), ldb, _p(C), ldc, _p(bias), int(accumulate)))
    return C


def gemm_nt_bf16a(A, B, bias=None, C=None, accumulate=False):
    """Same with A already bf16."""
    _need(A, torch.bfloat16, "A")
    _need(B, torch.bfloat16, "B")
    M, K = A.shape
    N = B.shape[0]
    if C is None:
        C = torch.empty((M, N), device=A.device, dtype=torch.float32)
    bind_stream()
    check(lib().sdb200_gemm_nt_bf16a(M, N, K, _p(A), A.stride(0), _p(B), B.stride(0), _p(C), C.stride(0), _p(bias),
                                     int(accumulate)))
    return C


def gemm_nt_f32(A, B, bias=None, C=None, accumulate=False, M=None, N=None, K=None, lda=None, ldb=None, ldc=None):
    """C[M,N] = A[M,K] B[N,K]^T (+bias) (+C), fp32 weights (tf32 tensor cores)."""
    _need(A, torch.float32, "A")
    _need(B, torch.float32, "B")
    M = A.shape[0] if M is None else M
    N = B.shape[0] if N is None else N
    K = A.shape[1] if K is None else K
    lda = A.stride(0) if lda is None else lda
    ldb = B.stride(0) if ldb is None else ldb
    if C is None:
        C = torch.empty((M, N), device=A.device, dtype=torch.float32)
    ldc = C.stride(0) if ldc is None else ldc
    bind_stream()
    check(lib().sdb200_gemm_nt_f32(M, N, K, _p(A), lda, _p(B), ldb, _p(C), ldc, _p(bias), int(accumulate)))
    return C


def gemm_bf16_epilogue(A, B, bias=None, epi=0, y_bf16=False, Y=None):
    """Fused-epilogue GEMM: epi 0 plain, 1 SwiGLU, 2 GEGLU (B rows interleaved in
    blocks of 16, see interleave_gated). A fp32 or bf16."""
    a_bf16 = A.dtype == torch.bfloat16
    _need(B, torch.bfloat16, "B")
    M, K = A.shape
    N = B.shape[0]
    ncols = N if epi == 0 else N // 2
    if Y is None:
        Y = torch.empty((M, ncols), device=A.device, dtype=torch.bfloat16 if y_bf16 else torch.float32)
    bind_stream()
    check(lib().sdb200_gemm_bf16_epilogue(M, N, K, _p(A), A.stride(0), int(a_bf16), _p(B), B.stride(0), _p(Y),
                                          Y.stride(0), int(y_bf16), _p(bias), epi))
    return Y


def gemm_bf16_qkv_rope(X, Wqkv, cos, sin, gq=None, gk=None, bias=None, eps=1e-5):
    """Fused-QKV projection: X [M, K] (fp32 or bf16) times Wqkv [3 Dq, K] (bf16, rows
    q | k | v) (+bias), then the per-head RMS norm (gq / gk) and the interleaved rotary
    embedding (cos / sin [S, 128], row m uses m % S) of q and k. Returns fp16 (q, k, v),
    each [M, Dq]."""
    x_bf16 = X.dtype == torch.bfloat16
    _need(Wqkv, torch.bfloat16, "Wqkv")
    _need(cos, torch.float32, "cos")
    _need(sin, torch.float32, "sin")
    M, K = X.shape
    Dq = Wqkv.shape[0] // 3
    S = cos.shape[0]
    q, k, v = (torch.empty((M, Dq), device=X.device, dtype=torch.float16) for _ in range(3))
    bind_stream()
    check(lib().sdb200_gemm_bf16_qkv_rope(M, K, _p(X), X.stride(0), int(x_bf16), _p(Wqkv), Wqkv.stride(0), _p(bias),
                                          Dq, S, _p(cos), _p(sin), _p(gq), _p(gk), eps, _p(q), _p(k), _p(v)))
    return q, k, v


def interleave_gated(first, second, block=16):
    """Interleaves the rows of two [D, K] weights in blocks of `block`:
    rows [2jb, 2jb+b) from `first`, [2jb+b, 2jb+2b) from `second`. For SwiGLU
    first = gate (w1), second = up (w3); for GEGLU first = value, second = gate.
    Works on 1-D biases too."""
    D = first.shape[0]
    assert second.shape == first.shape and D % block == 0
    rest = first.shape[1:]
    f = first.reshape(D // block, block, *rest)
    s = second.reshape(D // block, block, *rest)
    return torch.stack([f, s], dim=1).reshape(2 * D, *rest).contiguous()


def linear(x, W, b=None):
    """tensor.cpp:481-501 linear(): flattens leading dims, bf16 or fp32 weights."""
    rows = x.numel() // x.shape[-1]
    x2 = x.reshape(rows, x.shape[-1])
    if W.dtype == torch.bfloat16:
        y = gemm_nt_bf16(x2, W, b)
    else:
        y = gemm_nt_f32(x2, W, b)
    return y.reshape(*x.shape[:-1], W.shape[0])


# ---------------------------------------------------------------------------------
# Attention and layers (backend_cuda.h:45-61)
# ---------------------------------------------------------------------------------
def attention(q, k, v, heads, causal=False, kv_heads=0):
    """tensor.cpp:776-810 attention(): q [N,Sq,heads*d], k/v [N,Skv,kv_heads*d]."""
    kv_heads = kv_heads or heads
    N, Sq, inner = q.shape
    Skv = k.shape[1]
    d = inner // heads
    out = torch.empty_like(q)
    bind_stream()
    check(lib().sdb200_attention(_p(q), _p(k), _p(v), _p(out), N, Sq, Skv, heads, kv_heads, d, int(causal)))
    return out


def rms_norm(x, gamma=None, eps=1e-5):
    y = torch.empty_like(x)
    C = x.shape[-1]
    bind_stream()
    check(lib().sdb200_rms_norm(_p(x), _p(y), x.numel() // C, C, _p(gamma), eps))
    return y


def layer_norm(x, gamma=None, beta=None, eps=1e-5):
    y = torch.empty_like(x)
    C = x.shape[-1]
    bind_stream()
    check(lib().sdb200_layer_norm(_p(x), _p(y), x.numel() // C, C, _p(gamma), _p(beta), eps))
    return y


def rms_norm_heads_(x, dim, gamma=None, eps=1e-5):
    bind_stream()
    check(lib().sdb200_rms_norm_heads(_p(x), x.numel() // dim, dim, _p(gamma), eps))
    return x


def rope_(x, dim, cos, sin, interleaved):
    N, S, inner = x.shape
    bind_stream()
    check(lib().sdb200_rope(_p(x), N, S, inner, dim, _p(cos), _p(sin), int(interleaved)))
    return x


def softmax_rows_(x, scale, causal=False):
    bind_stream()
    check(lib().sdb200_softmax_rows(_p(x), x.shape[0], x.shape[1], scale, int(causal)))
    return x


def swiglu(g, u):
    y = torch.empty_like(g)
    bind_stream()
    check(lib().sdb200_swiglu(_p(g), _p(u), _p(y), g.numel()))
    return y


def geglu(x):
    D2 = x.shape[-1]
    y = torch.empty(*x.shape[:-1], D2 // 2, device=x.device, dtype=torch.float32)
    bind_stream()
    check(lib().sdb200_geglu(_p(x), _p(y), x.numel() // D2, D2 // 2))
    return y


def group_norm(x, groups, gamma, beta, eps):
    N, C = x.shape[:2]
    y = torch.empty_like(x)
    bind_stream()
    check(lib().sdb200_group_norm(_p(x), _p(y), N, C, x.numel() // (N * C), groups, _p(gamma), _p(beta), eps))
    return y


def conv2d(x, w, bias, stride, pad):
    N, Cin, H, W = x.shape
    Cout, _, kh, kw = w.shape
    Ho = (H + 2 * pad - kh) // stride + 1
    Wo = (W + 2 * pad - kw) // stride + 1
    out = torch.empty((N, Cout, Ho, Wo), device=x.device, dtype=torch.float32)
    bind_stream()
    check(lib().sdb200_conv2d(_p(x), N, Cin, H, W, _p(w), Cout, kh, kw, _p(bias), stride, pad, _p(out), Ho, Wo))
    return out


def mul_rows_(x, v):
    bind_stream()
    check(lib().sdb200_mul_rows(_p(x), _p(v), x.numel() // v.numel(), v.numel()))
    return x


def add_rows_scaled_(x, y, g):
    bind_stream()
    check(lib().sdb200_add_rows_scaled(_p(x), _p(y), _p(g), x.numel() // g.numel(), g.numel()))
    return x


def unary_(name, x):
    bind_stream()
    check(getattr(lib(), "sdb200_" + name)(_p(x), x.numel()))
    return x


def synchronize():
    check(lib().sdb200_synchronize())


def device_error_word() -> int:
    import ctypes

    w = ctypes.c_int(0)
    check(lib().sdb200_device_error_word(ctypes.byref(w)))
    return w.value
