"""Seeded synthetic inputs of the BASELINE configurations (no datasets or checkpoints
exist here; shapes and distributions follow BASELINE.json's configs)."""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns, inf/NaN truncated: the
    reference's f32_to_bf16 (tensor.cpp:114-121) vectorised."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32)
    special = (b & 0x7F800000) == 0x7F800000
    r = ((b + np.uint32(0x7FFF) + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(special, (b >> 16).astype(np.uint16), r)


def cfg1_inputs(M=4096, N=11520, K=3840):
    """X [M,K] ~N(0,1), W [N,K] ~N(0,0.02), bias [N] ~N(0,0.01), one
    generator seeded 0, drawn in that order. W is returned in fp32; the GEMM uses its
    bf16 rounding (f32_to_bf16_bits)."""
    rng = np.random.default_rng(0)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = (0.02 * rng.standard_normal((N, K), dtype=np.float32)).astype(np.float32)
    b = (0.01 * rng.standard_normal(N, dtype=np.float32)).astype(np.float32)
    return X, W, b
