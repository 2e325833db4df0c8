"""Deterministic inputs of the golden tables (shared by make_golden.py and the tests)."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402


def tf32_all_patterns() -> np.ndarray:
    """Every TF32 sign / 8-bit exponent / 10-bit mantissa combination (2^19 words)."""
    v = np.arange(1 << 19, dtype=np.uint32)
    return ((v >> 18) << 31) | (((v >> 10) & 0xFF) << 23) | ((v & 0x3FF) << 13)


def tf32_random_words() -> np.ndarray:
    """32-bit words with arbitrary low mantissa bits (the decoder ignores or tests them)."""
    return np.random.default_rng(1234).integers(0, 1 << 32, size=16384, dtype=np.uint64).astype(np.uint32)


def quant_inputs() -> np.ndarray:
    """FP32 inputs for the quantizers: specials, every FP16 value, boundary sweeps, random bit patterns."""
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 448.0, -448.0, 449.0, 480.0, 464.0, 57344.0, 61440.0,
                         0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.5, 6.0, 7.0, 1e30, -1e30, 2.0 ** 27, 2.0 ** 26,
                         2.0 ** -6, 2.0 ** -7, 2.0 ** -9, 2.0 ** -10, 65504.0, 65520.0, 65536.0, 1e-8, -1e-8],
                        dtype=np.float32)
    halves = np.arange(65536, dtype=np.uint16).view(np.float16).astype(np.float32)
    rng = np.random.default_rng(99)
    bits = rng.integers(0, 1 << 32, size=32768, dtype=np.uint64).astype(np.uint32).view(np.float32)
    # Dense sweep over the E4M3 / FP4 ranges, where double rounding and ties live.
    sweep = np.linspace(-470.0, 470.0, 65537, dtype=np.float32)
    small = (rng.standard_normal(16384) * 0.05).astype(np.float32)
    return np.concatenate([specials, halves, bits, sweep, small]).astype(np.float32)


# Small weight-only GEMMs run through the reference's CPU path: name -> format.
GEMM_CASES = {
    "e4m3": oracle.E4M3, "e5m2": oracle.E5M2, "e2m1": oracle.E2M1, "e2m1u": oracle.E2M1_UNPACKED,
    "bf16": oracle.BF16, "tf32": oracle.TF32,
}


def gemm_case(name: str):
    """(fmt, A stored [M x K], B16 [N x K] FP16 bits, M, N, K, alpha) for a golden GEMM."""
    fmt = GEMM_CASES[name]
    M, N, K = 40, 24, 96
    a = oracle.uniform(7, (M, K))
    b = oracle.uniform(8, (N, K))
    scale = oracle.per_tensor_scale(a, fmt)
    A = oracle.quantize(fmt, a, scale)
    B16 = oracle.f32_to_f16_bits(b).reshape(N, K)
    return fmt, A, B16, M, N, K, float(np.float32(1.0) / np.float32(scale))
